// Word-parallel AND-tree levels of the truth-table comparison gates, for the
// plans compiled into the level kernel (ot.cu).  Host and device, so that the
// logic can be checked on the CPU (tests/tt_lanes_check.cpp).
//
// The digit-share state of one element keeps 2 bits per digit (lt at 2g, eq
// at 2g + 1), as the level-1 table read writes it.  In the lane layout the
// combines never move their outputs down: combine i of a part at level l
// reads its L node at lane 2*base + i * 2^(l+1) and its H node 2^l bits above,
// and writes its output over the L node.  Every combine of a level therefore
// finds its two inputs at the same offsets from its lane, an odd top node is
// already where the next level looks for it, and the part roots stay at
// 2*base.  The openings of a level carry (e, f, f') of each combine at
// (lane, lane + 1, lane + 2); lanes are at least 4 apart, so a level's
// openings, the triple bits gathered to the lanes, and the closing logic each
// take one 32-bit word and a few word-wide operations for all its combines.
// The cross combine of the full-compare plans (H = the hi root at 0, L = the
// lo root) is alone at its level and uses lanes 0 (e) and 1 (f).
//
// Formulas (x ^ y: XOR; products: AND; p0 = 1 for party 0):
//   open:  e = eq_H ^ a,  f = lt_L ^ b,  f' = eq_L ^ b'
//   close: lt = lt_H ^ c ^ f a ^ e b ^ p0 e f,  eq = c' ^ f' a ^ e b' ^ p0 e f'
// with (a, b, b', c, c') the party's triple bits of the combine (5 bits at
// 5q of its triple words, c = a b, c' = a b' shared by the dealer).
#pragma once
#include <cstdint>
#include <type_traits>

#include "digit_plan.cuh"

namespace ddg {

template <int I, int END, class F>
__host__ __device__ __forceinline__ void static_for(const F &f)
{
    if constexpr (I < END) {
        f(std::integral_constant<int, I>{});
        static_for<I + 1, END>(f);
    }
}

// lane of combine q at level l (1-based) in the lane layout
__host__ __device__ constexpr int tt_lane(const OtPlan &P, int q, int l)
{
    return P.comb[q].part == 2 ? 0 : 2 * P.base[P.comb[q].part] + int(P.comb[q].out) * (2 << l);
}

// lanes of the combines of level l (eq_only: those that compute eq)
__host__ __device__ constexpr uint32_t tt_lane_mask(const OtPlan &P, int l, bool eq_only)
{
    uint32_t m = 0;
    if (l < 1 || l > P.levels) return 0;
    for (int q = P.lvl_first[l - 1]; q < P.lvl_first[l]; q++)
        if (!eq_only || P.comb[q].eq) m |= 1u << tt_lane(P, q, l);
    return m;
}

// bytes per element of the openings of level l (1..levels) in the compiled-in
// layouts: the smallest of 1, 2, 4 holding every opened bit (TT lanes: e, f,
// f' at lane, lane + 1, lane + 2; the cross combine: bits 0 and 1; OT: 3 bits
// per combine of the level from bit 0)
__host__ __device__ constexpr int open_width(const OtPlan &P, int l)
{
    if (l < 1 || l > P.levels) return 4;
    const int qa = P.lvl_first[l - 1], qb = P.lvl_first[l];
    uint64_t m = 0;
    if (P.mode == PLAN_OT) {
        m = (uint64_t(1) << (3 * (qb - qa))) - 1;
    } else if (qa < qb && P.comb[qa].part == 2) {
        m = 3;
    } else {
        const uint64_t a = tt_lane_mask(P, l, false), e = tt_lane_mask(P, l, true);
        m = a | (a << 1) | (e << 2);
    }
    return m < (uint64_t(1) << 8) ? 1 : m < (uint64_t(1) << 16) ? 2 : 4;
}

// bytes per element of the digit-share state in the compiled-in layouts: the
// truth-table modes keep it in 16 bits when their 2 bits per digit fit (the
// level kernels alone read and write it); the OT mode's garble step writes
// the plan's state_bytes()
__host__ __device__ constexpr int state_width(const OtPlan &P)
{
    return P.mode != PLAN_OT && 2 * P.D <= 16 ? 2 : P.state_bytes();
}

template <int W>
using open_word_t = typename std::conditional<W == 1, uint8_t, typename std::conditional<W == 2, uint16_t, uint32_t>::type>::type;

// the 5 triple bits at POS.. of the party's triple words (a combine's (a, b,
// b', c, c') where the plan keeps them contiguous)
template <int POS>
__host__ __device__ __forceinline__ uint32_t tri5(const uint32_t (&tw)[3])
{
    constexpr int b = POS, w = b / 32, sh = b % 32;
    // a packed group never straddles words; the 5q layout ends inside word 2
    if constexpr (sh + 5 <= 32 || w >= 2) {
        return (tw[w] >> sh) & 31u;
    } else {
        return ((tw[w] >> sh) | (tw[w + 1] << (32 - sh))) & 31u;
    }
}

// (a, b, b') of every combine of level L at lane, lane + 1, lane + 2 of one
// word: one shift and mask when the plan groups them (tpacked), else gathered
// combine by combine
template <int MODE, int NB, int SB, int L>
__host__ __device__ __forceinline__ uint32_t tt_gather3(const uint32_t (&tw)[3])
{
    constexpr OtPlan P = digit_plan(NB, SB, MODE);
    constexpr int qa = P.lvl_first[L - 1], qb = P.lvl_first[L];
    if constexpr (P.tpacked) {
        constexpr int g = P.tpa[qa] - tt_lane(P, qa, L);
        uint32_t m = 0;
        static_for<qa, qb>([&](auto qi) {
            constexpr OtPlan P = digit_plan(NB, SB, MODE);
            constexpr int q = decltype(qi)::value;
            m |= (P.comb[q].eq ? 7u : 3u) << tt_lane(P, q, L);
        });
        return (tw[g >> 5] >> (g & 31)) & m;
    } else {
        uint32_t t3 = 0;
        static_for<qa, qb>([&](auto qi) {
            constexpr OtPlan P = digit_plan(NB, SB, MODE);
            constexpr int q = decltype(qi)::value;
            t3 |= (tri5<P.tpa[q]>(tw) & 7u) << tt_lane(P, q, L);
        });
        return t3;
    }
}

// (c, c') of every combine of level L at lane, lane + 1
template <int MODE, int NB, int SB, int L>
__host__ __device__ __forceinline__ uint32_t tt_gather2(const uint32_t (&tw)[3])
{
    constexpr OtPlan P = digit_plan(NB, SB, MODE);
    constexpr int qa = P.lvl_first[L - 1], qb = P.lvl_first[L];
    if constexpr (P.tpacked) {
        constexpr int g = P.tpc[qa] - tt_lane(P, qa, L);
        uint32_t m = 0;
        static_for<qa, qb>([&](auto qi) {
            constexpr OtPlan P = digit_plan(NB, SB, MODE);
            constexpr int q = decltype(qi)::value;
            m |= (P.comb[q].eq ? 3u : 1u) << tt_lane(P, q, L);
        });
        return (tw[g >> 5] >> (g & 31)) & m;
    } else {
        uint32_t t2 = 0;
        static_for<qa, qb>([&](auto qi) {
            constexpr OtPlan P = digit_plan(NB, SB, MODE);
            constexpr int q = decltype(qi)::value;
            t2 |= (tri5<P.tpc[q]>(tw) & 3u) << tt_lane(P, q, L);
        });
        return t2;
    }
}

// openings of level L (1 <= L <= levels) from the state after level L - 1
template <int MODE, int NB, int SB, int L>
__host__ __device__ __forceinline__ uint32_t tt_open(uint32_t st, const uint32_t (&tw)[3])
{
    constexpr OtPlan P = digit_plan(NB, SB, MODE);
    constexpr int qa = P.lvl_first[L - 1], qb = P.lvl_first[L];
    if constexpr (qa >= qb) {
        return 0u;
    } else if constexpr (P.comb[qa].part == 2) {
        // the cross combine: e = eq of the hi root, f = lt of the lo root
        constexpr int lo = 2 * P.base[1];
        const uint32_t g = tri5<P.tpa[qa]>(tw);  // a, b at bits 0, 1
        return (((st >> 1) ^ g) & 1u) | ((((st >> lo) ^ (g >> 1)) & 1u) << 1);
    } else {
        const uint32_t t3 = tt_gather3<MODE, NB, SB, L>(tw);  // (a, b, b') of every combine at its lane
        constexpr uint32_t M = tt_lane_mask(P, L, false), Meq = tt_lane_mask(P, L, true);
        constexpr int S = 1 << L;  // the H node sits S bits above the lane
        const uint32_t e = (st >> (S + 1)) ^ t3;
        const uint32_t f = st ^ (t3 >> 1);
        const uint32_t f2 = (st >> 1) ^ (t3 >> 2);
        return (e & M) | ((f & M) << 1) | ((f2 & Meq) << 2);
    }
}

// close level L - 1 (2 <= L): O = both parties' openings of level L - 1, XORed
template <int MODE, int NB, int SB, int PARTY, int L>
__host__ __device__ __forceinline__ uint32_t tt_close(uint32_t st, const uint32_t (&tw)[3], uint32_t O)
{
    constexpr OtPlan P = digit_plan(NB, SB, MODE);
    constexpr int lf = L - 1;
    constexpr int qa = lf >= 1 ? P.lvl_first[lf - 1] : 0, qb = lf >= 1 ? P.lvl_first[lf] : 0;
    if constexpr (qa >= qb) {
        return st;
    } else if constexpr (P.comb[qa].part == 2) {
        const uint32_t g = tri5<P.tpa[qa]>(tw), c = tri5<P.tpc[qa]>(tw);  // a, b at bits 0, 1; c at bit 0
        const uint32_t e = O & 1u, f = (O >> 1) & 1u;
        uint32_t lt = (st ^ c ^ (f & g) ^ (e & (g >> 1))) & 1u;
        if constexpr (PARTY == 0) lt ^= e & f;
        return (st & ~3u) | lt;
    } else {
        // (a, b, b') and (c, c') of every combine at its lane
        const uint32_t t3 = tt_gather3<MODE, NB, SB, lf>(tw), t2 = tt_gather2<MODE, NB, SB, lf>(tw);
        constexpr uint32_t M = tt_lane_mask(P, lf, false), Meq = tt_lane_mask(P, lf, true);
        constexpr int S = 1 << lf;
        const uint32_t e = O, f = O >> 1, f2 = O >> 2;
        uint32_t lt = (st >> S) ^ t2 ^ (f & t3) ^ (e & (t3 >> 1));
        uint32_t eq = (t2 >> 1) ^ (f2 & t3) ^ (e & (t3 >> 2));
        if constexpr (PARTY == 0) lt ^= e & f, eq ^= e & f2;
        return (st & ~(M | (M << 1))) | (lt & M) | ((eq & Meq) << 1);
    }
}

}  // namespace ddg
