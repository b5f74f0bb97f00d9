// OT-leaf comparison gates: the evaluators' kernels (garble, AND-tree levels)
// and the dealer's part of the key (called from the gate keygen kernel).
// The protocol, the digit plan and the key layout are described in ot.cuh.
//
// Reference call sites replaced: DDGOrca::relu with the LSS backend switched
// on (DDG_LSS_RELU=1: gpu_mpc/lss/lss_online.cpp relu, lss_compare.cpp
// compare_gt / AND tree; bridged to the masked-public GPU pipeline as
// lss_protocol.md section 8 describes).
#include <mutex>
#include <type_traits>

#include "ot.cuh"
#include "tt_lanes.cuh"

namespace ddg {

// ---------------------------------------------------------------- host plan

const OtPlan &ot_plan_cached(int bw, int s)
{
    static OtPlan plans[2][64];
    static std::once_flag once;
    std::call_once(once, [] {
        for (int b = 0; b < 2; b++)
            for (int sc = 1; sc < 64; sc++) plans[b][sc] = ot_plan(b ? 64 : 32, sc);
    });
    return plans[bw == 64 ? 1 : 0][s > 0 && s < 64 ? s : 0];
}

AesKey ot_party_key(const AesKey &dk, uint32_t op, int party)
{
    const uint32_t in[4] = {uint32_t(party), 0u, op, P_OT_PARTY};
    uint32_t out[4];
    aes_encrypt_host(dk, in, out);
    uint8_t k[16];
    for (int i = 0; i < 16; i++) k[i] = uint8_t(out[i / 4] >> (8 * (i % 4)));
    AesKey r;
    aes_expand_host(k, r);
    return r;
}

// ---------------------------------------------------------------- device helpers

__device__ __forceinline__ uint32_t aux_bit(const Blk &a0, const Blk &a1, int i)
{
    return uint32_t(blk_bit(i < 128 ? a0 : a1, uint32_t(i & 127)));
}

template <typename ST>
__device__ __forceinline__ uint32_t st_bit(ST st, int i) { return uint32_t(st >> i) & 1u; }

// 32 bits of the concatenated aux blocks x0 || x1 from bit pos (pos + 32 <= 256)
__device__ __forceinline__ uint32_t aux_word(const Blk &x0, const Blk &x1, int pos)
{
    const int k = pos >> 5, r = pos & 31;
    auto w = [&](int i) { return i < 4 ? (i == 0 ? x0.w[0] : i == 1 ? x0.w[1] : i == 2 ? x0.w[2] : x0.w[3])
                                       : (i == 4 ? x1.w[0] : i == 5 ? x1.w[1] : i == 6 ? x1.w[2] : x1.w[3]); };
    const uint32_t lo = w(k), hi = k + 1 < 8 ? w(k + 1) : 0u;
    return r ? __funnelshift_r(lo, hi, uint32_t(r)) : lo;
}

// triple bit i (= 5q + field) of the stored triple words
__device__ __forceinline__ uint32_t tri_bit(const uint32_t (&t)[3], int i)
{
    const int k = i >> 5;
    return ((k == 0 ? t[0] : k == 1 ? t[1] : t[2]) >> (i & 31)) & 1u;
}

// the digit-share state: 32 bits when 2 D <= 32 (every specialised plan), else 64
template <typename ST>
__device__ __forceinline__ ST load_state(const void *state, uint64_t e)
{
    return static_cast<const ST *>(state)[e];
}
template <typename ST>
__device__ __forceinline__ void store_state(void *state, uint64_t e, ST st)
{
    static_cast<ST *>(state)[e] = st;
}
// the same with a 32-bit element index (compiled-in plans)
template <typename ST>
__device__ __forceinline__ ST load_state32(const void *state, uint32_t e)
{
    return static_cast<const ST *>(state)[e];
}
template <typename ST>
__device__ __forceinline__ void store_state32(void *state, uint32_t e, ST st)
{
    static_cast<ST *>(state)[e] = st;
}

// ---------------------------------------------------------------- garble

template <typename T>
struct OtGarbleArgs {
    OtPlan P;
    int party;
    uint64_t N;
    const T *xhat;
    const uint32_t *ks;  // the party's 44 round keys in its gate key
    uint32_t *tables;    // [local digit][N]
    void *state;         // [N] digit shares of the garbled digits (u32 or u64)
    uint32_t *tri;       // [tri_words][N] triple bits
};

// One element of party PARTY's first message.  With a compile-time plan every
// digit's shift, width and bit offsets are constants after unrolling.
template <int PARTY, typename ST, typename T, class E>
__device__ __forceinline__ void garble_elem(const E &A, const OtPlan &P, const OtGarbleArgs<T> &a, const uint32_t *rk,
                                            uint64_t e)
{
    const uint64_t N = a.N;
    const int G = P.garbled_by(PARTY), g0 = PARTY == 0 ? 0 : P.G0;
    const uint64_t x = uint64_t(__ldcs(a.xhat + e));
    const Blk x0 = A.prg(rk, 0, P_OT_AUX, e);
    Blk x1 = x0;
    if (P.naux > 1) x1 = A.prg(rk, 0, P_OT_AUX + 1, e);
    ST st = 0;
    Blk pad = x0;
#pragma unroll
    for (int t = 0; t < OT_MAX_DIGITS / 2; t++) {
        if (t >= G) break;
        if ((t & 3) == 0) pad = A.prg(rk, 0, P_OT_PAD + uint32_t(t >> 2), e);
        const int g = g0 + t, w = P.width(g);
        const uint32_t wm = (1u << w) - 1u;
        uint32_t delta = 0;
#pragma unroll
        for (int i = 0; i < 4; i++) delta |= aux_bit(x0, x1, 6 * t + i) << i;
        delta &= wm;
        const uint32_t slt = aux_bit(x0, x1, 6 * t + 4), seq = aux_bit(x0, x1, 6 * t + 5);
        const uint32_t xd = uint32_t(x >> P.shift(g)) & wm;
        const uint32_t pw = (t & 3) == 0 ? pad.w[0] : (t & 3) == 1 ? pad.w[1] : (t & 3) == 2 ? pad.w[2] : pad.w[3];
        __stcs(a.tables + uint64_t(t) * N + e, ot_table(xd, w, delta, slt, seq, pw));
        st |= (ST(slt) << (2 * g)) | (ST(seq) << (2 * g + 1));
    }
    store_state<ST>(a.state, e, st);
#pragma unroll
    for (int w = 0; w < 3; w++)
        if (w < P.tri_words()) a.tri[uint64_t(w) * N + e] = aux_word(x0, x1, P.tri0 + 32 * w);
}

// NB, SB: the (bw, scale) whose plan is compiled in; 0, 0 = the plan in the arguments
template <typename T, class E, int NB, int SB, int PARTY>
__global__ void __launch_bounds__(E::THREADS, E::CTAS) ot_garble_kernel(const __grid_constant__ OtGarbleArgs<T> a)
{
    extern __shared__ uint32_t smem_tab[];
    uint32_t *rk = smem_tab + E::SMEM / 4;
    E::stage(smem_tab);
    if (threadIdx.x < 44) rk[threadIdx.x] = a.ks[threadIdx.x];
    __syncthreads();
    E A(smem_tab);
    for (uint64_t e = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < a.N; e += uint64_t(gridDim.x) * blockDim.x) {
        if constexpr (NB != 0) {
            constexpr OtPlan P = ot_plan(NB, SB);
            static_assert(P.state_bytes() == 4, "compiled-in plans keep a 32-bit state");
            garble_elem<PARTY, uint32_t>(A, P, a, rk, e);
        } else if (a.P.state_bytes() == 4) {
            garble_elem<PARTY, uint32_t>(A, a.P, a, rk, e);
        } else {
            garble_elem<PARTY, uint64_t>(A, a.P, a, rk, e);
        }
    }
}

// ---------------------------------------------------------------- AND-tree levels

struct OtLevelArgs {
    OtPlan P;
    int party, level;  // level 1..levels+1
    uint64_t N, nw;
    const uint8_t *recv;         // OT level 1: the party's receiver records [slot][N]
    const uint32_t *peer_tables; // OT level 1: the peer's tables [slot][N]
    const uint32_t *c0;          // OT: party 0's explicit triple c bits [N]
    const void *xhat, *xhat2;    // TT level 1: the masked input (ring words; xhat2: its second addend or null)
    const uint32_t *tables;      // TT level 1: the party's digit truth-table rows [row][N]
    const void *open_own, *open_peer;  // level >= 2: the previous level's openings (ot_open_bytes each)
    void *state;
    const uint32_t *tri;         // [tri_words][N]
    void *open_out;              // level <= levels
    uint32_t *bits_hi, *bits_lo; // level == levels + 1: masked comparison bits (split-gate layout)
    int vec4;                    // compiled-in TT level 1: four elements per thread, 16-byte loads
};

// One element of party PARTY at AND-tree level l (see ot_level): returns the
// three masked output bits at the last level.
template <int PARTY, typename ST>
__device__ __forceinline__ void level_elem(const OtPlan &P, const OtLevelArgs &a, int l, uint64_t e, uint32_t &hl,
                                           uint32_t &he, uint32_t &ll)
{
    const uint64_t N = a.N;
    constexpr uint32_t p0 = PARTY == 0 ? 1u : 0u;
    const bool tt = P.mode != PLAN_OT;
    ST st = (tt && l == 1) ? ST(0) : load_state<ST>(a.state, e);
    uint32_t tw[3] = {0u, 0u, 0u};
#pragma unroll
    for (int w = 0; w < 3; w++)
        if (w < P.tri_words()) tw[w] = __ldcs(a.tri + uint64_t(w) * N + e);
    if (tt && l == 1) {
        // the party's share of every digit's (lt, eq): its table read at the public digit
        uint64_t x = P.n == 32 ? uint64_t(__ldcs(static_cast<const uint32_t *>(a.xhat) + e))
                               : __ldcs(static_cast<const unsigned long long *>(a.xhat) + e);
        if (a.xhat2)
            x = P.n == 32 ? uint64_t(uint32_t(x + __ldcs(static_cast<const uint32_t *>(a.xhat2) + e)))
                          : x + __ldcs(static_cast<const unsigned long long *>(a.xhat2) + e);
#pragma unroll
        for (int g = 0; g < OT_MAX_DIGITS; g++) {
            if (g >= P.D) break;
            const int w = P.width(g), W = 1 << w;
            const uint32_t xd = uint32_t(x >> P.shift(g)) & uint32_t(W - 1);
            const uint32_t *tb = a.tables + uint64_t(P.drow0(g)) * N + e;
            const uint32_t il = xd, ie = uint32_t(W) + xd;
            const uint32_t lt = (__ldcs(tb + uint64_t(il >> 5) * N) >> (il & 31)) & 1u;
            uint32_t eq = 0;
            if (P.deq(g)) eq = (__ldcs(tb + uint64_t(ie >> 5) * N) >> (ie & 31)) & 1u;
            st |= (ST(lt) << (2 * g)) | (ST(eq) << (2 * g + 1));
        }
    } else if (l == 1) {
        // shares of the digits the peer garbled: T[c] ^ k_c
        constexpr int q = 1 - PARTY;
        const int G = P.garbled_by(q), g0 = q == 0 ? 0 : P.G0;
#pragma unroll
        for (int t = 0; t < OT_MAX_DIGITS / 2; t++) {
            if (t >= G) break;
            const uint32_t rec = __ldcs(a.recv + uint64_t(t) * N + e);
            const uint32_t word = __ldcs(a.peer_tables + uint64_t(t) * N + e);
            const uint32_t c = rec & 15u;
            const uint32_t lt = ((word >> c) ^ (rec >> 4)) & 1u, eq = ((word >> (16 + c)) ^ (rec >> 5)) & 1u;
            const int g = g0 + t;
            st |= (ST(lt) << (2 * g)) | (ST(eq) << (2 * g + 1));
        }
    } else {
        // close level l - 1: z = c ^ f a ^ e b ^ [p = 0] e f
        const uint32_t O = __ldcs(static_cast<const uint32_t *>(a.open_own) + e) ^
                           __ldcs(static_cast<const uint32_t *>(a.open_peer) + e);
        const bool cword = !tt && PARTY == 0;  // OT party 0 keeps its triple c bits in a key word
        const uint32_t cw = cword ? __ldcs(a.c0 + e) : 0u;
        const int qa = P.lvl_first[l - 2];
#pragma unroll
        for (int q = 0; q < OT_MAX_COMB; q++) {
            if (q >= P.ncomb) break;
            if (P.level_of(q) != l - 1) continue;
            const OtComb &C = P.comb[q];
            const int j = q - qa;
            const uint32_t eo = (O >> (3 * j)) & 1u, f = (O >> (3 * j + 1)) & 1u, f2 = (O >> (3 * j + 2)) & 1u;
            const uint32_t ta = tri_bit(tw, P.tpos(q, 0)), tb1 = tri_bit(tw, P.tpos(q, 1)),
                           tb2 = tri_bit(tw, P.tpos(q, 2));
            const uint32_t c = cword ? (cw >> (2 * q)) & 1u : tri_bit(tw, P.tpos(q, 3));
            const uint32_t c2 = cword ? (cw >> (2 * q + 1)) & 1u : tri_bit(tw, P.tpos(q, 4));
            const uint32_t lt = st_bit(st, P.hpos(q)) ^ c ^ (f & ta) ^ (eo & tb1) ^ (p0 & eo & f);
            const uint32_t eq = C.eq ? (c2 ^ (f2 & ta) ^ (eo & tb2) ^ (p0 & eo & f2)) : 0u;
            const int o = P.opos(q);
            st = (st & ~(ST(3) << o)) | (ST(lt) << o) | (ST(eq) << (o + 1));
        }
#pragma unroll
        for (int pt = 0; pt < 2; pt++) {
            const int from = P.pass_from[l - 1][pt];
            if (from >= 0) {
                const int b = 2 * P.base[pt], o = b + 2 * P.pass_to[l - 1][pt];
                const ST v = (st >> (b + 2 * from)) & ST(3);
                st = (st & ~(ST(3) << o)) | (v << o);
            }
        }
    }
    if (l <= P.levels) {
        // open level l: e = eq_H ^ a, f = lt_L ^ b, f' = eq_L ^ b'
        uint32_t w = 0;
        const int qa = P.lvl_first[l - 1];
#pragma unroll
        for (int q = 0; q < OT_MAX_COMB; q++) {
            if (q >= P.ncomb) break;
            if (P.level_of(q) != l) continue;
            const OtComb &C = P.comb[q];
            const int j = q - qa;
            const uint32_t eH = st_bit(st, P.hpos(q) + 1), lL = st_bit(st, P.lpos(q)), eL = st_bit(st, P.lpos(q) + 1);
            w |= ((eH ^ tri_bit(tw, P.tpos(q, 0))) << (3 * j)) | ((lL ^ tri_bit(tw, P.tpos(q, 1))) << (3 * j + 1));
            if (C.eq) w |= (eL ^ tri_bit(tw, P.tpos(q, 2))) << (3 * j + 2);
        }
        static_cast<uint32_t *>(a.open_out)[e] = w;
        store_state<ST>(a.state, e, st);
    } else {
        if (P.nd[0]) hl = st_bit(st, 0), he = st_bit(st, 1);
        ll = st_bit(st, 2 * P.base[1]);
        if (P.mode == PLAN_TT_FULL) ll ^= tri_bit(tw, P.mu_bit());  // the lo compare's mask share
    }
}

// ---- the same step with the plan compiled in.  Every digit, combine and
// pass is visited by a compile-time loop (static_for, tt_lanes.cuh), and plan
// fields are read only into constexpr locals, so no plan object exists at run
// time (a constexpr plan object indexed from unrolled loops ended up in local
// memory).  The truth-table modes close and open their AND levels with the
// word-parallel lane layout of tt_lanes.cuh; the OT mode keeps the per-combine
// form of level_elem.  Both parties and every level of a gate run the same
// compiled-in plan (level_launch covers levels 1..6), so the two layouts never
// meet.
template <int MODE, int NB, int SB, int PARTY, int L>
__device__ __forceinline__ void level_elem_c(const OtLevelArgs &a, uint32_t e, uint32_t N, uint32_t &hl,
                                             uint32_t &he, uint32_t &ll)
{
    constexpr OtPlan P = digit_plan(NB, SB, MODE);
    static_assert(P.ok && P.state_bytes() == 4, "compiled-in plans keep a 32-bit state");
    constexpr bool TT = MODE != PLAN_OT;
    constexpr uint32_t p0 = PARTY == 0 ? 1u : 0u;
    // openings read (level L - 1) and written (level L), each in its own width
    using OI = open_word_t<open_width(P, L - 1)>;
    using OO = open_word_t<open_width(P, L)>;
    using SW = open_word_t<state_width(P)>;
    auto open_in = [&]() {
        return uint32_t(__ldcs(static_cast<const OI *>(a.open_own) + e)) ^
               uint32_t(__ldcs(static_cast<const OI *>(a.open_peer) + e));
    };
    uint32_t st = 0;
    if constexpr (!(TT && L == 1)) st = uint32_t(load_state32<SW>(a.state, e));
    uint32_t tw[3] = {0u, 0u, 0u};
    static_for<0, P.tri_words()>([&](auto wi) {
        constexpr int w = decltype(wi)::value;
        tw[w] = __ldcs(a.tri + (uint32_t(w) * N + e));
    });
    auto tbit = [&](int i) { return (tw[i >> 5] >> (i & 31)) & 1u; };
    if constexpr (TT && L == 1) {
        uint64_t x;
        if constexpr (NB == 32) {
            uint32_t x32 = __ldcs(static_cast<const uint32_t *>(a.xhat) + e);
            if (a.xhat2) x32 += __ldcs(static_cast<const uint32_t *>(a.xhat2) + e);
            x = x32;
        } else {
            x = __ldcs(static_cast<const unsigned long long *>(a.xhat) + e);
            if (a.xhat2) x += __ldcs(static_cast<const unsigned long long *>(a.xhat2) + e);
        }
        static_for<0, P.D>([&](auto gi) {
            constexpr OtPlan P = digit_plan(NB, SB, MODE);
            constexpr int g = decltype(gi)::value;
            constexpr int W = 1 << P.width(g), sh = P.shift(g), r0 = P.drow0(g);
            constexpr bool deq = P.deq(g) != 0;
            const uint32_t xd = uint32_t(x >> sh) & uint32_t(W - 1);
            const uint32_t *tb = a.tables + (uint32_t(r0) * N + e);
            const uint32_t ie = uint32_t(W) + xd;
            uint32_t lt, eq = 0;
            if constexpr (W <= 32) {
                lt = (__ldcs(tb) >> xd) & 1u;
                if constexpr (deq) eq = (__ldcs(tb + (ie >> 5) * N) >> (ie & 31)) & 1u;
            } else {
                lt = (__ldcs(tb + (xd >> 5) * N) >> (xd & 31)) & 1u;
                if constexpr (deq) eq = (__ldcs(tb + (ie >> 5) * N) >> (ie & 31)) & 1u;
            }
            st |= (lt << (2 * g)) | (eq << (2 * g + 1));
        });
    } else if constexpr (L == 1) {
        constexpr int q = 1 - PARTY;
        constexpr int G = P.garbled_by(q), g0 = q == 0 ? 0 : P.G0;
        static_for<0, G>([&](auto ti) {
            constexpr int t = decltype(ti)::value;
            const uint32_t rec = __ldcs(a.recv + (uint32_t(t) * N + e));
            const uint32_t word = __ldcs(a.peer_tables + (uint32_t(t) * N + e));
            const uint32_t c = rec & 15u;
            const uint32_t lt = ((word >> c) ^ (rec >> 4)) & 1u, eq = ((word >> (16 + c)) ^ (rec >> 5)) & 1u;
            st |= (lt << (2 * (g0 + t))) | (eq << (2 * (g0 + t) + 1));
        });
    } else if constexpr (TT) {
        const uint32_t O = open_in();
        st = tt_close<MODE, NB, SB, PARTY, L>(st, tw, O);
    } else {
        const uint32_t O = open_in();
        constexpr bool cword = !TT && PARTY == 0;
        const uint32_t cw = cword ? __ldcs(a.c0 + e) : 0u;
        constexpr int qa = P.lvl_first[L - 2], qb = P.lvl_first[L - 1];
        static_for<qa, qb>([&](auto qi) {
            constexpr OtPlan P = digit_plan(NB, SB, MODE);
            constexpr int q = decltype(qi)::value;
            constexpr int j = q - qa, h = P.hpos(q), o = P.opos(q);
            constexpr bool ceq = P.comb[q].eq != 0;
            const uint32_t eo = (O >> (3 * j)) & 1u, f = (O >> (3 * j + 1)) & 1u, f2 = (O >> (3 * j + 2)) & 1u;
            const uint32_t ta = tbit(P.tpos(q, 0)), tb1 = tbit(P.tpos(q, 1)), tb2 = tbit(P.tpos(q, 2));
            const uint32_t c = cword ? (cw >> (2 * q)) & 1u : tbit(P.tpos(q, 3));
            const uint32_t c2 = cword ? (cw >> (2 * q + 1)) & 1u : tbit(P.tpos(q, 4));
            const uint32_t lt = ((st >> h) & 1u) ^ c ^ (f & ta) ^ (eo & tb1) ^ (p0 & eo & f);
            const uint32_t eq = ceq ? (c2 ^ (f2 & ta) ^ (eo & tb2) ^ (p0 & eo & f2)) : 0u;
            st = (st & ~(3u << o)) | (lt << o) | (eq << (o + 1));
        });
        static_for<0, 2>([&](auto pi) {
            constexpr OtPlan P = digit_plan(NB, SB, MODE);
            constexpr int pt = decltype(pi)::value;
            constexpr int from = P.pass_from[L - 1][pt];
            if constexpr (from >= 0) {
                constexpr int b = 2 * P.base[pt], o = b + 2 * P.pass_to[L - 1][pt];
                const uint32_t v = (st >> (b + 2 * from)) & 3u;
                st = (st & ~(3u << o)) | (v << o);
            }
        });
    }
    if constexpr (TT && L <= P.levels) {
        static_cast<OO *>(a.open_out)[e] = OO(tt_open<MODE, NB, SB, L>(st, tw));
        store_state32<SW>(a.state, e, SW(st));
    } else if constexpr (L <= P.levels) {
        uint32_t w = 0;
        constexpr int qa = P.lvl_first[L - 1], qb = P.lvl_first[L];
        static_for<qa, qb>([&](auto qi) {
            constexpr OtPlan P = digit_plan(NB, SB, MODE);
            constexpr int q = decltype(qi)::value;
            constexpr int j = q - qa, hb = P.hpos(q), lb = P.lpos(q);
            const uint32_t eH = (st >> (hb + 1)) & 1u, lL = (st >> lb) & 1u, eL = (st >> (lb + 1)) & 1u;
            w |= ((eH ^ tbit(P.tpos(q, 0))) << (3 * j)) | ((lL ^ tbit(P.tpos(q, 1))) << (3 * j + 1));
            if constexpr (P.comb[q].eq != 0) w |= (eL ^ tbit(P.tpos(q, 2))) << (3 * j + 2);
        });
        static_cast<OO *>(a.open_out)[e] = OO(w);
        store_state32<SW>(a.state, e, SW(st));
    } else {
        if constexpr (P.nd[0] != 0) hl = st & 1u, he = (st >> 1) & 1u;
        ll = (st >> (2 * P.base[1])) & 1u;
        if constexpr (MODE == PLAN_TT_FULL) ll ^= tbit(P.mu_bit());  // the lo compare's mask share
    }
}

// word j of a 16-byte vector
__device__ __forceinline__ uint32_t lane4(const uint4 &v, int j) { return j == 0 ? v.x : j == 1 ? v.y : j == 2 ? v.z : v.w; }

// word j of row `row` (run-time, < NR) of the rows loaded for a digit
template <int NR>
__device__ __forceinline__ uint32_t row_word(const uint4 (&rv)[NR], uint32_t row, int j)
{
    uint32_t w = lane4(rv[0], j);
    static_for<1, NR>([&](auto ki) {
        constexpr int k = decltype(ki)::value;
        if (row == uint32_t(k)) w = lane4(rv[k], j);
    });
    return w;
}

// Truth-table level 1 of a compiled-in plan for four consecutive elements
// e..e+3 (e % 4 == 0): every key row, the triple words and x_hat (+ its second
// addend) as 16-byte loads (512 contiguous bytes per row and warp instead of
// 128), the same digit reads, state and openings as level_elem_c, the
// openings and state stored as one vector each.  ot_level takes it when N is
// a multiple of 4 and every array is 16-byte aligned.
template <int MODE, int NB, int SB, int PARTY>
__device__ __forceinline__ void level1_tt_x4(const OtLevelArgs &a, uint32_t e, uint32_t N)
{
    constexpr OtPlan P = digit_plan(NB, SB, MODE);
    using OO = open_word_t<open_width(P, 1)>;
    using SW = open_word_t<state_width(P)>;
    uint32_t tw[4][3] = {{0u, 0u, 0u}, {0u, 0u, 0u}, {0u, 0u, 0u}, {0u, 0u, 0u}};
    static_for<0, P.tri_words()>([&](auto wi) {
        constexpr int w = decltype(wi)::value;
        const uint4 v = __ldcs(reinterpret_cast<const uint4 *>(a.tri + (uint32_t(w) * N + e)));
        tw[0][w] = v.x, tw[1][w] = v.y, tw[2][w] = v.z, tw[3][w] = v.w;
    });
    uint64_t x[4];
    if constexpr (NB == 32) {
        uint4 v = __ldcs(reinterpret_cast<const uint4 *>(static_cast<const uint32_t *>(a.xhat) + e));
        if (a.xhat2) {
            const uint4 w = __ldcs(reinterpret_cast<const uint4 *>(static_cast<const uint32_t *>(a.xhat2) + e));
            v.x += w.x, v.y += w.y, v.z += w.z, v.w += w.w;
        }
        x[0] = v.x, x[1] = v.y, x[2] = v.z, x[3] = v.w;
    } else {
        const ulonglong2 *p = reinterpret_cast<const ulonglong2 *>(static_cast<const unsigned long long *>(a.xhat) + e);
        ulonglong2 v0 = __ldcs(p), v1 = __ldcs(p + 1);
        if (a.xhat2) {
            const ulonglong2 *q =
                reinterpret_cast<const ulonglong2 *>(static_cast<const unsigned long long *>(a.xhat2) + e);
            const ulonglong2 w0 = __ldcs(q), w1 = __ldcs(q + 1);
            v0.x += w0.x, v0.y += w0.y, v1.x += w1.x, v1.y += w1.y;
        }
        x[0] = v0.x, x[1] = v0.y, x[2] = v1.x, x[3] = v1.y;
    }
    uint32_t st[4] = {0u, 0u, 0u, 0u};
    static_for<0, P.D>([&](auto gi) {
        constexpr OtPlan P = digit_plan(NB, SB, MODE);
        constexpr int g = decltype(gi)::value;
        constexpr int W = 1 << P.width(g), sh = P.shift(g), r0 = P.drow0(g), nr = P.drows(g);
        constexpr bool deq = P.deq(g) != 0;
        uint4 rv[nr];
        static_for<0, nr>([&](auto ki) {
            constexpr int k = decltype(ki)::value;
            rv[k] = __ldcs(reinterpret_cast<const uint4 *>(a.tables + (uint32_t(r0 + k) * N + e)));
        });
        static_for<0, 4>([&](auto ji) {
            constexpr int j = decltype(ji)::value;
            const uint32_t xd = uint32_t(x[j] >> sh) & uint32_t(W - 1);
            const uint32_t ie = uint32_t(W) + xd;
            uint32_t lt, eq = 0;
            if constexpr (W <= 32) {
                lt = (lane4(rv[0], j) >> xd) & 1u;
                if constexpr (deq) eq = (lane4(rv[W == 32 ? 1 : 0], j) >> (ie & 31)) & 1u;
            } else {
                lt = (row_word<nr>(rv, xd >> 5, j) >> (xd & 31)) & 1u;
                if constexpr (deq) eq = (row_word<nr>(rv, ie >> 5, j) >> (ie & 31)) & 1u;
            }
            st[j] |= (lt << (2 * g)) | (eq << (2 * g + 1));
        });
    });
    uint32_t o[4];
    static_for<0, 4>([&](auto ji) {
        constexpr int j = decltype(ji)::value;
        o[j] = tt_open<MODE, NB, SB, 1>(st[j], tw[j]);
    });
    if constexpr (sizeof(OO) == 1) {
        *reinterpret_cast<uint32_t *>(static_cast<uint8_t *>(a.open_out) + e) =
            (o[0] & 0xffu) | ((o[1] & 0xffu) << 8) | ((o[2] & 0xffu) << 16) | ((o[3] & 0xffu) << 24);
    } else if constexpr (sizeof(OO) == 2) {
        *reinterpret_cast<uint2 *>(static_cast<uint16_t *>(a.open_out) + e) =
            make_uint2((o[0] & 0xffffu) | ((o[1] & 0xffffu) << 16), (o[2] & 0xffffu) | ((o[3] & 0xffffu) << 16));
    } else {
        *reinterpret_cast<uint4 *>(static_cast<uint32_t *>(a.open_out) + e) = make_uint4(o[0], o[1], o[2], o[3]);
    }
    if constexpr (sizeof(SW) == 2) {
        *reinterpret_cast<uint2 *>(static_cast<uint16_t *>(a.state) + e) =
            make_uint2((st[0] & 0xffffu) | ((st[1] & 0xffffu) << 16), (st[2] & 0xffffu) | ((st[3] & 0xffffu) << 16));
    } else {
        *reinterpret_cast<uint4 *>(static_cast<uint32_t *>(a.state) + e) = make_uint4(st[0], st[1], st[2], st[3]);
    }
}

// Truth-table levels 2..levels+1 of a compiled-in plan for four consecutive
// elements e..e+3 (e % 4 == 0, all four below N): the triple words, the state
// and both parties' openings of level L - 1 as vector loads, the closing and
// opening of level_elem_c per element, the state and openings stored as one
// vector each.  At the last level it returns the elements' masked comparison
// bits as nibbles (bit j = element e + j) for the caller to gather per word.
template <int MODE, int NB, int SB, int PARTY, int L>
__device__ __forceinline__ void levelN_tt_x4(const OtLevelArgs &a, uint32_t e, uint32_t N, uint32_t &nh,
                                             uint32_t &ne, uint32_t &nl)
{
    constexpr OtPlan P = digit_plan(NB, SB, MODE);
    using OI = open_word_t<open_width(P, L - 1)>;
    using OO = open_word_t<open_width(P, L)>;
    using SW = open_word_t<state_width(P)>;
    uint32_t tw[4][3] = {{0u, 0u, 0u}, {0u, 0u, 0u}, {0u, 0u, 0u}, {0u, 0u, 0u}};
    static_for<0, P.tri_words()>([&](auto wi) {
        constexpr int w = decltype(wi)::value;
        const uint4 v = __ldcs(reinterpret_cast<const uint4 *>(a.tri + (uint32_t(w) * N + e)));
        tw[0][w] = v.x, tw[1][w] = v.y, tw[2][w] = v.z, tw[3][w] = v.w;
    });
    // four narrow words as their 4, 8 or 16 bytes
    auto ld4 = [&](const void *base, auto tag, uint32_t (&out)[4]) {
        using U = decltype(tag);
        if constexpr (sizeof(U) == 1) {
            const uint32_t v = __ldcs(reinterpret_cast<const uint32_t *>(static_cast<const uint8_t *>(base) + e));
            out[0] = v & 0xffu, out[1] = (v >> 8) & 0xffu, out[2] = (v >> 16) & 0xffu, out[3] = v >> 24;
        } else if constexpr (sizeof(U) == 2) {
            const uint2 v = __ldcs(reinterpret_cast<const uint2 *>(static_cast<const uint16_t *>(base) + e));
            out[0] = v.x & 0xffffu, out[1] = v.x >> 16, out[2] = v.y & 0xffffu, out[3] = v.y >> 16;
        } else {
            const uint4 v = __ldcs(reinterpret_cast<const uint4 *>(static_cast<const uint32_t *>(base) + e));
            out[0] = v.x, out[1] = v.y, out[2] = v.z, out[3] = v.w;
        }
    };
    auto st4 = [&](void *base, auto tag, const uint32_t (&in)[4]) {
        using U = decltype(tag);
        if constexpr (sizeof(U) == 1) {
            *reinterpret_cast<uint32_t *>(static_cast<uint8_t *>(base) + e) =
                (in[0] & 0xffu) | ((in[1] & 0xffu) << 8) | ((in[2] & 0xffu) << 16) | ((in[3] & 0xffu) << 24);
        } else if constexpr (sizeof(U) == 2) {
            *reinterpret_cast<uint2 *>(static_cast<uint16_t *>(base) + e) =
                make_uint2((in[0] & 0xffffu) | ((in[1] & 0xffffu) << 16), (in[2] & 0xffffu) | ((in[3] & 0xffffu) << 16));
        } else {
            *reinterpret_cast<uint4 *>(static_cast<uint32_t *>(base) + e) = make_uint4(in[0], in[1], in[2], in[3]);
        }
    };
    uint32_t st[4], oo[4], op[4];
    ld4(a.state, SW{}, st);
    ld4(a.open_own, OI{}, oo);
    ld4(a.open_peer, OI{}, op);
    static_for<0, 4>([&](auto ji) {
        constexpr int j = decltype(ji)::value;
        st[j] = tt_close<MODE, NB, SB, PARTY, L>(st[j], tw[j], oo[j] ^ op[j]);
    });
    if constexpr (L <= P.levels) {
        uint32_t o[4];
        static_for<0, 4>([&](auto ji) {
            constexpr int j = decltype(ji)::value;
            o[j] = tt_open<MODE, NB, SB, L>(st[j], tw[j]);
        });
        st4(a.open_out, OO{}, o);
        st4(a.state, SW{}, st);
        nh = ne = nl = 0u;
    } else {
        nh = ne = nl = 0u;
        static_for<0, 4>([&](auto ji) {
            constexpr OtPlan P = digit_plan(NB, SB, MODE);
            constexpr int j = decltype(ji)::value;
            uint32_t ll = (st[j] >> (2 * P.base[1])) & 1u;
            if constexpr (MODE == PLAN_TT_FULL) ll ^= (tw[j][P.mu_bit() >> 5] >> (P.mu_bit() & 31)) & 1u;
            if constexpr (P.nd[0] != 0) nh |= (st[j] & 1u) << j, ne |= ((st[j] >> 1) & 1u) << j;
            nl |= ll << j;
        });
    }
}

// MODE, NB, SB: the plan compiled in (NB = 0: the plan in the arguments);
// LV: the level compiled in (0 = a.level)
template <int MODE, int NB, int SB, int PARTY, int LV>
__global__ void ot_level_kernel(const __grid_constant__ OtLevelArgs a)
{
    if constexpr (NB != 0 && LV == 1 && MODE != PLAN_OT) {
        if (a.vec4) {
            const uint32_t N = uint32_t(a.N), nq = N / 4, stride = gridDim.x * blockDim.x;
            for (uint32_t q = blockIdx.x * blockDim.x + threadIdx.x; q < nq; q += stride)
                level1_tt_x4<MODE, NB, SB, PARTY>(a, 4 * q, N);
            return;
        }
    }
    if constexpr (NB != 0 && LV >= 2 && MODE != PLAN_OT) {
        if (a.vec4) {
            constexpr bool last = LV > digit_plan(NB, SB, MODE).levels;
            const uint32_t N = uint32_t(a.N), nq = N / 4, stride = gridDim.x * blockDim.x;
            // the last level gathers a word of bits from eight lanes: whole warps step together
            const uint32_t qend = last ? (nq + 31u) & ~31u : nq;
            for (uint32_t q = blockIdx.x * blockDim.x + threadIdx.x; q < qend; q += stride) {
                uint32_t nh = 0, ne = 0, nl = 0;
                if (q < nq) levelN_tt_x4<MODE, NB, SB, PARTY, LV>(a, 4 * q, N, nh, ne, nl);
                if constexpr (last) {
                    // word q / 8 holds elements 32 (q / 8) .. +31: lane q % 8 of each group of eight gives 4 bits
                    const int sh = 4 * int(threadIdx.x & 7);
                    uint32_t wh = nh << sh, we = ne << sh, wl = nl << sh;
#pragma unroll
                    for (int m = 1; m < 8; m <<= 1) {
                        wh |= __shfl_xor_sync(0xFFFFFFFFu, wh, m);
                        we |= __shfl_xor_sync(0xFFFFFFFFu, we, m);
                        wl |= __shfl_xor_sync(0xFFFFFFFFu, wl, m);
                    }
                    const uint32_t wi = q >> 3;
                    if ((threadIdx.x & 7) == 0 && uint64_t(wi) * 32 < N) {
                        if (a.bits_hi) {
                            a.bits_hi[wi] = wh;
                            if constexpr (MODE != PLAN_TT_FULL) a.bits_hi[uint32_t(a.nw) + wi] = we;
                        }
                        a.bits_lo[wi] = wl;
                    }
                }
            }
            return;
        }
    }
    if constexpr (NB != 0 && LV != 0) {
        // compiled-in plan: 32-bit element offsets (ot_level routes gates whose
        // key rows would reach 2^32 words to the runtime-plan kernel)
        constexpr bool last = LV > digit_plan(NB, SB, MODE).levels;
        const uint32_t N = uint32_t(a.N), Npad = (N + 31u) & ~31u, stride = gridDim.x * blockDim.x;
        for (uint32_t e = blockIdx.x * blockDim.x + threadIdx.x; e < Npad; e += stride) {
            uint32_t hl = 0, he = 0, ll = 0;
            if (e < N) level_elem_c<MODE, NB, SB, PARTY, LV>(a, e, N, hl, he, ll);
            if constexpr (last) {
                const uint32_t wh = __ballot_sync(0xFFFFFFFFu, hl), we = __ballot_sync(0xFFFFFFFFu, he),
                               wl = __ballot_sync(0xFFFFFFFFu, ll);
                if ((threadIdx.x & 31) == 0) {
                    const uint32_t wi = e >> 5;
                    if (a.bits_hi) {
                        a.bits_hi[wi] = wh;
                        if constexpr (MODE != PLAN_TT_FULL) a.bits_hi[uint32_t(a.nw) + wi] = we;
                    }
                    a.bits_lo[wi] = wl;
                }
            }
        }
        return;
    }
    const uint64_t N = a.N;
    const int l = LV ? LV : a.level;
    const uint64_t Npad = (N + 31) & ~uint64_t(31);
    const bool last = l > a.P.levels;
    for (uint64_t e = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < Npad; e += uint64_t(gridDim.x) * blockDim.x) {
        uint32_t hl = 0, he = 0, ll = 0;
        if (e < N) {
            if (a.P.state_bytes() == 4) {
                level_elem<PARTY, uint32_t>(a.P, a, l, e, hl, he, ll);
            } else {
                level_elem<PARTY, uint64_t>(a.P, a, l, e, hl, he, ll);
            }
        }
        if (last) {
            const uint32_t wh = __ballot_sync(0xFFFFFFFFu, hl), we = __ballot_sync(0xFFFFFFFFu, he),
                           wl = __ballot_sync(0xFFFFFFFFu, ll);
            if ((threadIdx.x & 31) == 0) {
                const uint64_t wi = e >> 5;
                if (a.bits_hi) {
                    a.bits_hi[wi] = wh;
                    if (a.P.mode != PLAN_TT_FULL) a.bits_hi[a.nw + wi] = we;
                }
                a.bits_lo[wi] = wl;
            }
        }
    }
}

// ---------------------------------------------------------------- launchers

template <typename T, class E, int NB, int SB, int PARTY>
static int garble_launch(const OtGarbleArgs<T> &a, cudaStream_t st)
{
    const int smem = E::SMEM + 256;
    auto k = ot_garble_kernel<T, E, NB, SB, PARTY>;
    DDG_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    k<<<aes_blocks<E>(a.N), E::THREADS, smem, st>>>(a);
    return DDG_OK;
}

// the plan compiled in for (bw, scale) = (32, 12) / (64, 12), else the runtime plan
template <typename T, class E>
static int garble_dispatch(const OtGarbleArgs<T> &a, int s, cudaStream_t st)
{
    constexpr int NB = sizeof(T) == 4 ? 32 : 64;
    if (s == 12) return a.party == 0 ? garble_launch<T, E, NB, 12, 0>(a, st) : garble_launch<T, E, NB, 12, 1>(a, st);
    return a.party == 0 ? garble_launch<T, E, 0, 0, 0>(a, st) : garble_launch<T, E, 0, 0, 1>(a, st);
}

int ot_garble(const GateLayout &L, int party, const void *xhat, const void *key, uint32_t *tables, void *state,
              uint32_t *tri, cudaStream_t st)
{
    DDG_TRY(aes_device_init());
    if (L.n == 0) return DDG_OK;
    const OtPlan &P = ot_plan_cached(L.bw, L.s);
    DDG_CHECK(P.ok, DDG_ERR_ARG, "no OT-gate plan for bw %d, scale %d", L.bw, L.s);
    DDG_CHECK(party == 0 || party == 1, DDG_ERR_ARG, "party must be 0 or 1");
    const uint8_t *k = static_cast<const uint8_t *>(key);
    TimedLaunch tl;
    DDG_TRY(tl.begin(st));
    if (L.bw == 32) {
        OtGarbleArgs<uint32_t> a{P, party, L.n, static_cast<const uint32_t *>(xhat),
                                 reinterpret_cast<const uint32_t *>(k + L.ot_ks), tables, state, tri};
        DDG_TRY((aes_tables() == 4 ? garble_dispatch<uint32_t, AesLane4>(a, L.s, st)
                                   : garble_dispatch<uint32_t, AesLane2>(a, L.s, st)));
    } else {
        OtGarbleArgs<uint64_t> a{P, party, L.n, static_cast<const uint64_t *>(xhat),
                                 reinterpret_cast<const uint32_t *>(k + L.ot_ks), tables, state, tri};
        DDG_TRY((aes_tables() == 4 ? garble_dispatch<uint64_t, AesLane4>(a, L.s, st)
                                   : garble_dispatch<uint64_t, AesLane2>(a, L.s, st)));
    }
    note_launch();
    DDG_CUDA(cudaGetLastError());
    // algorithmic bytes: the input, the tables, the digit shares and the aux blocks written
    const double n = double(L.n), G = P.garbled_by(party);
    DDG_TRY(tl.end(st, n * (L.bw / 8.0 + 4.0 * G + P.state_bytes() + 4.0 * P.tri_words()), n * (P.naux + P.npad[party]),
                   n));
    return DDG_OK;
}

// a compiled-in plan also compiles in the level (every node and bit offset a constant)
template <int MODE, int NB, int SB, int PARTY>
static void level_launch(const OtLevelArgs &a, int grid, cudaStream_t st)
{
    switch (a.level) {
    case 1: ot_level_kernel<MODE, NB, SB, PARTY, 1><<<grid, 256, 0, st>>>(a); break;
    case 2: ot_level_kernel<MODE, NB, SB, PARTY, 2><<<grid, 256, 0, st>>>(a); break;
    case 3: ot_level_kernel<MODE, NB, SB, PARTY, 3><<<grid, 256, 0, st>>>(a); break;
    case 4: ot_level_kernel<MODE, NB, SB, PARTY, 4><<<grid, 256, 0, st>>>(a); break;
    case 5: ot_level_kernel<MODE, NB, SB, PARTY, 5><<<grid, 256, 0, st>>>(a); break;
    case 6: ot_level_kernel<MODE, NB, SB, PARTY, 6><<<grid, 256, 0, st>>>(a); break;
    default: ot_level_kernel<MODE, NB, SB, PARTY, 0><<<grid, 256, 0, st>>>(a); break;
    }
}

static bool plan_compiled_in(const GateLayout &L);

template <int MODE, int PARTY>
static void level_dispatch(const GateLayout &L, const OtLevelArgs &a, int grid, cudaStream_t st)
{
    if (plan_compiled_in(L) && L.bw == 32) level_launch<MODE, 32, 12, PARTY>(a, grid, st);
    else if (plan_compiled_in(L)) level_launch<MODE, 64, 12, PARTY>(a, grid, st);
    else ot_level_kernel<MODE, 0, 0, PARTY, 0><<<grid, 256, 0, st>>>(a);
}

const OtPlan &gate_digit_plan(const GateLayout &L)
{
    static OtPlan tt[4][2][64];
    static std::once_flag once;
    std::call_once(once, [] {
        for (int m = PLAN_TT_RELU; m <= PLAN_TT_FULL; m++)
            for (int b = 0; b < 2; b++)
                for (int sc = 1; sc < 64; sc++) tt[m][b][sc] = digit_plan(b ? 64 : 32, sc, m);
    });
    if (L.ot) return ot_plan_cached(L.bw, L.s);
    return tt[tt_mode_of(L.kind)][L.bw == 64 ? 1 : 0][L.s > 0 && L.s < 64 ? L.s : 0];
}

// the level kernels take the compiled-in plan exactly when level_dispatch does:
// the scale-12 plans, on gates whose key rows stay below 2^32 words (its
// element offsets are 32-bit)
static bool plan_compiled_in(const GateLayout &L)
{
    if (L.s != 12 || (L.bw != 32 && L.bw != 64)) return false;
    const OtPlan &P = gate_digit_plan(L);
    return uint64_t(L.n) * uint64_t(P.rows + P.Gmax + P.tri_words() + 4) < (uint64_t(1) << 32);
}

int ot_open_bytes(const GateLayout &L, int level)
{
    return plan_compiled_in(L) ? open_width(gate_digit_plan(L), level) : 4;
}

// bytes per element of the digit-share state the level kernels read and write
static int ot_state_bytes(const GateLayout &L)
{
    const OtPlan &P = gate_digit_plan(L);
    return plan_compiled_in(L) ? state_width(P) : P.state_bytes();
}

int ot_level(const GateLayout &L, int party, int level, const void *key, const uint32_t *peer_tables,
             const void *open_own, const void *open_peer, void *state, const uint32_t *tri, void *open_out,
             uint32_t *bits_hi, uint32_t *bits_lo, cudaStream_t st, const void *xhat, const void *xhat2)
{
    if (L.n == 0) return DDG_OK;
    DDG_CHECK(L.ot || L.tt, DDG_ERR_ARG, "not an AND-tree gate");
    const OtPlan &P = gate_digit_plan(L);
    DDG_CHECK(P.ok && level >= 1 && level <= P.levels + 1, DDG_ERR_ARG, "AND-tree level %d out of range", level);
    DDG_CHECK(party == 0 || party == 1, DDG_ERR_ARG, "party must be 0 or 1");
    DDG_CHECK(!L.tt || level > 1 || xhat, DDG_ERR_ARG, "truth-table level 1 needs x_hat");
    const uint8_t *k = static_cast<const uint8_t *>(key);
    OtLevelArgs a;
    a.P = P, a.party = party, a.level = level, a.N = L.n, a.nw = (L.n + 31) / 32;
    a.recv = L.ot ? k + L.ot_recv : nullptr;
    a.peer_tables = peer_tables;
    a.c0 = L.ot ? reinterpret_cast<const uint32_t *>(k + L.ot_c0) : nullptr;
    a.xhat = xhat, a.xhat2 = L.tt && level == 1 ? xhat2 : nullptr;
    a.tables = L.tt ? reinterpret_cast<const uint32_t *>(k + L.tt_tables) : nullptr;
    a.open_own = open_own, a.open_peer = open_peer;
    a.state = state;
    a.tri = L.tt ? reinterpret_cast<const uint32_t *>(k + L.tt_tri) : tri;
    a.open_out = open_out, a.bits_hi = P.nd[0] ? bits_hi : nullptr, a.bits_lo = bits_lo;
    auto al16 = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    // four elements per thread (compiled-in TT plans): level 1 reads the tables and x_hat, later levels
    // the openings of the level before (4-byte aligned at 1-byte openings), the last level writes bit words
    a.vec4 = L.tt && plan_compiled_in(L) && L.n % 4 == 0 && al16(a.tri) && al16(state) &&
             (level == 1 ? al16(a.tables) && al16(xhat) && al16(a.xhat2) && al16(open_out)
                         : al16(open_own) && al16(open_peer) && (level > P.levels || al16(open_out)));
    const int sms = device_sms();
    const uint64_t threads = a.vec4 ? L.n / 4 : L.n;
    const uint64_t blocks = (threads + 255) / 256, cap = uint64_t(sms > 0 ? sms : 148) * 8;
    const int grid = int(blocks < cap ? blocks : cap);
    TimedLaunch tl;
    DDG_TRY(tl.begin(st));
    if (L.ot) party == 0 ? level_dispatch<PLAN_OT, 0>(L, a, grid, st) : level_dispatch<PLAN_OT, 1>(L, a, grid, st);
    else if (P.mode == PLAN_TT_FULL)
        party == 0 ? level_dispatch<PLAN_TT_FULL, 0>(L, a, grid, st) : level_dispatch<PLAN_TT_FULL, 1>(L, a, grid, st);
    else if (L.kind == GATE_LRS_TT)
        party == 0 ? level_dispatch<PLAN_TT_LRS, 0>(L, a, grid, st) : level_dispatch<PLAN_TT_LRS, 1>(L, a, grid, st);
    else party == 0 ? level_dispatch<PLAN_TT_RELU, 0>(L, a, grid, st) : level_dispatch<PLAN_TT_RELU, 1>(L, a, grid, st);
    note_launch();
    DDG_CUDA(cudaGetLastError());
    // algorithmic bytes: state and triple words in (the TT first level: x_hat
    // and the truth-table rows instead of the state); OT level 1 also the
    // receiver records and the peer's tables, later levels both parties'
    // openings (+ OT party 0's c word); state and openings out, or the
    // comparison bit arrays at the last level
    const double n = double(L.n), Gq = P.garbled_by(1 - party);
    double bytes = n * 4.0 * P.tri_words();
    const double sb = ot_state_bytes(L);
    if (L.tt && level == 1) bytes += n * ((xhat2 ? 2.0 : 1.0) * L.bw / 8.0 + 4.0 * P.rows);
    else bytes += n * sb;
    if (level > 1) bytes += n * (2.0 * ot_open_bytes(L, level - 1) + (L.ot && party == 0 ? 4.0 : 0.0));
    else if (L.ot) bytes += n * 5.0 * Gq;
    const double arrays = P.mode == PLAN_TT_FULL ? 2.0 : P.nd[0] ? 3.0 : 1.0;
    bytes += level <= P.levels ? n * (double(ot_open_bytes(L, level)) + sb) : n * arrays / 8.0;
    DDG_TRY(tl.end(st, bytes, 0.0, n));
    return DDG_OK;
}

OtScratch ot_scratch_bytes(const GateLayout &L)
{
    const OtPlan &P = gate_digit_plan(L);
    if (L.tt) return OtScratch{0, uint64_t(P.state_bytes()) * L.n, 0};
    const uint64_t n = L.n;
    return OtScratch{4ull * uint64_t(P.Gmax) * n, uint64_t(P.state_bytes()) * n, 4ull * uint64_t(P.tri_words()) * n};
}

}  // namespace ddg
