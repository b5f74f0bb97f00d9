// The digit plan of the comparison gates that split a comparison into
// radix-2^w digits combined by a Beaver AND tree: the OT gates
// (GATE_RELU_OT, GATE_RELU_ARS_OT; ot.cuh) and the truth-table gates
// (GATE_RELU_TT, GATE_RELU_ARS_TT, GATE_LRS_TT).  Host and device, constexpr.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace ddg {

constexpr int OT_W = 4;                // digit bits (radix 16)
constexpr int OT_MAX_DIGITS = 18;      // n - 1 <= 63 bits in two parts
constexpr int OT_MAX_COMB = 16;        // D - 2 combines at most
constexpr int OT_MAX_LEVELS = 5;       // ceil(log2(16))
constexpr int OT_MAX_AUX = 2;          // aux PRF blocks per party and element
constexpr int OT_MAX_PAD = 3;          // pad PRF blocks per party and element (Gmax <= 9)
constexpr int TT_MAX_ROWS = 24;        // truth-table rows (32 bits) per element and party

struct OtComb {
    uint8_t part, h, l, out;  // part 0 = hi, 1 = lo, 2 = the cross combine; node indices within the part
    uint8_t eq, root;         // computes eq; its output is opened (carries a mask bit)
};

// plan modes: the OT gates' two parts of radix-16 digits; the truth-table
// (TT) gates' ReLU comparison (hi digits of 5 bits at bw=32, 4 at bw=64; lo
// digits of 4) and their truncation carry (one part of two 6-bit digits)
// PLAN_TT_FULL: the ReLU digits of PLAN_TT_RELU, whose two part roots feed one
// more AND (the cross combine) giving the full (n-1)-bit comparison, so that
// round 2 only needs the full compare bit and the lo compare bit
enum : int { PLAN_OT = 0, PLAN_TT_RELU = 1, PLAN_TT_LRS = 2, PLAN_TT_FULL = 3 };

struct OtPlan {
    int mode = PLAN_OT;
    int n = 0, s = 0;
    int D = 0, G0 = 0, Gmax = 0;        // digits; OT: party 0 garbles [0, G0), party 1 [G0, D); Gmax = G0
    int bits[2] = {0, 0}, wid[2] = {0, 0};  // bits and digit width of each part (hi, lo)
    bool peq[2] = {true, false};        // the part's root needs its equality bit
    int nd[2] = {0, 0};                 // digits per part (hi, lo)
    int base[2] = {0, 0};               // global index of a part's first digit
    // TT: digit g's truth table is drows(g) 32-bit rows from row drow0(g): its
    // 2^w lt bits, then (deq(g)) its 2^w eq bits, packed from bit 0.  Packed
    // in one int per digit (deq | rows << 8 | first row << 16): 8-bit arrays
    // of other lengths in the plan made the compiler keep compiled-in plans in
    // local memory.
    int dinfo[OT_MAX_DIGITS] = {};
    int rows = 0;
    int levels = 0, ncomb = 0;
    int lvl_first[OT_MAX_LEVELS + 2] = {};  // combines of level l (1-based): [lvl_first[l-1], lvl_first[l])
    // pass-through of an odd top node at level l: part p moves node pass_from to pass_to (-1: none)
    int8_t pass_from[OT_MAX_LEVELS + 1][2] = {}, pass_to[OT_MAX_LEVELS + 1][2] = {};
    OtComb comb[OT_MAX_COMB] = {};
    // position of combine q's triple bits in the party's triple words: (a, b,
    // b') at tpa[q] + 0..2, (c, c') at tpc[q] + 0..1 (b' and c' only for a
    // combine that computes eq: the others have no such bits); the
    // lo-compare mask bit (PLAN_TT_FULL) at mu_pos.  TT plans group them by AND
    // level in the lane layout of the level kernels (tt_place: every level's
    // (a, b, b') of all its combines is one shifted mask of one word, its (c,
    // c') another), when that fits the plan's triple words (tpacked);
    // otherwise, and for the OT plans, 5 bits per combine from 5q and the mask
    // bit at 5 ncomb.
    uint8_t tpa[OT_MAX_COMB] = {}, tpc[OT_MAX_COMB] = {};
    int mu_pos = 0;
    bool tpacked = false;
    int aux_bits = 0, naux = 0, tri0 = 0;  // OT: aux bits used, aux blocks, first triple bit (6 * Gmax)
    int npad[2] = {0, 0};               // OT: pad blocks of party 0 / 1
    bool ok = false;

    __host__ __device__ constexpr int garbler(int g) const { return g < G0 ? 0 : 1; }
    __host__ __device__ constexpr int local(int g) const { return g < G0 ? g : g - G0; }
    __host__ __device__ constexpr int part_of(int g) const { return g < nd[0] ? 0 : 1; }
    // bit position of digit g in x_hat / r, and its width
    __host__ __device__ constexpr int shift(int g) const { return g < nd[0] ? s + wid[0] * g : wid[1] * (g - nd[0]); }
    __host__ __device__ constexpr int width(int g) const
    {
        const int p = g < nd[0] ? 0 : 1, j = g < nd[0] ? g : g - nd[0];
        const int rem = bits[p] - wid[p] * j;
        return rem < wid[p] ? rem : wid[p];
    }
    __host__ __device__ constexpr int garbled_by(int p) const { return p == 0 ? G0 : D - G0; }
    __host__ __device__ constexpr int deq(int g) const { return dinfo[g] & 0xff; }
    __host__ __device__ constexpr int drows(int g) const { return (dinfo[g] >> 8) & 0xff; }
    __host__ __device__ constexpr int drow0(int g) const { return dinfo[g] >> 16; }
    // evaluator scratch per element: digit-share state (2 bits per node) and
    // the triple bits (a, b, b', c1, c1') of every combine, 32-bit words
    __host__ __device__ constexpr int state_bytes() const { return 2 * D <= 32 ? 4 : 8; }
    __host__ __device__ constexpr int tri_words() const { return (5 * ncomb + (mode == PLAN_TT_FULL ? 1 : 0) + 31) / 32; }
    // state bit positions (lt; eq at +1) of combine q's H and L inputs and of
    // its output.  The cross combine takes the hi root (H) and the lo root (L)
    // and overwrites the hi root.
    __host__ __device__ constexpr int hpos(int q) const
    {
        return comb[q].part == 2 ? 2 * base[0] : 2 * base[comb[q].part] + 2 * comb[q].h;
    }
    __host__ __device__ constexpr int lpos(int q) const
    {
        return comb[q].part == 2 ? 2 * base[1] : 2 * base[comb[q].part] + 2 * comb[q].l;
    }
    __host__ __device__ constexpr int opos(int q) const
    {
        return comb[q].part == 2 ? 2 * base[0] : 2 * base[comb[q].part] + 2 * comb[q].out;
    }
    // PLAN_TT_FULL: the position of the party's share of the lo compare's mask bit
    __host__ __device__ constexpr int mu_bit() const { return mu_pos; }
    // bit k (0..4 = a, b, b', c, c') of combine q in the triple words
    __host__ __device__ constexpr int tpos(int q, int k) const { return k < 3 ? tpa[q] + k : tpc[q] + k - 3; }
    // lane of combine q at its level in the level kernels' word-parallel layout:
    // 2 base + i 2^(l+1) for combine i of a part at level l; 0 for the cross combine
    __host__ __device__ constexpr int lane_of(int q) const
    {
        return comb[q].part == 2 ? 0 : 2 * base[comb[q].part] + int(comb[q].out) * (2 << level_of(q));
    }
    // AND-tree level (1-based) of combine q
    __host__ __device__ constexpr int level_of(int q) const
    {
        int l = 1;
        while (l <= levels && q >= lvl_first[l]) l++;
        return l;
    }
};

// first fit of the bit group m (offsets from bit 0, all below 32) into the
// free bits of words [0, words): global position of its bit 0, or -1
__host__ __device__ constexpr int place_bits(uint32_t (&used)[3], int words, uint32_t m)
{
    int hi = 0;
    for (int b = 0; b < 32; b++)
        if ((m >> b) & 1u) hi = b;
    for (int w = 0; w < words; w++)
        for (int sh = 0; sh + hi < 32; sh++)
            if (((m << sh) & used[w]) == 0u) {
                used[w] |= m << sh;
                return 32 * w + sh;
            }
    return -1;
}

// triple-bit positions of a TT plan (see OtPlan::tpa): per level in order its
// (a, b, b') group, then its (c, c') group (b', c' only for the combines that
// compute eq), then the mask bit; first fit, in the plan's tri_words() words.
// Plans whose digit state does not fit 32 bits keep 5 bits per combine.
// The oracle (oracle/fss_ref.c, tt_place) places them by the same steps.
__host__ __device__ constexpr void tt_place(OtPlan &P)
{
    for (int q = 0; q < P.ncomb; q++) P.tpa[q] = uint8_t(5 * q), P.tpc[q] = uint8_t(5 * q + 3);
    P.mu_pos = 5 * P.ncomb;
    P.tpacked = false;
    // the lane layout needs the digit state in one 32-bit word (2 D <= 32): its
    // lanes, and every group's bits lane .. lane + 2, then stay below bit 31
    if (P.mode == PLAN_OT || 2 * P.D > 32) return;
    uint32_t used[3] = {0u, 0u, 0u};
    uint8_t pa[OT_MAX_COMB] = {}, pc[OT_MAX_COMB] = {};
    const int words = P.tri_words();
    for (int l = 1; l <= P.levels; l++) {
        const int qa = P.lvl_first[l - 1], qb = P.lvl_first[l];
        if (qa >= qb) continue;
        uint32_t ma = 0u, mc = 0u;
        for (int q = qa; q < qb; q++) {
            const bool eq = P.comb[q].eq != 0;
            ma |= (eq ? 7u : 3u) << P.lane_of(q), mc |= (eq ? 3u : 1u) << P.lane_of(q);
        }
        const int ga = place_bits(used, words, ma);
        if (ga < 0) return;
        const int gc = place_bits(used, words, mc);
        if (gc < 0) return;
        for (int q = qa; q < qb; q++) pa[q] = uint8_t(ga + P.lane_of(q)), pc[q] = uint8_t(gc + P.lane_of(q));
    }
    int mu = 5 * P.ncomb;
    if (P.mode == PLAN_TT_FULL) {
        mu = place_bits(used, words, 1u);
        if (mu < 0) return;
    }
    for (int q = 0; q < P.ncomb; q++) P.tpa[q] = pa[q], P.tpc[q] = pc[q];
    P.mu_pos = mu;
    P.tpacked = true;
}

// Plan for an n-bit ring and scale s.  OT and TT ReLU: hi = bits [s, n-1),
// lo = bits [0, s); TT truncation: lo = bits [0, s) only.  constexpr, so
// kernels specialised for a (bw, scale, mode) see every digit, node and bit
// position as a compile-time constant.
__host__ __device__ constexpr OtPlan digit_plan(int n, int s, int mode)
{
    OtPlan P;
    P.mode = mode;
    P.n = n, P.s = s;
    P.bits[0] = mode == PLAN_TT_LRS ? 0 : n - 1 - s;
    P.bits[1] = s;
    P.wid[0] = (mode == PLAN_TT_RELU || mode == PLAN_TT_FULL) && n == 32 ? 5 : OT_W;
    P.wid[1] = mode == PLAN_TT_LRS ? 6 : OT_W;
    if ((mode != PLAN_TT_LRS && P.bits[0] < 1) || P.bits[1] < 1) return P;
    P.nd[0] = (P.bits[0] + P.wid[0] - 1) / P.wid[0];
    P.nd[1] = (P.bits[1] + P.wid[1] - 1) / P.wid[1];
    P.base[0] = 0, P.base[1] = P.nd[0];
    P.D = P.nd[0] + P.nd[1];
    if (P.D > OT_MAX_DIGITS) return P;
    P.G0 = mode == PLAN_OT ? (P.D + 1) / 2 : 0;
    P.Gmax = P.G0;
    int row = 0;
    for (int g = 0; g < P.D; g++) {
        const int p = g < P.nd[0] ? 0 : 1, j = g < P.nd[0] ? g : g - P.nd[0];
        const int eq = (j > 0 || P.peq[p]) ? 1 : 0;
        const int nr = ((1 << P.width(g)) * (eq ? 2 : 1) + 31) / 32;
        P.dinfo[g] = eq | (nr << 8) | (row << 16);
        row += nr;
    }
    P.rows = row;
    int k[2] = {P.nd[0], P.nd[1]};
    int q = 0, l = 0;
    P.lvl_first[0] = 0;
    while (k[0] > 1 || k[1] > 1) {
        l++;
        if (l > OT_MAX_LEVELS) return P;
        for (int p = 0; p < 2; p++) {
            P.pass_from[l][p] = -1, P.pass_to[l][p] = -1;
            if (k[p] <= 1) continue;
            const int nk = (k[p] + 1) / 2;
            for (int i = 0; i < k[p] / 2; i++) {
                if (q >= OT_MAX_COMB) return P;
                OtComb &c = P.comb[q++];
                c.part = uint8_t(p), c.h = uint8_t(2 * i + 1), c.l = uint8_t(2 * i), c.out = uint8_t(i);
                c.root = uint8_t(nk == 1 && mode != PLAN_TT_FULL);
                c.eq = uint8_t(i > 0 || P.peq[p]);
            }
            if (k[p] & 1) P.pass_from[l][p] = int8_t(k[p] - 1), P.pass_to[l][p] = int8_t(k[p] / 2);
            k[p] = nk;
        }
        P.lvl_first[l] = q;
    }
    if (mode == PLAN_TT_FULL) {
        // one more level: full compare = hi_lt ^ (hi_eq & lo_lt), opened
        l++;
        if (l > OT_MAX_LEVELS || q >= OT_MAX_COMB) return P;
        OtComb &c = P.comb[q++];
        c.part = 2, c.h = 0, c.l = 0, c.out = 0, c.eq = 0, c.root = 1;
        P.pass_from[l][0] = P.pass_from[l][1] = -1, P.pass_to[l][0] = P.pass_to[l][1] = -1;
        P.lvl_first[l] = q;
    }
    P.levels = l, P.ncomb = q;
    P.tri0 = 6 * P.Gmax;
    P.aux_bits = P.tri0 + 5 * q;
    P.naux = (P.aux_bits + 127) / 128;
    if (P.naux < 1) P.naux = 1;
    P.npad[0] = (P.G0 + 3) / 4, P.npad[1] = (P.D - P.G0 + 3) / 4;
    P.ok = (mode != PLAN_OT || (P.naux <= OT_MAX_AUX && P.npad[0] <= OT_MAX_PAD && P.npad[1] <= OT_MAX_PAD)) &&
           P.tri_words() <= 3 && P.rows <= TT_MAX_ROWS;
    if (P.ok) tt_place(P);
    return P;
}
__host__ __device__ constexpr OtPlan ot_plan(int n, int s) { return digit_plan(n, s, PLAN_OT); }

}  // namespace ddg
