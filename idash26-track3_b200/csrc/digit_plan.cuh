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
    // PLAN_TT_FULL: the party's share of the lo compare's mask bit sits in its
    // triple words right after the combines' bits
    __host__ __device__ constexpr int mu_bit() const { return 5 * ncomb; }
    // AND-tree level (1-based) of combine q
    __host__ __device__ constexpr int level_of(int q) const
    {
        int l = 1;
        while (l <= levels && q >= lvl_first[l]) l++;
        return l;
    }
};

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
    return P;
}
__host__ __device__ constexpr OtPlan ot_plan(int n, int s) { return digit_plan(n, s, PLAN_OT); }

}  // namespace ddg
