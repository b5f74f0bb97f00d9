// OT-leaf comparison gates (GATE_RELU_OT, GATE_RELU_ARS_OT): the plan shared
// by the dealer, the evaluators and the C oracle.
//
// These gates compute what GATE_RELU_SPLIT / GATE_RELU_ARS_SPLIT compute and
// reuse their round-2 algebra and dealer words; only the comparison bits are
// produced differently.  The split comparison needs, for the masked input
// x_hat and the dealer's mask r, the XOR-shared bits
//   hi: 1{U < A}, 1{U == A}   U, A = bits [s, n-1) of x_hat and r
//   lo: 1{V < B}              V, B = bits [0, s)
// each XORed with a dealer mask bit (rho_c, rho_e, rho_L), which both parties
// then open.  Instead of evaluating a DCF key (an AES tree per element), the
// parties run the millionaires' structure of the reference's LSS backend
// (gpu_mpc/lss/lss_compare.cpp: radix-16 digits, a 1-out-of-16 OT per digit
// giving shares of the digit's (>, ==) pair, then a tree of Beaver ANDs,
// gpu_mpc/lss/lss_protocol.md sections 1-2 and 5), adapted to masked-public
// inputs:
//
// * Digits.  Each part is cut into radix-16 digits from its least significant
//   bit (the top digit keeps the remainder).  Digit g of the global list
//   (hi digits, then lo digits) is "garbled" by party 0 if g < G0 = ceil(D/2),
//   else by party 1, so both directions of the first message carry the same
//   number of tables.
// * One message per digit, no receiver query.  The garbler knows x_hat, the
//   receiver does not need to: its choice is c = (a_d + delta) mod 16 where a_d
//   is the mask digit, known only to the dealer, and delta a garbler-side
//   random rotation, so c is uniform to the receiver and c, together with the
//   pad k_c, sits in the receiver's key.  The garbler sends the 16 entries
//   T[u] = (1{x_d < u - delta}, 1{x_d == u - delta}) ^ (s_lt, s_eq) ^ k_u as one
//   32-bit word (lt entries in bits 0-15, eq entries in bits 16-31) and keeps
//   (s_lt, s_eq) as its share; the receiver's share is T[c] ^ k_c.  (The
//   reference's OT16 sends delta = r - d from the receiver first,
//   lss_protocol.md section 2; here the dealer knows the receiver's choice.)
// * AND tree.  Nodes of a part, least significant first, are combined in
//   pairs (H = node 2i+1, L = node 2i):
//     lt = lt_H ^ (eq_H & lt_L),   eq = eq_H & eq_L,
//   an odd top node passes up.  Each AND is a Beaver bit triple (a, b, c = ab)
//   with eq_H's mask a shared by the two ANDs of a node; one round per level.
//   A node's eq is computed when it will be an H later (index > 0) or when it
//   is the root of the hi part.
// * Output masks.  The root combine of a part folds its mask bit into the
//   triple: c = ab ^ rho, so the AND outputs the masked bit directly; a part
//   with one digit folds rho into the receiver's pad instead.
// * Randomness.  Every party regenerates its own correlated randomness from a
//   per-gate AES-128 key K_p = AES_dealer(p || op || P_OT_PARTY) (its
//   expanded schedule is the first 176 bytes of
//   the party's key): aux block j = AES_Kp(e || 0 || P_OT_AUX + j) holds, per
//   garbled local digit t, delta (bits 6t..6t+3) and (s_lt, s_eq) (6t+4, 6t+5),
//   then from bit 6*Gmax, per combine q, (a, b, b', c1, c1') at 5q..5q+4; pad
//   block j = AES_Kp(e || 0 || P_OT_PAD + j) gives digit t's 32 pad bits in
//   word t mod 4 of block t / 4.  Party 0's triple c bits are explicit in its
//   key (the c0 word: bits 2q, 2q+1), party 1's come from its aux block, as
//   the reference's LSS2 format splits explicit and regenerated shares
//   (lss_protocol.md section 9.2).
//
// Key of one OT gate, per party, N elements:
//   [ks: 44 u32 AES round keys of K_p] [recv: Gmax x N bytes, byte = c | k_lt << 4 | k_eq << 5
//   for the digits the peer garbles, slot = the garbler's local index]
//   [c0: N u32, party 0 only (zero for party 1)] [words: nwords x N ring words]
#pragma once
#include <cstdint>

#include "aes_dev.cuh"
#include "common.cuh"

namespace ddg {

constexpr int OT_W = 4;                // digit bits (radix 16)
constexpr int OT_MAX_DIGITS = 18;      // n - 1 <= 63 bits in two parts
constexpr int OT_MAX_COMB = 16;        // D - 2 combines at most
constexpr int OT_MAX_LEVELS = 5;       // ceil(log2(16))
constexpr int OT_MAX_AUX = 2;          // aux PRF blocks per party and element
constexpr int OT_MAX_PAD = 3;          // pad PRF blocks per party and element (Gmax <= 9)

// PRF purposes of the OT gates: the party keys under the dealer key (clear of
// the dealer's word shares P_SHARE + k, k < 80), aux and pad blocks under K_p
enum : uint32_t { P_OT_PARTY = 0x100, P_OT_AUX = 0x110, P_OT_PAD = 0x120 };

struct OtComb {
    uint8_t part, h, l, out;  // part 0 = hi, 1 = lo; node indices within the part
    uint8_t eq, root;         // computes eq; produces the part's root
};

struct OtPlan {
    int n = 0, s = 0;
    int D = 0, G0 = 0, Gmax = 0;        // digits; party 0 garbles [0, G0), party 1 [G0, D); Gmax = G0
    int nd[2] = {0, 0};                 // digits per part (hi, lo)
    int base[2] = {0, 0};               // global index of a part's first digit
    int levels = 0, ncomb = 0;
    int lvl_first[OT_MAX_LEVELS + 2] = {};  // combines of level l (1-based): [lvl_first[l-1], lvl_first[l])
    // pass-through of an odd top node at level l: part p moves node pass_from to pass_to (-1: none)
    int8_t pass_from[OT_MAX_LEVELS + 1][2] = {}, pass_to[OT_MAX_LEVELS + 1][2] = {};
    OtComb comb[OT_MAX_COMB] = {};
    int aux_bits = 0, naux = 0, tri0 = 0;  // aux bits used, aux blocks, first triple bit (6 * Gmax)
    int npad[2] = {0, 0};               // pad blocks of party 0 / 1
    bool ok = false;

    __host__ __device__ constexpr int garbler(int g) const { return g < G0 ? 0 : 1; }
    __host__ __device__ constexpr int local(int g) const { return g < G0 ? g : g - G0; }
    __host__ __device__ constexpr int part_of(int g) const { return g < nd[0] ? 0 : 1; }
    // bit position of digit g in x_hat / r, and its width
    __host__ __device__ constexpr int shift(int g) const { return g < nd[0] ? s + OT_W * g : OT_W * (g - nd[0]); }
    __host__ __device__ constexpr int width(int g) const
    {
        const int bits = g < nd[0] ? n - 1 - s : s;
        const int j = g < nd[0] ? g : g - nd[0];
        const int rem = bits - OT_W * j;
        return rem < OT_W ? rem : OT_W;
    }
    __host__ __device__ constexpr int garbled_by(int p) const { return p == 0 ? G0 : D - G0; }
    // evaluator scratch per element: digit-share state (2 bits per node) and
    // the triple bits (a, b, b', c1, c1') of every combine, 32-bit words
    __host__ __device__ constexpr int state_bytes() const { return 2 * D <= 32 ? 4 : 8; }
    __host__ __device__ constexpr int tri_words() const { return (5 * ncomb + 31) / 32; }
    // AND-tree level (1-based) of combine q
    __host__ __device__ constexpr int level_of(int q) const
    {
        int l = 1;
        while (l <= levels && q >= lvl_first[l]) l++;
        return l;
    }
};

// Plan for an n-bit ring and scale s: hi = bits [s, n-1), lo = bits [0, s).
// constexpr, so kernels specialised for a (bw, scale) see every digit, node
// and bit position as a compile-time constant.
__host__ __device__ constexpr OtPlan ot_plan(int n, int s)
{
    OtPlan P;
    P.n = n, P.s = s;
    const int hb = n - 1 - s, lb = s;
    if (hb < 1 || lb < 1) return P;
    P.nd[0] = (hb + OT_W - 1) / OT_W;
    P.nd[1] = (lb + OT_W - 1) / OT_W;
    P.base[0] = 0, P.base[1] = P.nd[0];
    P.D = P.nd[0] + P.nd[1];
    if (P.D > OT_MAX_DIGITS) return P;
    P.G0 = (P.D + 1) / 2;
    P.Gmax = P.G0;
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
                c.root = uint8_t(nk == 1);
                c.eq = uint8_t(i > 0 || p == 0);
            }
            if (k[p] & 1) P.pass_from[l][p] = int8_t(k[p] - 1), P.pass_to[l][p] = int8_t(k[p] / 2);
            k[p] = nk;
        }
        P.lvl_first[l] = q;
    }
    P.levels = l, P.ncomb = q;
    P.tri0 = 6 * P.Gmax;
    P.aux_bits = P.tri0 + 5 * q;
    P.naux = (P.aux_bits + 127) / 128;
    if (P.naux < 1) P.naux = 1;
    P.npad[0] = (P.G0 + 3) / 4, P.npad[1] = (P.D - P.G0 + 3) / 4;
    P.ok = P.naux <= OT_MAX_AUX && P.npad[0] <= OT_MAX_PAD && P.npad[1] <= OT_MAX_PAD;
    return P;
}

// garbler's table word for digit value xd (width w), rotation delta, share
// (s_lt, s_eq) and pad word: bit u (u < 2^w) = 1{xd < u - delta} ^ s_lt ^
// pad_u, bit 16 + u = 1{xd == u - delta} ^ s_eq ^ pad_{16+u}
__host__ __device__ inline uint32_t ot_table(uint32_t xd, int w, uint32_t delta, uint32_t s_lt, uint32_t s_eq,
                                             uint32_t pad)
{
    const uint32_t W = 1u << w, m = (1u << W) - 1u;     // W <= 16 entries
    const uint32_t lt = m & ~((2u << xd) - 1u);         // v in (xd, W)
    const uint32_t eq = 1u << xd;
    const uint32_t rl = ((lt << delta) | (lt >> (W - delta))) & m;
    const uint32_t re = ((eq << delta) | (eq >> (W - delta))) & m;
    const uint32_t word = (rl ^ (s_lt ? m : 0u)) | ((re ^ (s_eq ? m : 0u)) << 16);
    return word ^ (pad & (m | (m << 16)));
}

// ---- dealer, per element (gate keygen kernel): the receivers' records and
// party 0's triple c bits.  r = the element's input mask; rho_* = the opened
// bits' masks (hi compare, hi equality, lo compare).
template <class E>
__device__ __forceinline__ void ot_keygen_elem(const E &A, const OtPlan &P, const uint32_t *rk0, const uint32_t *rk1,
                                               uint64_t e, uint64_t N, uint64_t r, uint32_t rho_c, uint32_t rho_e,
                                               uint32_t rho_L, uint8_t *recv0, uint8_t *recv1, uint32_t *c0)
{
    Blk aux[2][OT_MAX_AUX];
    for (int p = 0; p < 2; p++) {
        const uint32_t *rk = p ? rk1 : rk0;
        aux[p][0] = A.prg(rk, 0, P_OT_AUX, e);
        aux[p][1] = P.naux > 1 ? A.prg(rk, 0, P_OT_AUX + 1, e) : aux[p][0];
    }
    auto abit = [&](int p, int i) -> uint32_t {
        return uint32_t(blk_bit(i < 128 ? aux[p][0] : aux[p][1], uint32_t(i & 127)));
    };
    const uint64_t rhi = (r >> P.s) & ((uint64_t(1) << (P.n - 1 - P.s)) - 1), rlo = r & ((uint64_t(1) << P.s) - 1);
    Blk pad = aux[0][0];
    int pad_for = -1;  // (party << 8) | block of the pad block held
    for (int g = 0; g < P.D; g++) {
        const int pg = P.garbler(g), t = P.local(g), w = P.width(g), part = P.part_of(g);
        const uint32_t wm = (1u << w) - 1u;
        const int want = (pg << 8) | (t >> 2);
        if (want != pad_for) pad = A.prg(pg ? rk1 : rk0, 0, P_OT_PAD + uint32_t(t >> 2), e), pad_for = want;
        uint32_t delta = 0;
        for (int i = 0; i < 4; i++) delta |= abit(pg, 6 * t + i) << i;
        delta &= wm;
        const uint32_t alpha = uint32_t((part == 0 ? rhi >> (OT_W * g) : rlo >> (OT_W * (g - P.nd[0])))) & wm;
        const uint32_t c = (alpha + delta) & wm;
        const uint32_t pw = (t & 3) == 0 ? pad.w[0] : (t & 3) == 1 ? pad.w[1] : (t & 3) == 2 ? pad.w[2] : pad.w[3];
        uint32_t klt = (pw >> c) & 1u, keq = (pw >> (16 + c)) & 1u;
        if (P.nd[part] == 1) klt ^= part == 0 ? rho_c : rho_L, keq ^= part == 0 ? rho_e : 0u;
        (pg ? recv0 : recv1)[uint64_t(t) * N + e] = uint8_t(c | (klt << 4) | (keq << 5));
    }
    uint32_t cw = 0;
    for (int q = 0; q < P.ncomb; q++) {
        const OtComb &C = P.comb[q];
        const int tb = P.tri0 + 5 * q;
        const uint32_t ta = abit(0, tb) ^ abit(1, tb), tbb = abit(0, tb + 1) ^ abit(1, tb + 1),
                       tb2 = abit(0, tb + 2) ^ abit(1, tb + 2);
        uint32_t cc = (ta & tbb) ^ abit(1, tb + 3), cc2 = (ta & tb2) ^ abit(1, tb + 4);
        if (C.root) cc ^= C.part == 0 ? rho_c : rho_L, cc2 ^= C.part == 0 ? rho_e : 0u;
        cw |= (cc << (2 * q)) | ((C.eq ? cc2 : 0u) << (2 * q + 1));
    }
    c0[e] = cw;
}

// ---- host side (ot.cu)

// the plan of (bw, s), built once per process
const OtPlan &ot_plan_cached(int bw, int s);
// K_p = AES_dk(p || op || P_OT_PARTY), expanded
AesKey ot_party_key(const AesKey &dk, uint32_t op, int party);
// party's first message: its garbled tables [Gmax][N] u32, its digit shares
// (state: N x state_bytes()) and its triple bits (tri: [tri_words()][N] u32)
int ot_garble(const GateLayout &L, int party, const void *xhat, const void *key, uint32_t *tables, void *state,
              uint32_t *tri, cudaStream_t st);
// level 1..levels: (level 1: take the peer's tables) close the previous level
// with both parties' openings, open this level's ANDs into open_out;
// level levels + 1: close the last level and write the masked comparison bits
// (bits_hi: [lt | eq] x ceil(N/32) words, bits_lo: lt)
int ot_level(const GateLayout &L, int party, int level, const void *key, const uint32_t *peer_tables,
             const uint32_t *open_own, const uint32_t *open_peer, void *state, const uint32_t *tri,
             uint32_t *open_out, uint32_t *bits_hi, uint32_t *bits_lo, cudaStream_t st);
// scratch of one party's OT gate, bytes: garbled tables, state, triple bits
struct OtScratch {
    uint64_t tables, state, tri;
};
OtScratch ot_scratch_bytes(const GateLayout &L);

}  // namespace ddg
