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
#include "digit_plan.cuh"

namespace ddg {

// PRF purposes of the OT gates: the party keys under the dealer key (clear of
// the dealer's word shares P_SHARE + k, k < 80), aux and pad blocks under K_p
enum : uint32_t { P_OT_PARTY = 0x100, P_OT_AUX = 0x110, P_OT_PAD = 0x120 };

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

// ---- truth-table gates, dealer, per element (gate keygen kernel).  Each digit
// g of x_hat's comparison parts gets a table over its 2^w values: lt bits
// 1{x < a_g} at [0, 2^w), then (deq) eq bits 1{x == a_g} at [2^w, 2^(w+1)),
// a_g the mask digit; party 0's rows are dealer-PRG bits, party 1's rows are
// party 0's XOR the truth table (a part with one digit XORs its mask bits
// into every entry).  Every combine gets a Beaver triple: party 0's (a, b, b',
// c, c') and party 1's (a, b, b') from the PRG, party 1's c = ab ^ c0 (^ rho
// at a part's root), c' likewise.  Both parties' triple bits: 5 per combine.
enum : uint32_t { P_TT_RAND = 0x140 };

// pb: the element's mask-bit word (P_BITS); rho_c = bit 0 ^ bit 1, rho_L = bit
// 2 ^ bit 3, rho_e = bit 4 ^ bit 5.  PLAN_TT_FULL opens the full compare
// (cross combine, rho_c) and the lo root with the parties' own shares of
// rho_L (bits 2 and 3) added at the last level.
template <class E>
__device__ __forceinline__ void tt_keygen_elem(const E &A, const OtPlan &P, const uint32_t *dk, uint32_t op,
                                               uint64_t e, uint64_t N, uint64_t r, uint32_t pb, uint32_t *tab0,
                                               uint32_t *tab1, uint32_t *tri0, uint32_t *tri1)
{
    const uint32_t rho_c = (pb ^ (pb >> 1)) & 1u, rho_L = ((pb >> 2) ^ (pb >> 3)) & 1u,
                   rho_e = ((pb >> 4) ^ (pb >> 5)) & 1u;
    const bool full = P.mode == PLAN_TT_FULL;
    Blk blk{{0u, 0u, 0u, 0u}};
    int held = -1;
    // 32-bit word w of the dealer's random stream for this element
    auto word = [&](int w) -> uint32_t {
        const int b = w >> 2;
        if (b != held) blk = A.prg(dk, op, P_TT_RAND + uint32_t(b), e), held = b;
        const int k = w & 3;
        return k == 0 ? blk.w[0] : k == 1 ? blk.w[1] : k == 2 ? blk.w[2] : blk.w[3];
    };
    auto bit = [&](int i) -> uint32_t { return (word(i >> 5) >> (i & 31)) & 1u; };
    const uint64_t rhi = P.nd[0] ? (r >> P.s) & ((uint64_t(1) << P.bits[0]) - 1) : 0;
    const uint64_t rlo = r & ((uint64_t(1) << P.s) - 1);
    for (int g = 0; g < P.D; g++) {
        const int p = P.part_of(g), w = P.width(g), W = 1 << w;
        const uint64_t wm = W == 64 ? ~uint64_t(0) : (uint64_t(1) << W) - 1;
        const uint32_t alpha =
            uint32_t(p == 0 ? rhi >> (P.wid[0] * g) : rlo >> (P.wid[1] * (g - P.nd[0]))) & uint32_t(W - 1);
        uint64_t lt = alpha ? (uint64_t(1) << alpha) - 1 : 0, eq = uint64_t(1) << alpha;
        if (P.nd[p] == 1 && !full) {
            if (p == 0 ? rho_c : rho_L) lt ^= wm;
            if (p == 0 && rho_e) eq ^= wm;
        }
        // truth bits as a 128-bit value (lo, hi): lt at [0, W), eq at [W, 2W)
        uint64_t lo = lt, hi = 0;
        if (P.deq(g)) {
            if (W < 64) lo |= eq << W;
            if (W == 32) hi = 0;
            if (W == 64) hi = eq;
        }
        for (int k = 0; k < P.drows(g); k++) {
            const int row = P.drow0(g) + k;
            const uint64_t src = k < 2 ? lo : hi;
            const uint32_t t = uint32_t(src >> (32 * (k & 1)));
            const uint32_t s0 = word(row);
            tab0[uint64_t(row) * N + e] = s0;
            tab1[uint64_t(row) * N + e] = s0 ^ t;
        }
    }
    const int o0 = 32 * P.rows, o1 = o0 + 5 * P.ncomb;
    uint32_t t0[3] = {0u, 0u, 0u}, t1[3] = {0u, 0u, 0u};
    for (int q = 0; q < P.ncomb; q++) {
        const OtComb &C = P.comb[q];
        uint32_t v0[5], v1[5];
        for (int k = 0; k < 5; k++) v0[k] = bit(o0 + 5 * q + k);
        for (int k = 0; k < 3; k++) v1[k] = bit(o1 + 3 * q + k);
        const uint32_t a = v0[0] ^ v1[0], b = v0[1] ^ v1[1], b2 = v0[2] ^ v1[2];
        v1[3] = (a & b) ^ v0[3];
        v1[4] = (a & b2) ^ v0[4];
        if (C.root) v1[3] ^= C.part != 1 ? rho_c : rho_L, v1[4] ^= C.part == 0 ? rho_e : 0u;
        if (!C.eq) v0[4] = 0, v1[4] = 0;
        for (int k = 0; k < 5; k++) {
            if (!C.eq && (k == 2 || k == 4)) continue;  // no b', c' without an eq AND
            const int i = P.tpos(q, k);
            t0[i >> 5] |= v0[k] << (i & 31);
            t1[i >> 5] |= v1[k] << (i & 31);
        }
    }
    if (full) {
        const int i = P.mu_bit();
        t0[i >> 5] |= ((pb >> 2) & 1u) << (i & 31);
        t1[i >> 5] |= ((pb >> 3) & 1u) << (i & 31);
    }
    for (int k = 0; k < P.tri_words(); k++) tri0[uint64_t(k) * N + e] = t0[k], tri1[uint64_t(k) * N + e] = t1[k];
}

// ---- host side (ot.cu)

// the plan of (bw, s), built once per process
const OtPlan &ot_plan_cached(int bw, int s);
// the digit plan of an OT or TT gate's layout (built once per process)
const OtPlan &gate_digit_plan(const GateLayout &L);
// K_p = AES_dk(p || op || P_OT_PARTY), expanded
AesKey ot_party_key(const AesKey &dk, uint32_t op, int party);
// party's first message: its garbled tables [Gmax][N] u32, its digit shares
// (state: N x state_bytes()) and its triple bits (tri: [tri_words()][N] u32)
int ot_garble(const GateLayout &L, int party, const void *xhat, const void *key, uint32_t *tables, void *state,
              uint32_t *tri, cudaStream_t st);
// level 1..levels: (level 1: take the peer's tables) close the previous level
// with both parties' openings, open this level's ANDs into open_out
// (ot_open_bytes(L, level) bytes per element);
// level levels + 1: close the last level and write the masked comparison bits
// (bits_hi: [lt | eq] x ceil(N/32) words, bits_lo: lt)
// Truth-table (TT) kinds run the same levels without a garble step: level 1
// reads the party's digit tables at the digits of x_hat (xhat, TT only; plus
// xhat2 when not null: the opened input still held as both parties' shares),
// the triple words come from the key (tri ignored), and the last level writes
// bits_lo only for GATE_LRS_TT.
int ot_level(const GateLayout &L, int party, int level, const void *key, const uint32_t *peer_tables,
             const void *open_own, const void *open_peer, void *state, const uint32_t *tri, void *open_out,
             uint32_t *bits_hi, uint32_t *bits_lo, cudaStream_t st, const void *xhat = nullptr,
             const void *xhat2 = nullptr);
// bytes per element of the openings of AND level `level` (1..levels): the
// plans compiled into the level kernel (scale 12) store them in the smallest
// of 1, 2 or 4 bytes that holds every opened bit, other plans in 4 bytes
int ot_open_bytes(const GateLayout &L, int level);
// scratch of one party's OT gate, bytes: garbled tables, state, triple bits
struct OtScratch {
    uint64_t tables, state, tri;
};
OtScratch ot_scratch_bytes(const GateLayout &L);

}  // namespace ddg
