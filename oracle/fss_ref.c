/*
 * fss_ref.c -- CPU restatement of the FSS primitives used on the online
 * 2PC inference path.  TEST INFRASTRUCTURE ONLY: it is linked by tests/,
 * by __graft_entry__.smoke() and by bench.py's cpu_baseline leg as a checker.
 * The product (libddg.so) never links or calls it.
 *
 * Why this file exists
 * --------------------
 * The reference's FSS arithmetic (DCF/DPF tree evaluation, DReLU + select,
 * DPF-LUT, truncation) is un-vendored EzPC GPU-MPC code (reference
 * gpu_mpc/ddg_orca_base.h:1 names commit 66d9cddc); it is not present, so the
 * reference's key formats cannot be reproduced.  This build therefore uses
 * its own published-algorithm FSS scheme, restated here byte-for-byte in plain
 * C so the CUDA kernels can be checked share-for-share:
 *
 *  - AES-128 as in FIPS-197 (S-box derived from the GF(2^8) inverse plus the
 *    affine map; pinned by the FIPS-197 appendix C.1 vector that the
 *    reference's own test uses, gpu_mpc/lss/lss_test.cpp:52-70).
 *  - Fixed-key circular-correlation-robust hash H(x) = pi(sigma(x)) ^ sigma(x)
 *    with sigma(lo,hi) = (hi, lo^hi) (Guo, Katz, Wang, Yu, "Efficient and
 *    secure multiparty computation from fixed-key block ciphers", S&P 2020).
 *  - Half-tree DPF (Guo, Yang, Wang, Zhang, Xie, Liu, Zhao, EUROCRYPT 2023):
 *    on-path seeds differ by a fixed Delta with lsb(Delta)=1, the control bit
 *    is lsb(seed), the right child is left ^ parent, one H call per level.
 *  - DCF 1{x < alpha} derived from that DPF: XOR of the control bits of the
 *    right siblings of x's path at every level where x goes left, plus a
 *    128-bit early-termination leaf holding 1{y < alpha_low}.
 *  - Gates (ReLU, ReLU o ARS, ARS, LRS of a non-negative value) built from a
 *    high (n-1)-bit DCF and a low s-bit DCF, as documented in gate_keygen.
 *  - DPF look-up table over an 8-bit domain (secure_adj_norm.h:139-184 table
 *    t[0]=0, t[d]=llround(2^s/sqrt(d)) for 1<=d<=nmax).
 *
 * All integer arithmetic is on uint64_t reduced to n bits (n = 32 or 64).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

/* ------------------------------------------------------------------ AES */

static uint8_t SBOX[256];
static int sbox_ready = 0;

static uint8_t xtime(uint8_t a) { return (uint8_t)((a << 1) ^ ((a & 0x80) ? 0x1b : 0)); }

static uint8_t gmul(uint8_t a, uint8_t b)
{
    uint8_t p = 0;
    while (b) {
        if (b & 1) p ^= a;
        a = xtime(a);
        b >>= 1;
    }
    return p;
}

static uint8_t rotl8(uint8_t x, int k) { return (uint8_t)((x << k) | (x >> (8 - k))); }

static void build_sbox(void)
{
    for (int x = 0; x < 256; x++) {
        /* multiplicative inverse in GF(2^8): x^254 (0 maps to 0) */
        uint8_t inv = 0;
        if (x) {
            uint8_t r = 1, base = (uint8_t)x;
            int e = 254;
            while (e) {
                if (e & 1) r = gmul(r, base);
                base = gmul(base, base);
                e >>= 1;
            }
            inv = r;
        }
        SBOX[x] = (uint8_t)(inv ^ rotl8(inv, 1) ^ rotl8(inv, 2) ^ rotl8(inv, 3) ^ rotl8(inv, 4) ^ 0x63);
    }
    sbox_ready = 1;
}

typedef struct { uint8_t rk[176]; } aes_ks;

void ref_aes128_expand(const uint8_t key[16], aes_ks *ks)
{
    if (!sbox_ready) build_sbox();
    memcpy(ks->rk, key, 16);
    uint8_t rcon = 1;
    for (int i = 4; i < 44; i++) {
        uint8_t t[4];
        memcpy(t, ks->rk + 4 * (i - 1), 4);
        if (i % 4 == 0) {
            uint8_t t0 = t[0];
            t[0] = (uint8_t)(SBOX[t[1]] ^ rcon);
            t[1] = SBOX[t[2]];
            t[2] = SBOX[t[3]];
            t[3] = SBOX[t0];
            rcon = xtime(rcon);
        }
        for (int k = 0; k < 4; k++) ks->rk[4 * i + k] = (uint8_t)(ks->rk[4 * (i - 4) + k] ^ t[k]);
    }
}

void ref_aes128_encrypt(const aes_ks *ks, const uint8_t in[16], uint8_t out[16])
{
    uint8_t st[16], tmp[16];
    for (int i = 0; i < 16; i++) st[i] = (uint8_t)(in[i] ^ ks->rk[i]);
    for (int round = 1; round <= 10; round++) {
        for (int i = 0; i < 16; i++) st[i] = SBOX[st[i]];
        /* ShiftRows: byte (row r, col c) lives at r + 4c */
        for (int c = 0; c < 4; c++)
            for (int r = 0; r < 4; r++) tmp[r + 4 * c] = st[r + 4 * ((c + r) & 3)];
        if (round != 10) {
            for (int c = 0; c < 4; c++) {
                uint8_t a0 = tmp[4 * c], a1 = tmp[4 * c + 1], a2 = tmp[4 * c + 2], a3 = tmp[4 * c + 3];
                st[4 * c + 0] = (uint8_t)(gmul(a0, 2) ^ gmul(a1, 3) ^ a2 ^ a3);
                st[4 * c + 1] = (uint8_t)(a0 ^ gmul(a1, 2) ^ gmul(a2, 3) ^ a3);
                st[4 * c + 2] = (uint8_t)(a0 ^ a1 ^ gmul(a2, 2) ^ gmul(a3, 3));
                st[4 * c + 3] = (uint8_t)(gmul(a0, 3) ^ a1 ^ a2 ^ gmul(a3, 2));
            }
        } else {
            memcpy(st, tmp, 16);
        }
        for (int i = 0; i < 16; i++) st[i] ^= ks->rk[16 * round + i];
    }
    memcpy(out, st, 16);
}

/* ------------------------------------------------------- fixed-key hashes */

static const char KEY_H[17] = "ddg-halftree-H:0"; /* tree-node hash key */
static const char KEY_C[17] = "ddg-halftree-C:1"; /* leaf conversion key */
static aes_ks ks_h, ks_c;
static int fixed_ready = 0;

static void fixed_init(void)
{
    ref_aes128_expand((const uint8_t *)KEY_H, &ks_h);
    ref_aes128_expand((const uint8_t *)KEY_C, &ks_c);
    fixed_ready = 1;
}

static void sigma(const uint8_t x[16], uint8_t y[16])
{
    /* x = lo (bytes 0..7) || hi (bytes 8..15);  sigma(x) = hi || (lo ^ hi) */
    for (int i = 0; i < 8; i++) {
        y[i] = x[8 + i];
        y[8 + i] = (uint8_t)(x[i] ^ x[8 + i]);
    }
}

static void ccr(const aes_ks *ks, const uint8_t x[16], uint8_t out[16])
{
    uint8_t sx[16], e[16];
    sigma(x, sx);
    ref_aes128_encrypt(ks, sx, e);
    for (int i = 0; i < 16; i++) out[i] = (uint8_t)(e[i] ^ sx[i]);
}

void ref_hash_h(const uint8_t x[16], uint8_t out[16])
{
    if (!fixed_ready) fixed_init();
    ccr(&ks_h, x, out);
}

void ref_hash_c(const uint8_t x[16], uint8_t out[16])
{
    if (!fixed_ready) fixed_init();
    ccr(&ks_c, x, out);
}

/* ------------------------------------------------------------ dealer PRG */

/* dealer key bytes: seed (8 bytes LE) || "dealerK1" */
void ref_dealer_key(uint64_t seed, aes_ks *ks)
{
    uint8_t k[16];
    for (int i = 0; i < 8; i++) k[i] = (uint8_t)(seed >> (8 * i));
    memcpy(k + 8, "dealerK1", 8);
    ref_aes128_expand(k, ks);
}

/* one pseudo-random block for (op, purpose, index): AES_K(index || op || purpose) */
void ref_prg(const aes_ks *ks, uint32_t op, uint32_t purpose, uint64_t idx, uint8_t out[16])
{
    uint8_t pt[16];
    for (int i = 0; i < 8; i++) pt[i] = (uint8_t)(idx >> (8 * i));
    for (int i = 0; i < 4; i++) pt[8 + i] = (uint8_t)(op >> (8 * i));
    for (int i = 0; i < 4; i++) pt[12 + i] = (uint8_t)(purpose >> (8 * i));
    ref_aes128_encrypt(ks, pt, out);
}

static uint64_t nmask(int n) { return n >= 64 ? ~0ULL : ((1ULL << n) - 1); }

static uint64_t ring_of(const uint8_t b[16], int n)
{
    uint64_t v = 0;
    for (int i = 0; i < 8; i++) v |= (uint64_t)b[i] << (8 * i);
    return v & nmask(n);
}

/* ------------------------------------------------------------------- DCF */

static int tree_levels(int d) { return d > 7 ? d - 7 : 0; }

static void xor16(uint8_t *a, const uint8_t *b)
{
    for (int i = 0; i < 16; i++) a[i] ^= b[i];
}

static int block_bit(const uint8_t b[16], int y) { return (b[y >> 3] >> (y & 7)) & 1; }

/*
 * Keys for 1{x < alpha} over d-bit x.  Levels j = 0..L-1 consume x's bits from
 * the most significant down; the last min(d,7) bits index the 128-bit leaf.
 * cw receives L blocks (16 bytes each).
 */
void ref_dcf_keygen(int d, uint64_t alpha, const uint8_t s0[16], const uint8_t delta_in[16],
                    uint8_t root0[16], uint8_t root1[16], uint8_t *cw, uint8_t leafcw[16])
{
    if (!fixed_ready) fixed_init();
    int L = tree_levels(d), lb = d - L;
    uint8_t delta[16], cur[2][16], h[2][16];
    memcpy(delta, delta_in, 16);
    delta[0] |= 1;
    memcpy(cur[0], s0, 16);
    memcpy(cur[1], s0, 16);
    xor16(cur[1], delta);
    memcpy(root0, cur[0], 16);
    memcpy(root1, cur[1], 16);
    for (int j = 0; j < L; j++) {
        int a = (int)((alpha >> (d - 1 - j)) & 1);
        ccr(&ks_h, cur[0], h[0]);
        ccr(&ks_h, cur[1], h[1]);
        uint8_t *c = cw + 16 * j;
        for (int i = 0; i < 16; i++) c[i] = (uint8_t)(h[0][i] ^ h[1][i] ^ (a ? 0 : delta[i]));
        for (int b = 0; b < 2; b++) {
            int t = cur[b][0] & 1;
            uint8_t cl[16];
            for (int i = 0; i < 16; i++) cl[i] = (uint8_t)(h[b][i] ^ (t ? c[i] : 0));
            if (a) xor16(cur[b], cl); /* right child: left ^ parent */
            else memcpy(cur[b], cl, 16);
        }
    }
    uint8_t g0[16], g1[16], m[16];
    memset(m, 0, 16);
    uint64_t al = alpha & ((1ULL << lb) - 1);
    for (uint64_t y = 0; y < al; y++) m[y >> 3] |= (uint8_t)(1u << (y & 7));
    ccr(&ks_c, cur[0], g0);
    ccr(&ks_c, cur[1], g1);
    for (int i = 0; i < 16; i++) leafcw[i] = (uint8_t)(g0[i] ^ g1[i] ^ m[i]);
}

/* party's XOR share of 1{x < alpha} */
int ref_dcf_eval(int d, uint64_t x, const uint8_t root[16], const uint8_t *cw, const uint8_t leafcw[16])
{
    if (!fixed_ready) fixed_init();
    int L = tree_levels(d), lb = d - L;
    uint8_t s[16], h[16], cl[16];
    memcpy(s, root, 16);
    int c = 0;
    for (int j = 0; j < L; j++) {
        int xj = (int)((x >> (d - 1 - j)) & 1);
        int t = s[0] & 1;
        ccr(&ks_h, s, h);
        for (int i = 0; i < 16; i++) cl[i] = (uint8_t)(h[i] ^ (t ? cw[16 * j + i] : 0));
        if (!xj) {
            c ^= (cl[0] ^ s[0]) & 1; /* lsb of the right sibling */
            memcpy(s, cl, 16);
        } else {
            xor16(s, cl);
        }
    }
    int t = s[0] & 1;
    uint8_t g[16];
    ccr(&ks_c, s, g);
    if (t) xor16(g, leafcw);
    c ^= block_bit(g, (int)(x & ((1ULL << lb) - 1)));
    return c;
}

/*
 * DCF with an equality output over d-bit x: the same half-tree walk, but the
 * 128-bit leaf holds 64 slots of 2 bits for the low 6 bits y of x:
 * bit 2y = 1{y < alpha_low6}, bit 2y+1 = 1{y == alpha_low6}.  Returns the party's
 * XOR shares of (1{x < alpha}, 1{x == alpha}) as bit0 / bit1.  Used as the upper
 * part of a split comparison: 1{x < a} over (U,V) = 1{U<A} ^ (1{U==A} & 1{V<B}).
 */
void ref_dcfeq_keygen(int d, uint64_t alpha, const uint8_t s0[16], const uint8_t delta_in[16],
                      uint8_t root0[16], uint8_t root1[16], uint8_t *cw, uint8_t leafcw[16])
{
    if (!fixed_ready) fixed_init();
    int L = d > 6 ? d - 6 : 0;
    uint8_t delta[16], cur[2][16], h[2][16];
    memcpy(delta, delta_in, 16);
    delta[0] |= 1;
    memcpy(cur[0], s0, 16);
    memcpy(cur[1], s0, 16);
    xor16(cur[1], delta);
    memcpy(root0, cur[0], 16);
    memcpy(root1, cur[1], 16);
    for (int j = 0; j < L; j++) {
        int a = (int)((alpha >> (d - 1 - j)) & 1);
        ccr(&ks_h, cur[0], h[0]);
        ccr(&ks_h, cur[1], h[1]);
        uint8_t *c = cw + 16 * j;
        for (int i = 0; i < 16; i++) c[i] = (uint8_t)(h[0][i] ^ h[1][i] ^ (a ? 0 : delta[i]));
        for (int b = 0; b < 2; b++) {
            int t = cur[b][0] & 1;
            uint8_t cl[16];
            for (int i = 0; i < 16; i++) cl[i] = (uint8_t)(h[b][i] ^ (t ? c[i] : 0));
            if (a) xor16(cur[b], cl);
            else memcpy(cur[b], cl, 16);
        }
    }
    uint8_t g0[16], g1[16], m[16];
    memset(m, 0, 16);
    int al = (int)(alpha & 63);
    for (int y = 0; y < 64; y++) {
        if (y < al) m[(2 * y) >> 3] |= (uint8_t)(1u << ((2 * y) & 7));
        if (y == al) m[(2 * y + 1) >> 3] |= (uint8_t)(1u << ((2 * y + 1) & 7));
    }
    ccr(&ks_c, cur[0], g0);
    ccr(&ks_c, cur[1], g1);
    for (int i = 0; i < 16; i++) leafcw[i] = (uint8_t)(g0[i] ^ g1[i] ^ m[i]);
}

int ref_dcfeq_eval(int d, uint64_t x, const uint8_t root[16], const uint8_t *cw, const uint8_t leafcw[16])
{
    if (!fixed_ready) fixed_init();
    int L = d > 6 ? d - 6 : 0;
    uint8_t s[16], h[16], cl[16];
    memcpy(s, root, 16);
    int c = 0;
    for (int j = 0; j < L; j++) {
        int xj = (int)((x >> (d - 1 - j)) & 1);
        int t = s[0] & 1;
        ccr(&ks_h, s, h);
        for (int i = 0; i < 16; i++) cl[i] = (uint8_t)(h[i] ^ (t ? cw[16 * j + i] : 0));
        if (!xj) {
            c ^= (cl[0] ^ s[0]) & 1;
            memcpy(s, cl, 16);
        } else {
            xor16(s, cl);
        }
    }
    int t = s[0] & 1;
    uint8_t g[16];
    ccr(&ks_c, s, g);
    if (t) xor16(g, leafcw);
    int y = (int)(x & 63);
    return (c ^ block_bit(g, 2 * y)) | (block_bit(g, 2 * y + 1) << 1);
}

/* ----------------------------------------------------------------- gates */

enum { GATE_RELU = 0, GATE_RELU_ARS = 1, GATE_ARS = 2, GATE_LRS = 3, GATE_RELU_SPLIT = 4, GATE_RELU_ARS_SPLIT = 5,
       GATE_LRS_SPLIT = 6, GATE_RELU_SPLIT3 = 7, GATE_RELU_ARS_SPLIT3 = 8 };

/* three-part split ReLU gates: the (n-1)-bit compare over (U1, U2, V) with
 * U2 = SPLIT3_MID bits above the low s bits V and U1 the rest:
 * 1{x_l < r_l} = c1 + e1*(c2 + e2*cL), every sum exclusive */
#define SPLIT3_MID 6
static int is_split3(int kind) { return kind == GATE_RELU_SPLIT3 || kind == GATE_RELU_ARS_SPLIT3; }

/* kinds whose high DCF has an equality output */
static int is_split(int kind)
{
    return kind == GATE_RELU_SPLIT || kind == GATE_RELU_ARS_SPLIT || kind == GATE_LRS_SPLIT || is_split3(kind);
}
/* GATE_LRS_SPLIT: the s-bit carry comparison over (V1, V2), V2 the low
 * lrs_lo_bits(s) bits: 1{V < B} = 1{V1 < B1} + 1{V1 == B1} * 1{V2 < B2} */
static int lrs_lo_bits(int s) { return s - 1 < 7 ? s - 1 : 7; }

enum {
    P_HI_S0 = 1, P_HI_DELTA = 2, P_LO_S0 = 3, P_LO_DELTA = 4,
    P_ROUT = 5, P_BITS = 6, P_MID_S0 = 9, P_MID_DELTA = 10, P_SHARE = 16
};

typedef struct {
    uint8_t hi_root[16];
    uint8_t hi_cw[56][16];
    uint8_t hi_leaf[16];
    int32_t hi_mu;
    int32_t hi_mu_eq;
    uint8_t lo_root[16];
    uint8_t lo_cw[56][16];
    uint8_t lo_leaf[16];
    int32_t lo_mu;
    uint8_t mid_root[16];
    uint8_t mid_cw[56][16];
    uint8_t mid_leaf[16];
    int32_t mid_mu;
    int32_t mid_mu_eq;
    uint64_t w[80];
} ref_gate_key;

int ref_gate_has_hi(int kind) { return kind != GATE_LRS; }
int ref_gate_has_lo(int kind) { return kind != GATE_RELU; }
int ref_gate_nwords(int kind)
{
    switch (kind) {
    case GATE_RELU: return 4;
    case GATE_RELU_ARS: return 8;
    case GATE_ARS: return 6;
    case GATE_RELU_SPLIT: return 16;
    case GATE_RELU_ARS_SPLIT: return 32;
    case GATE_LRS_SPLIT: return 7;
    case GATE_RELU_SPLIT3: return 40;
    case GATE_RELU_ARS_SPLIT3: return 80;
    default: return 4;
    }
}

/*
 * Three-part split: the DReLU bit d = q ^ eps ^ t with q = 1^m_hat^c1_hat
 * public, eps = r_m ^ rho_c1, and t = e1*(c2 + e2*cL) in {0,1}.  With every
 * true bit b = b_hat + (1-2 b_hat) rho_b, t is multilinear in the mask bits
 * (rho_e1, rho_c2, rho_e2, rho_L) over the nine monomials SPLIT3_T below, and
 *   d = q + (1-2q) [tau_1 + (1-2 tau_1) eps + sum tau_m m - 2 sum tau_m eps m].
 * Dealer words carry the 19 monomials [eps, m (9), eps*m (9)].
 */
#define SPLIT3_NMONO 19
/* mask-bit monomials of t, as bit sets over (e1, c2, L, e2) = bits 0..3 */
static const int SPLIT3_T[9] = {2, 4, 8, 12, 1, 3, 5, 9, 13};

static void split3_monomials(uint64_t ep, uint64_t pe1, uint64_t p2, uint64_t pL, uint64_t pe2, uint64_t mono[19])
{
    const uint64_t var[4] = {pe1, p2, pL, pe2};
    mono[0] = ep;
    for (int k = 0; k < 9; k++) {
        uint64_t v = 1;
        for (int b = 0; b < 4; b++)
            if (SPLIT3_T[k] >> b & 1) v *= var[b];
        mono[1 + k] = v;
        mono[10 + k] = ep * v;
    }
}

/* evaluator: a0 and the coefficients of the 19 monomials (mod 2^64) */
static uint64_t split3_coeffs(uint64_t q, uint64_t e1h, uint64_t c2h, uint64_t e2h, uint64_t cLh, uint64_t a[19])
{
    const uint64_t su = 1 - 2 * q, se1 = 1 - 2 * e1h, sc2 = 1 - 2 * c2h, se2 = 1 - 2 * e2h, sL = 1 - 2 * cLh;
    /* g = c2 + e2*cL = g0 + gc*rho_c2 + gL*rho_L + ge*rho_e2 + geL*rho_e2*rho_L */
    const uint64_t g0 = c2h + e2h * cLh, gc = sc2, gL = e2h * sL, ge = cLh * se2, geL = se2 * sL;
    /* t = e1*g: constant and the SPLIT3_T monomials in order */
    const uint64_t t1 = e1h * g0;
    const uint64_t tau[9] = {e1h * gc, e1h * gL, e1h * ge, e1h * geL, se1 * g0, se1 * gc, se1 * gL, se1 * ge,
                             se1 * geL};
    a[0] = su * (1 - 2 * t1);
    for (int k = 0; k < 9; k++) {
        a[1 + k] = su * tau[k];
        a[10 + k] = 0 - 2 * su * tau[k];
    }
    return q + su * t1;
}
/* domain bits of the high DCF: n-1, the upper n-1-s bits for the split ReLU
 * gates, the upper s - lrs_lo_bits(s) carry bits for GATE_LRS_SPLIT */
int ref_gate_hi_bits(int kind, int n, int s)
{
    if (kind == GATE_LRS_SPLIT) return s - lrs_lo_bits(s);
    if (is_split3(kind)) return n - 1 - s - SPLIT3_MID;
    return is_split(kind) ? n - 1 - s : n - 1;
}

/*
 * Dealer side for one element.  r_in is the input mask (x_hat = x + r_in),
 * the output mask is drawn from the PRG and returned.
 *
 * Notation: r_m = msb(r_in), r_l = r_in mod 2^(n-1), r_H = r_in >> s,
 * r_L = r_in mod 2^s.  The high DCF opens c_hat = 1{xh_l < r_l} ^ rho_c, the
 * low DCF opens cL_hat = 1{xh_L < r_L} ^ rho_L; e = r_m ^ rho_c.
 * Word lists (additively shared in Z_2^n):
 *   RELU     : e, r, e*r, r_y
 *   RELU_ARS : e, r_H, e*r_H, rho_L, e*rho_L, r_m, e*r_m, r_y
 *   ARS      : r_H, rho_L, rho_c, r_m, r_m*rho_c, r_y
 *   LRS      : r_H, rho_L, r_m, r_y
 */
uint64_t ref_gate_keygen(int kind, int n, int s, uint64_t seed, uint32_t op, uint64_t i,
                         uint64_t r_in, ref_gate_key *k0, ref_gate_key *k1)
{
    aes_ks ks;
    ref_dealer_key(seed, &ks);
    uint64_t M = nmask(n);
    uint8_t blk[16], blk2[16];
    memset(k0, 0, sizeof(*k0));
    memset(k1, 0, sizeof(*k1));
    r_in &= M;

    ref_prg(&ks, op, P_ROUT, i, blk);
    uint64_t r_y = ring_of(blk, n);
    ref_prg(&ks, op, P_BITS, i, blk);
    int mu0h = blk[0] & 1, mu1h = (blk[0] >> 1) & 1, mu0l = (blk[0] >> 2) & 1, mu1l = (blk[0] >> 3) & 1;
    int mu0e = (blk[0] >> 4) & 1, mu1e = (blk[0] >> 5) & 1;
    /* three-part split: the middle DCF's compare (bits 6/7) and equality (bits 8/9) masks */
    int mu0m = (blk[0] >> 6) & 1, mu1m = (blk[0] >> 7) & 1, mu0me = blk[1] & 1, mu1me = (blk[1] >> 1) & 1;
    int rho_c = mu0h ^ mu1h, rho_L = mu0l ^ mu1l, rho_e = mu0e ^ mu1e;
    int rho_m = mu0m ^ mu1m, rho_me = mu0me ^ mu1me;

    uint64_t r_m = (r_in >> (n - 1)) & 1;
    uint64_t r_l = r_in & (M >> 1);
    uint64_t r_H = r_in >> s;
    uint64_t r_L = r_in & ((1ULL << s) - 1);
    uint64_t e = r_m ^ (uint64_t)rho_c;

    if (kind == GATE_LRS_SPLIT) {
        int lo = lrs_lo_bits(s), hi = s - lo;
        ref_prg(&ks, op, P_HI_S0, i, blk);
        ref_prg(&ks, op, P_HI_DELTA, i, blk2);
        ref_dcfeq_keygen(hi, r_L >> lo, blk, blk2, k0->hi_root, k1->hi_root, &k0->hi_cw[0][0], k0->hi_leaf);
        memcpy(k1->hi_cw, k0->hi_cw, sizeof(k0->hi_cw));
        memcpy(k1->hi_leaf, k0->hi_leaf, 16);
        k0->hi_mu = mu0h, k1->hi_mu = mu1h;
        k0->hi_mu_eq = mu0e, k1->hi_mu_eq = mu1e;
        ref_prg(&ks, op, P_LO_S0, i, blk);
        ref_prg(&ks, op, P_LO_DELTA, i, blk2);
        ref_dcf_keygen(lo, r_L & ((1ULL << lo) - 1), blk, blk2, k0->lo_root, k1->lo_root, &k0->lo_cw[0][0],
                       k0->lo_leaf);
        memcpy(k1->lo_cw, k0->lo_cw, sizeof(k0->lo_cw));
        memcpy(k1->lo_leaf, k0->lo_leaf, 16);
        k0->lo_mu = mu0l, k1->lo_mu = mu1l;
    } else if (ref_gate_has_hi(kind)) {
        ref_prg(&ks, op, P_HI_S0, i, blk);
        ref_prg(&ks, op, P_HI_DELTA, i, blk2);
        if (is_split3(kind))
            ref_dcfeq_keygen(n - 1 - s - SPLIT3_MID, r_l >> (s + SPLIT3_MID), blk, blk2, k0->hi_root, k1->hi_root,
                             &k0->hi_cw[0][0], k0->hi_leaf);
        else if (is_split(kind))
            ref_dcfeq_keygen(n - 1 - s, r_l >> s, blk, blk2, k0->hi_root, k1->hi_root, &k0->hi_cw[0][0], k0->hi_leaf);
        else
            ref_dcf_keygen(n - 1, r_l, blk, blk2, k0->hi_root, k1->hi_root, &k0->hi_cw[0][0], k0->hi_leaf);
        memcpy(k1->hi_cw, k0->hi_cw, sizeof(k0->hi_cw));
        memcpy(k1->hi_leaf, k0->hi_leaf, 16);
        k0->hi_mu = mu0h;
        k1->hi_mu = mu1h;
        if (is_split(kind)) {
            k0->hi_mu_eq = mu0e;
            k1->hi_mu_eq = mu1e;
        }
    }
    if (is_split3(kind)) {
        ref_prg(&ks, op, P_MID_S0, i, blk);
        ref_prg(&ks, op, P_MID_DELTA, i, blk2);
        ref_dcfeq_keygen(SPLIT3_MID, (r_in >> s) & ((1ULL << SPLIT3_MID) - 1), blk, blk2, k0->mid_root, k1->mid_root,
                         &k0->mid_cw[0][0], k0->mid_leaf);
        memcpy(k1->mid_cw, k0->mid_cw, sizeof(k0->mid_cw));
        memcpy(k1->mid_leaf, k0->mid_leaf, 16);
        k0->mid_mu = mu0m, k1->mid_mu = mu1m;
        k0->mid_mu_eq = mu0me, k1->mid_mu_eq = mu1me;
    }
    if (ref_gate_has_lo(kind) && kind != GATE_LRS_SPLIT) {
        ref_prg(&ks, op, P_LO_S0, i, blk);
        ref_prg(&ks, op, P_LO_DELTA, i, blk2);
        ref_dcf_keygen(s, r_L, blk, blk2, k0->lo_root, k1->lo_root, &k0->lo_cw[0][0], k0->lo_leaf);
        memcpy(k1->lo_cw, k0->lo_cw, sizeof(k0->lo_cw));
        memcpy(k1->lo_leaf, k0->lo_leaf, 16);
        k0->lo_mu = mu0l;
        k1->lo_mu = mu1l;
    }
    uint64_t v[80];
    int nw = ref_gate_nwords(kind);
    uint64_t m3[SPLIT3_NMONO];
    split3_monomials(r_m ^ (uint64_t)rho_c, (uint64_t)rho_e, (uint64_t)rho_m, (uint64_t)rho_L, (uint64_t)rho_me, m3);
    /* split gates: monomials of the dealer bits that the DReLU bit depends on,
     * eps = r_m ^ rho_c:  eps, rho_L, rho_e, rho_e*rho_L, eps*rho_L, eps*rho_e, eps*rho_e*rho_L */
    uint64_t ep = r_m ^ (uint64_t)rho_c, pl = (uint64_t)rho_L, pe = (uint64_t)rho_e;
    uint64_t mono[7] = {ep, pl, pe, pe * pl, ep * pl, ep * pe, ep * pe * pl};
    switch (kind) {
    case GATE_RELU:
        v[0] = e; v[1] = r_in; v[2] = e * r_in; v[3] = r_y;
        break;
    case GATE_RELU_ARS:
        v[0] = e; v[1] = r_H; v[2] = e * r_H; v[3] = (uint64_t)rho_L;
        v[4] = e * (uint64_t)rho_L; v[5] = r_m; v[6] = e * r_m; v[7] = r_y;
        break;
    case GATE_ARS:
        v[0] = r_H; v[1] = (uint64_t)rho_L; v[2] = (uint64_t)rho_c; v[3] = r_m;
        v[4] = r_m * (uint64_t)rho_c; v[5] = r_y;
        break;
    case GATE_RELU_SPLIT:
        for (int k = 0; k < 7; k++) v[k] = mono[k], v[8 + k] = mono[k] * r_in;
        v[7] = r_in;
        v[15] = r_y;
        break;
    case GATE_LRS_SPLIT:
        /* carry = c1 + e1*c2; masks rho_c (c1), rho_e (e1), rho_L (c2) */
        v[0] = r_H; v[1] = (uint64_t)rho_c; v[2] = pe; v[3] = pl; v[4] = pe * pl; v[5] = r_m; v[6] = r_y;
        break;
    case GATE_RELU_SPLIT3:
        for (int k = 0; k < SPLIT3_NMONO; k++) v[k] = m3[k], v[20 + k] = m3[k] * r_in;
        v[19] = r_in;
        v[39] = r_y;
        break;
    case GATE_RELU_ARS_SPLIT3: {
        uint64_t nj[3] = {r_H, pl, r_m};
        for (int k = 0; k < SPLIT3_NMONO; k++) v[k] = m3[k];
        for (int j = 0; j < 3; j++) v[19 + j] = nj[j];
        for (int k = 0; k < SPLIT3_NMONO; k++)
            for (int j = 0; j < 3; j++) v[22 + 3 * k + j] = m3[k] * nj[j];
        v[79] = r_y;
        break;
    }
    case GATE_RELU_ARS_SPLIT: {
        uint64_t nj[3] = {r_H, pl, r_m};
        for (int k = 0; k < 7; k++) v[k] = mono[k];
        for (int j = 0; j < 3; j++) v[7 + j] = nj[j];
        for (int k = 0; k < 7; k++)
            for (int j = 0; j < 3; j++) v[10 + 3 * k + j] = mono[k] * nj[j];
        v[31] = r_y;
        break;
    }
    default:
        v[0] = r_H; v[1] = (uint64_t)rho_L; v[2] = r_m; v[3] = r_y;
        break;
    }
    for (int w = 0; w < nw; w++) {
        ref_prg(&ks, op, P_SHARE + (uint32_t)w, i, blk);
        uint64_t a = ring_of(blk, n);
        k0->w[w] = a;
        k1->w[w] = (v[w] - a) & M;
    }
    return r_y;
}

/* round 1: the party's output bits: bit0 = high DCF (compare), bit1 = low DCF,
 * bit2 = high DCF equality (split gates), bit3 / bit4 = middle DCF compare /
 * equality (three-part split gates) */
int ref_gate_round1(int kind, int n, int s, uint64_t xhat, const ref_gate_key *k)
{
    uint64_t M = nmask(n);
    xhat &= M;
    int out = 0;
    if (kind == GATE_LRS_SPLIT) {
        int lo = lrs_lo_bits(s), hi = s - lo;
        int b = ref_dcfeq_eval(hi, (xhat >> lo) & ((1ULL << hi) - 1), k->hi_root, &k->hi_cw[0][0], k->hi_leaf);
        out |= ((b & 1) ^ k->hi_mu) | ((((b >> 1) & 1) ^ k->hi_mu_eq) << 2);
        out |= ((ref_dcf_eval(lo, xhat & ((1ULL << lo) - 1), k->lo_root, &k->lo_cw[0][0], k->lo_leaf) ^ k->lo_mu) & 1)
               << 1;
        return out;
    }
    if (ref_gate_has_hi(kind)) {
        if (is_split3(kind)) {
            int d = n - 1 - s - SPLIT3_MID;
            int b = ref_dcfeq_eval(d, (xhat & (M >> 1)) >> (s + SPLIT3_MID), k->hi_root, &k->hi_cw[0][0], k->hi_leaf);
            out |= ((b & 1) ^ k->hi_mu) | ((((b >> 1) & 1) ^ k->hi_mu_eq) << 2);
            b = ref_dcfeq_eval(SPLIT3_MID, (xhat >> s) & ((1ULL << SPLIT3_MID) - 1), k->mid_root, &k->mid_cw[0][0],
                               k->mid_leaf);
            out |= (((b & 1) ^ k->mid_mu) << 3) | ((((b >> 1) & 1) ^ k->mid_mu_eq) << 4);
        } else if (is_split(kind)) {
            int b = ref_dcfeq_eval(n - 1 - s, (xhat & (M >> 1)) >> s, k->hi_root, &k->hi_cw[0][0], k->hi_leaf);
            out |= ((b & 1) ^ k->hi_mu) | ((((b >> 1) & 1) ^ k->hi_mu_eq) << 2);
        } else {
            out |= (ref_dcf_eval(n - 1, xhat & (M >> 1), k->hi_root, &k->hi_cw[0][0], k->hi_leaf) ^ k->hi_mu) & 1;
        }
    }
    if (ref_gate_has_lo(kind))
        out |= ((ref_dcf_eval(s, xhat & ((1ULL << s) - 1), k->lo_root, &k->lo_cw[0][0], k->lo_leaf) ^ k->lo_mu) & 1)
               << 1;
    return out;
}

/* round 2: party's additive share of the masked output, given the opened bits
 * (bit0 = c_hat, bit1 = cL_hat, bit2 = e_hat, bit3 / bit4 = the middle DCF's
 * c2_hat / e2_hat) */
uint64_t ref_gate_round2(int kind, int n, int s, int party, uint64_t xhat, int bits, const ref_gate_key *k)
{
    uint64_t M = nmask(n);
    xhat &= M;
    uint64_t p0 = party == 0 ? 1 : 0;
    uint64_t mh = (xhat >> (n - 1)) & 1;
    uint64_t xH = xhat >> s;
    uint64_t two_ns = 1ULL << (n - s); /* n - s < 64 */
    const uint64_t *w = k->w;
    uint64_t ch = (uint64_t)(bits & 1), cl = (uint64_t)((bits >> 1) & 1), eh = (uint64_t)((bits >> 2) & 1);
    uint64_t q = 1 ^ mh ^ ch;                 /* public part of DReLU */
    uint64_t a1 = 1 - 2 * q;                  /* 1 - 2q  (mod 2^n) */
    uint64_t b1 = 1 - 2 * cl;                 /* 1 - 2*cL_hat */
    uint64_t y = 0;
    /* split gates: DReLU = a0 + sum_k a[k] * mono[k] (see ref_gate_keygen) */
    uint64_t su = 1 - 2 * q, se = 1 - 2 * eh, sc = 1 - 2 * cl;
    uint64_t G0 = eh * cl, GL = eh * sc, Ge = cl * se, GeL = se * sc;
    uint64_t a0 = q + su * G0;
    uint64_t a[7] = {su * (1 - 2 * G0), su * GL, su * Ge, su * GeL, 0 - 2 * su * GL, 0 - 2 * su * Ge, 0 - 2 * su * GeL};
    switch (kind) {
    case GATE_RELU:
        y = p0 * q * xhat + a1 * xhat * w[0] - q * w[1] - a1 * w[2] + w[3];
        break;
    case GATE_RELU_ARS:
        y = p0 * (q * xH - q * cl) + w[0] * (a1 * xH - a1 * cl) - q * w[1] - a1 * w[2] - q * b1 * w[3] -
            a1 * b1 * w[4] + two_ns * (1 - mh) * (q * w[5] + a1 * w[6]) + w[7];
        break;
    case GATE_ARS: {
        uint64_t pub = xH - cl + two_ns * (mh * ch - mh);
        y = p0 * pub - w[0] - b1 * w[1] +
            two_ns * (mh * (1 - 2 * ch) * w[2] + ((1 - 2 * mh) * ch + mh) * w[3] + (1 - 2 * mh) * (1 - 2 * ch) * w[4]) +
            w[5];
        break;
    }
    case GATE_RELU_SPLIT: {
        uint64_t sx = 0, sr = 0;
        for (int t = 0; t < 7; t++) sx += a[t] * w[t], sr += a[t] * w[8 + t];
        y = p0 * a0 * xhat + xhat * sx - a0 * w[7] - sr + w[15];
        break;
    }
    case GATE_RELU_SPLIT3:
    case GATE_RELU_ARS_SPLIT3: {
        uint64_t a3[SPLIT3_NMONO];
        uint64_t b0 = split3_coeffs(q, eh, (uint64_t)((bits >> 3) & 1), (uint64_t)((bits >> 4) & 1), cl, a3);
        uint64_t sm = 0;
        for (int t = 0; t < SPLIT3_NMONO; t++) sm += a3[t] * w[t];
        if (kind == GATE_RELU_SPLIT3) {
            uint64_t sr = 0;
            for (int t = 0; t < SPLIT3_NMONO; t++) sr += a3[t] * w[20 + t];
            y = p0 * b0 * xhat + xhat * sm - b0 * w[19] - sr + w[39];
        } else {
            uint64_t Y0 = xH - cl;
            uint64_t yj[3] = {0 - 1, 0 - sc, two_ns * (1 - mh)};
            uint64_t sn = 0, smn = 0;
            for (int j = 0; j < 3; j++) sn += yj[j] * w[19 + j];
            for (int t = 0; t < SPLIT3_NMONO; t++)
                for (int j = 0; j < 3; j++) smn += a3[t] * yj[j] * w[22 + 3 * t + j];
            y = p0 * b0 * Y0 + Y0 * sm + b0 * sn + smn + w[79];
        }
        break;
    }
    case GATE_LRS_SPLIT: {
        /* bits: ch = c1_hat, eh = e1_hat, cl = c2_hat */
        uint64_t sc1 = 1 - 2 * ch, se1 = 1 - 2 * eh, sc2 = 1 - 2 * cl;
        y = p0 * (xH - ch - eh * cl) - w[0] - sc1 * w[1] - cl * se1 * w[2] - eh * sc2 * w[3] - se1 * sc2 * w[4] +
            two_ns * (1 - mh) * w[5] + w[6];
        break;
    }
    case GATE_RELU_ARS_SPLIT: {
        uint64_t Y0 = xH - cl;
        uint64_t yj[3] = {0 - 1, 0 - sc, two_ns * (1 - mh)};
        uint64_t sm = 0, sn = 0, smn = 0;
        for (int t = 0; t < 7; t++) sm += a[t] * w[t];
        for (int j = 0; j < 3; j++) sn += yj[j] * w[7 + j];
        for (int t = 0; t < 7; t++)
            for (int j = 0; j < 3; j++) smn += a[t] * yj[j] * w[10 + 3 * t + j];
        y = p0 * a0 * Y0 + Y0 * sm + a0 * sn + smn + w[31];
        break;
    }
    default:
        y = p0 * (xH - cl) - w[0] - b1 * w[1] + two_ns * (1 - mh) * w[2] + w[3];
        break;
    }
    return y & M;
}

/* --------------------------------------------------- OT-leaf comparison gates
 *
 * GATE_RELU_OT (9) / GATE_RELU_ARS_OT (10): the functions and dealer words of
 * GATE_RELU_SPLIT / GATE_RELU_ARS_SPLIT, with the split comparison bits
 *   hi: 1{U < A}, 1{U == A} over bits [s, n-1);  lo: 1{V < B} over bits [0, s)
 * (each XORed with its dealer mask bit rho_c, rho_e, rho_L) computed by the
 * millionaires' structure of the reference's LSS backend
 * (gpu_mpc/lss/lss_compare.cpp, lss_protocol.md sections 1-2 and 5): radix-16
 * digits, one garbled 16-entry (lt, eq) table per digit read by the other
 * party at a dealer-given index c = (mask digit + delta) mod 16, then a tree
 * of Beaver ANDs combining node pairs (H = 2i+1, L = 2i):
 *   lt = lt_H ^ (eq_H & lt_L),  eq = eq_H & eq_L,
 * an odd top node passing up; the root AND of a part carries its mask bit in
 * the triple (c = ab ^ rho).  Each party's randomness: K_p = AES_dealer(p ||
 * op || 0x100); aux block j = AES_Kp(i || 0 || 0x110 + j): per garbled local
 * digit t, delta at bits 6t..6t+3 and (s_lt, s_eq) at 6t+4, 6t+5, then per
 * combine q (a, b, b', c1, c1') at 6*Gmax + 5q; pad block j = AES_Kp(i || 0 ||
 * 0x120 + j), digit t's pads = 32-bit word t mod 4 of block t / 4.  Party 0
 * holds its triple c bits explicitly (c0: bits 2q, 2q+1); party 1 uses c1.
 * Written independently of the CUDA code from that description. */
enum { GATE_RELU_OT = 9, GATE_RELU_ARS_OT = 10 };
enum { OT_P_PARTY = 0x100, OT_P_AUX = 0x110, OT_P_PAD = 0x120 };
#define OT_MAXD 18
#define OT_MAXC 16

typedef struct {
    int mode; /* 0 = OT, 1 = truth-table ReLU, 2 = truth-table carry, 3 = truth-table full compare */
    int wid[2], bits[2];
    int deq[OT_MAXD], drows[OT_MAXD], drow0[OT_MAXD], rows;
    int n, s, D, G0, nd[2], levels, ncomb, tri0, naux;
    int cpart[OT_MAXC], ch[OT_MAXC], cl[OT_MAXC], cout[OT_MAXC], ceq[OT_MAXC], croot[OT_MAXC], clevel[OT_MAXC];
    int pfrom[8][2], pto[8][2];
    /* TT triple-bit positions: (a, b, b') of combine q at tpa[q] + 0..2, (c, c')
     * at tpc[q] + 0..1, the full compare's lo mask bit at mu_pos (tt_place) */
    int tpa[OT_MAXC], tpc[OT_MAXC], mu_pos;
} ot_plan_t;

/* digit width of digit g (the top digit of a part keeps the remainder) */
static int ot_width(const ot_plan_t *P, int g)
{
    int p = g < P->nd[0] ? 0 : 1, j = g < P->nd[0] ? g : g - P->nd[0];
    int rem = P->bits[p] - P->wid[p] * j;
    return rem < P->wid[p] ? rem : P->wid[p];
}

/* Parts: OT and TT ReLU compare bits [s, n-1) (hi) and [0, s) (lo); the TT
 * carry only [0, s).  Digit widths: OT 4 and 4; TT ReLU 5 (bw=32) or 4, and 4;
 * TT carry 6.  A digit keeps its equality entries unless it is the lowest
 * digit of the lo part (whose root needs only lt). */
static void tt_place(ot_plan_t *P);

static int digit_plan_build(int n, int s, int mode, ot_plan_t *P)
{
    memset(P, 0, sizeof(*P));
    P->mode = mode, P->n = n, P->s = s;
    P->bits[0] = mode == 2 ? 0 : n - 1 - s;
    P->bits[1] = s;
    P->wid[0] = (mode == 1 || mode == 3) && n == 32 ? 5 : 4;
    P->wid[1] = mode == 2 ? 6 : 4;
    if ((mode != 2 && P->bits[0] < 1) || P->bits[1] < 1) return 0;
    P->nd[0] = (P->bits[0] + P->wid[0] - 1) / P->wid[0];
    P->nd[1] = (P->bits[1] + P->wid[1] - 1) / P->wid[1];
    P->D = P->nd[0] + P->nd[1];
    if (P->D > OT_MAXD) return 0;
    P->G0 = mode == 0 ? (P->D + 1) / 2 : 0;
    for (int g = 0, row = 0; g < P->D; g++) {
        int p = g < P->nd[0] ? 0 : 1, j = g < P->nd[0] ? g : g - P->nd[0];
        P->deq[g] = j > 0 || p == 0;
        P->drows[g] = ((1 << ot_width(P, g)) * (P->deq[g] ? 2 : 1) + 31) / 32;
        P->drow0[g] = row;
        row += P->drows[g];
        P->rows = row;
    }
    int k[2] = {P->nd[0], P->nd[1]}, q = 0, l = 0;
    while (k[0] > 1 || k[1] > 1) {
        l++;
        if (l > 7) return 0;
        for (int p = 0; p < 2; p++) {
            P->pfrom[l][p] = P->pto[l][p] = -1;
            if (k[p] <= 1) continue;
            int nk = (k[p] + 1) / 2;
            for (int i = 0; i < k[p] / 2; i++) {
                if (q >= OT_MAXC) return 0;
                P->cpart[q] = p, P->ch[q] = 2 * i + 1, P->cl[q] = 2 * i, P->cout[q] = i;
                P->ceq[q] = (i > 0 || p == 0), P->croot[q] = (nk == 1 && mode != 3), P->clevel[q] = l;
                q++;
            }
            if (k[p] & 1) P->pfrom[l][p] = k[p] - 1, P->pto[l][p] = k[p] / 2;
            k[p] = nk;
        }
    }
    if (mode == 3) {
        /* the cross combine: full compare = hi_lt ^ (hi_eq & lo_lt), written over the hi root */
        l++;
        if (l > 7 || q >= OT_MAXC) return 0;
        P->pfrom[l][0] = P->pfrom[l][1] = P->pto[l][0] = P->pto[l][1] = -1;
        P->cpart[q] = 2, P->ch[q] = 0, P->cl[q] = 0, P->cout[q] = 0, P->ceq[q] = 0, P->croot[q] = 1;
        P->clevel[q] = l;
        q++;
    }
    P->levels = l, P->ncomb = q, P->tri0 = 6 * P->G0;
    P->naux = (P->tri0 + 5 * q + 127) / 128;
    int ok = P->naux <= 2 && 5 * q + 1 <= 96 && P->rows <= 24;
    if (ok) tt_place(P);
    return ok;
}

static int ot_plan_build(int n, int s, ot_plan_t *P) { return digit_plan_build(n, s, 0, P); }

/* Triple-bit positions of a truth-table plan, restating the CUDA plan's
 * tt_place (idash26-track3_b200/csrc/digit_plan.cuh): combine q of part p at
 * AND level l has the lane 2 base[p] + out * 2^(l+1) (base[0] = 0, base[1] =
 * the hi digit count; the cross combine lane 0).  Per level in order, the
 * level's (a, b, b') group (7 << lane of each combine computing eq, 3 <<
 * lane of the others: they have no b') and then its (c, c') group (3 or 1
 * << lane) are placed first-fit (lowest word, then lowest shift) in the free
 * bits of the tri words, and last the mask bit of the full compare.  When a
 * group does not fit, or the digit state needs more than 32 bits (2 D > 32),
 * every combine keeps (a, b, b', c, c') at 5q and the mask bit sits at
 * 5 ncomb. */
static int place_bits(uint32_t used[3], int words, uint32_t m)
{
    int hi = 0;
    for (int b = 0; b < 32; b++)
        if ((m >> b) & 1) hi = b;
    for (int w = 0; w < words; w++)
        for (int sh = 0; sh + hi < 32; sh++)
            if (((m << sh) & used[w]) == 0) {
                used[w] |= m << sh;
                return 32 * w + sh;
            }
    return -1;
}

static int comb_lane(const ot_plan_t *P, int q)
{
    if (P->cpart[q] == 2) return 0;
    return 2 * (P->cpart[q] == 0 ? 0 : P->nd[0]) + P->cout[q] * (2 << P->clevel[q]);
}

static void tt_place(ot_plan_t *P)
{
    for (int q = 0; q < P->ncomb; q++) P->tpa[q] = 5 * q, P->tpc[q] = 5 * q + 3;
    P->mu_pos = 5 * P->ncomb;
    if (P->mode == 0 || 2 * P->D > 32) return; /* the lane layout needs the digit state in 32 bits */
    uint32_t used[3] = {0, 0, 0};
    int pa[OT_MAXC], pc[OT_MAXC];
    const int words = (5 * P->ncomb + (P->mode == 3) + 31) / 32;
    for (int l = 1; l <= P->levels; l++) {
        uint32_t ma = 0, mc = 0;
        for (int q = 0; q < P->ncomb; q++) {
            if (P->clevel[q] != l) continue;
            ma |= (P->ceq[q] ? 7u : 3u) << comb_lane(P, q), mc |= (P->ceq[q] ? 3u : 1u) << comb_lane(P, q);
        }
        if (!ma) continue;
        int ga = place_bits(used, words, ma);
        if (ga < 0) return;
        int gc = place_bits(used, words, mc);
        if (gc < 0) return;
        for (int q = 0; q < P->ncomb; q++)
            if (P->clevel[q] == l) pa[q] = ga + comb_lane(P, q), pc[q] = gc + comb_lane(P, q);
    }
    int mu = 5 * P->ncomb;
    if (P->mode == 3 && (mu = place_bits(used, words, 1u)) < 0) return;
    for (int q = 0; q < P->ncomb; q++) P->tpa[q] = pa[q], P->tpc[q] = pc[q];
    P->mu_pos = mu;
}

static int tri_pos(const ot_plan_t *P, int q, int k) { return k < 3 ? P->tpa[q] + k : P->tpc[q] + k - 3; }

static int ot_part(const ot_plan_t *P, int g) { return g < P->nd[0] ? 0 : 1; }
static int ot_shift(const ot_plan_t *P, int g)
{
    return g < P->nd[0] ? P->s + P->wid[0] * g : P->wid[1] * (g - P->nd[0]);
}
static int ot_garbler(const ot_plan_t *P, int g) { return g < P->G0 ? 0 : 1; }
static int ot_local(const ot_plan_t *P, int g) { return g < P->G0 ? g : g - P->G0; }

typedef struct {
    uint8_t ks[176];     /* expanded AES key K_p (round keys, bytes) */
    uint8_t recv[OT_MAXD]; /* choice | pad_lt << 4 | pad_eq << 5 per receiver slot */
    uint32_t c0;         /* party 0's triple c bits (0 for party 1) */
    uint64_t w[32];      /* dealer words of the SPLIT kind */
} ref_ot_key;

int ref_ot_plan_info(int n, int s, int *out6)
{
    ot_plan_t P;
    if (!ot_plan_build(n, s, &P)) return 0;
    out6[0] = P.D, out6[1] = P.G0, out6[2] = P.levels, out6[3] = P.ncomb, out6[4] = P.naux, out6[5] = P.tri0;
    return 1;
}

/* bit y of the party's aux blocks */
static int ot_aux_bit(const uint8_t aux[2][16], int y) { return block_bit(aux[y >> 7], y & 127); }

static void ot_party_blocks(const ot_plan_t *P, const aes_ks *kp, uint64_t i, uint8_t aux[2][16])
{
    memset(aux, 0, 32);
    for (int j = 0; j < P->naux; j++) ref_prg(kp, 0, OT_P_AUX + (uint32_t)j, i, aux[j]);
}

static uint32_t ot_pad_word(const aes_ks *kp, uint64_t i, int t)
{
    uint8_t b[16];
    ref_prg(kp, 0, OT_P_PAD + (uint32_t)(t / 4), i, b);
    const uint8_t *w = b + 4 * (t % 4);
    return (uint32_t)w[0] | ((uint32_t)w[1] << 8) | ((uint32_t)w[2] << 16) | ((uint32_t)w[3] << 24);
}

/* The mask bits of the SPLIT kinds come from the same P_BITS block as in ref_gate_keygen. */
uint64_t ref_ot_keygen(int kind, int n, int s, uint64_t seed, uint32_t op, uint64_t i, uint64_t r_in,
                       ref_ot_key *k0, ref_ot_key *k1)
{
    ot_plan_t P;
    memset(k0, 0, sizeof(*k0));
    memset(k1, 0, sizeof(*k1));
    if (!ot_plan_build(n, s, &P)) return 0;
    static ref_gate_key g0, g1; /* words of the SPLIT kind (its DCF parts are unused) */
    int wk = kind == GATE_RELU_OT ? GATE_RELU_SPLIT : GATE_RELU_ARS_SPLIT;
    uint64_t r_out = ref_gate_keygen(wk, n, s, seed, op, i, r_in, &g0, &g1);
    memcpy(k0->w, g0.w, sizeof(k0->w));
    memcpy(k1->w, g1.w, sizeof(k1->w));

    aes_ks dk, kp[2];
    ref_dealer_key(seed, &dk);
    uint8_t blk[16];
    for (int p = 0; p < 2; p++) {
        ref_prg(&dk, op, OT_P_PARTY, (uint64_t)p, blk);
        ref_aes128_expand(blk, &kp[p]);
    }
    memcpy(k0->ks, kp[0].rk, 176);
    memcpy(k1->ks, kp[1].rk, 176);
    ref_prg(&dk, op, P_BITS, i, blk);
    int rho_c = (blk[0] ^ (blk[0] >> 1)) & 1, rho_L = ((blk[0] >> 2) ^ (blk[0] >> 3)) & 1,
        rho_e = ((blk[0] >> 4) ^ (blk[0] >> 5)) & 1;
    uint64_t M = nmask(n);
    r_in &= M;
    uint64_t rhi = (r_in >> s) & ((1ULL << (n - 1 - s)) - 1), rlo = r_in & ((1ULL << s) - 1);
    uint8_t aux[2][2][16];
    ot_party_blocks(&P, &kp[0], i, aux[0]);
    ot_party_blocks(&P, &kp[1], i, aux[1]);
    ref_ot_key *kk[2] = {k0, k1};
    for (int g = 0; g < P.D; g++) {
        int pg = ot_garbler(&P, g), t = ot_local(&P, g), w = ot_width(&P, g), part = ot_part(&P, g);
        uint32_t wm = (1u << w) - 1;
        uint32_t delta = 0;
        for (int b = 0; b < 4; b++) delta |= (uint32_t)ot_aux_bit(aux[pg], 6 * t + b) << b;
        delta &= wm;
        uint32_t alpha = (uint32_t)((part == 0 ? rhi >> (4 * g) : rlo >> (4 * (g - P.nd[0])))) & wm;
        uint32_t c = (alpha + delta) & wm;
        uint32_t pw = ot_pad_word(&kp[pg], i, t);
        int klt = (pw >> c) & 1, keq = (pw >> (16 + c)) & 1;
        if (P.nd[part] == 1) {
            klt ^= part == 0 ? rho_c : rho_L;
            keq ^= part == 0 ? rho_e : 0;
        }
        kk[1 - pg]->recv[t] = (uint8_t)(c | (klt << 4) | (keq << 5));
    }
    uint32_t cw = 0;
    for (int q = 0; q < P.ncomb; q++) {
        int tb = P.tri0 + 5 * q;
        int a = ot_aux_bit(aux[0], tb) ^ ot_aux_bit(aux[1], tb);
        int b = ot_aux_bit(aux[0], tb + 1) ^ ot_aux_bit(aux[1], tb + 1);
        int b2 = ot_aux_bit(aux[0], tb + 2) ^ ot_aux_bit(aux[1], tb + 2);
        int c = (a & b) ^ ot_aux_bit(aux[1], tb + 3), c2 = (a & b2) ^ ot_aux_bit(aux[1], tb + 4);
        if (P.croot[q]) {
            c ^= P.cpart[q] == 0 ? rho_c : rho_L;
            c2 ^= P.cpart[q] == 0 ? rho_e : 0;
        }
        cw |= ((uint32_t)c << (2 * q)) | ((uint32_t)(P.ceq[q] ? c2 : 0) << (2 * q + 1));
    }
    k0->c0 = cw;
    k1->c0 = 0;
    return r_out;
}

/* the garbler's table word: entry u (u < 2^w) = (1{xd < u - delta}, 1{xd == u - delta}) ^ (s_lt, s_eq) ^ pad */
static uint32_t ot_table_word(uint32_t xd, int w, uint32_t delta, int slt, int seq, uint32_t pad)
{
    uint32_t W = 1u << w, word = 0;
    for (uint32_t u = 0; u < W; u++) {
        uint32_t v = (u + W - delta) % W;
        word |= (uint32_t)((xd < v) ^ slt) << u;
        word |= (uint32_t)((xd == v) ^ seq) << (16 + u);
    }
    uint32_t m = (W == 32 ? 0 : ((1u << W) - 1));
    return word ^ (pad & (m | (m << 16)));
}

/*
 * Both parties' online protocol for one element, openings in place.  Returns
 * through bits0 / bits1 each party's masked comparison-bit shares in the
 * round-1 encoding of ref_gate_round1 (bit0 hi lt, bit1 lo lt, bit2 hi eq);
 * tables0 / tables1 (optional, G0 words) receive each party's garbled tables.
 */
void ref_ot_eval_pair(int kind, int n, int s, uint64_t xhat, uint64_t i, const ref_ot_key *k0,
                      const ref_ot_key *k1, int *bits0, int *bits1, uint32_t *tables0, uint32_t *tables1)
{
    (void)kind;
    ot_plan_t P;
    *bits0 = *bits1 = 0;
    if (!ot_plan_build(n, s, &P)) return;
    const ref_ot_key *kk[2] = {k0, k1};
    xhat &= nmask(n);
    aes_ks kp[2];
    uint8_t aux[2][2][16];
    uint32_t tab[2][OT_MAXD];
    uint64_t st[2] = {0, 0};
    for (int p = 0; p < 2; p++) {
        memcpy(kp[p].rk, kk[p]->ks, 176);
        ot_party_blocks(&P, &kp[p], i, aux[p]);
    }
    /* message 1: garbled tables; own digit shares */
    for (int g = 0; g < P.D; g++) {
        int pg = ot_garbler(&P, g), t = ot_local(&P, g), w = ot_width(&P, g);
        uint32_t wm = (1u << w) - 1, delta = 0;
        for (int b = 0; b < 4; b++) delta |= (uint32_t)ot_aux_bit(aux[pg], 6 * t + b) << b;
        delta &= wm;
        int slt = ot_aux_bit(aux[pg], 6 * t + 4), seq = ot_aux_bit(aux[pg], 6 * t + 5);
        uint32_t xd = (uint32_t)(xhat >> ot_shift(&P, g)) & wm;
        tab[pg][t] = ot_table_word(xd, w, delta, slt, seq, ot_pad_word(&kp[pg], i, t));
        st[pg] |= ((uint64_t)slt << (2 * g)) | ((uint64_t)seq << (2 * g + 1));
    }
    if (tables0)
        for (int t = 0; t < P.G0; t++) tables0[t] = t < P.G0 ? tab[0][t] : 0;
    if (tables1)
        for (int t = 0; t < P.D - P.G0; t++) tables1[t] = tab[1][t];
    /* receivers: T[c] ^ k_c */
    for (int g = 0; g < P.D; g++) {
        int pg = ot_garbler(&P, g), t = ot_local(&P, g), pr = 1 - pg;
        uint32_t rec = kk[pr]->recv[t], c = rec & 15, word = tab[pg][t];
        uint64_t lt = ((word >> c) ^ (rec >> 4)) & 1, eq = ((word >> (16 + c)) ^ (rec >> 5)) & 1;
        st[pr] |= (lt << (2 * g)) | (eq << (2 * g + 1));
    }
    /* AND-tree levels */
    for (int l = 1; l <= P.levels; l++) {
        int e_[OT_MAXC], f_[OT_MAXC], f2_[OT_MAXC];
        for (int q = 0; q < P.ncomb; q++) {
            if (P.clevel[q] != l) continue;
            int base = 2 * (P.cpart[q] == 0 ? 0 : P.nd[0]), tb = P.tri0 + 5 * q;
            e_[q] = f_[q] = f2_[q] = 0;
            for (int p = 0; p < 2; p++) {
                e_[q] ^= (int)((st[p] >> (base + 2 * P.ch[q] + 1)) & 1) ^ ot_aux_bit(aux[p], tb);
                f_[q] ^= (int)((st[p] >> (base + 2 * P.cl[q])) & 1) ^ ot_aux_bit(aux[p], tb + 1);
                if (P.ceq[q]) f2_[q] ^= (int)((st[p] >> (base + 2 * P.cl[q] + 1)) & 1) ^ ot_aux_bit(aux[p], tb + 2);
            }
        }
        for (int p = 0; p < 2; p++) {
            for (int q = 0; q < P.ncomb; q++) {
                if (P.clevel[q] != l) continue;
                int base = 2 * (P.cpart[q] == 0 ? 0 : P.nd[0]), tb = P.tri0 + 5 * q;
                int a = ot_aux_bit(aux[p], tb), b = ot_aux_bit(aux[p], tb + 1), b2 = ot_aux_bit(aux[p], tb + 2);
                int c = p == 0 ? (int)((k0->c0 >> (2 * q)) & 1) : ot_aux_bit(aux[1], tb + 3);
                int c2 = p == 0 ? (int)((k0->c0 >> (2 * q + 1)) & 1) : ot_aux_bit(aux[1], tb + 4);
                int p0 = p == 0;
                int lt = (int)((st[p] >> (base + 2 * P.ch[q])) & 1) ^ c ^ (f_[q] & a) ^ (e_[q] & b) ^ (p0 & e_[q] & f_[q]);
                int eq = P.ceq[q] ? (c2 ^ (f2_[q] & a) ^ (e_[q] & b2) ^ (p0 & e_[q] & f2_[q])) : 0;
                int o = base + 2 * P.cout[q];
                st[p] = (st[p] & ~(3ULL << o)) | ((uint64_t)lt << o) | ((uint64_t)eq << (o + 1));
            }
            for (int pt = 0; pt < 2; pt++) {
                if (P.pfrom[l][pt] < 0) continue;
                int b = 2 * (pt == 0 ? 0 : P.nd[0]), o = b + 2 * P.pto[l][pt];
                uint64_t v = (st[p] >> (b + 2 * P.pfrom[l][pt])) & 3;
                st[p] = (st[p] & ~(3ULL << o)) | (v << o);
            }
        }
    }
    int *out[2] = {bits0, bits1};
    for (int p = 0; p < 2; p++)
        *out[p] = (int)(st[p] & 1) | ((int)((st[p] >> (2 * P.nd[0])) & 1) << 1) | ((int)((st[p] >> 1) & 1) << 2);
}

/* ----------------------------------------------- truth-table comparison gates
 *
 * GATE_RELU_TT (11) / GATE_RELU_ARS_TT (12) / GATE_LRS_TT (13): the functions
 * and dealer words of GATE_RELU_SPLIT / GATE_RELU_ARS_SPLIT / GATE_LRS.  The
 * comparison bits come from dealer truth tables: digit g of the compared part
 * of x_hat (public) indexes a table of its 2^w values holding (lt, eq) =
 * (1{x < a_g}, 1{x == a_g}) for the mask digit a_g, XOR-shared between the
 * parties (party 0's rows from the dealer stream, party 1's = party 0's XOR
 * the truth table; a one-digit part XORs its mask bit into every entry).  The
 * digits are combined by the AND tree of the OT gates with Beaver triples
 * whose bits are all explicit: party 0's (a, b, b', c, c') and party 1's
 * (a, b, b') from the dealer stream, party 1's c = ab ^ c0 (^ rho at a root).
 * Dealer stream: 32-bit word w = word w mod 4 of AES_dealer(i || op ||
 * 0x140 + w / 4); party 0's table rows, then its 5 triple bits per combine,
 * then party 1's 3.  Written independently of the CUDA code. */
enum { GATE_RELU_TT = 11, GATE_RELU_ARS_TT = 12, GATE_LRS_TT = 13, GATE_RELU_TTF = 14, GATE_RELU_ARS_TTF = 15 };

/* state positions of a combine's H and L inputs and of its output (the cross
 * combine, part 2, reads the hi root and the lo root and overwrites the hi root) */
static int comb_hpos(const ot_plan_t *P, int q)
{
    return P->cpart[q] == 2 ? 0 : 2 * (P->cpart[q] == 0 ? 0 : P->nd[0]) + 2 * P->ch[q];
}
static int comb_lpos(const ot_plan_t *P, int q)
{
    return P->cpart[q] == 2 ? 2 * P->nd[0] : 2 * (P->cpart[q] == 0 ? 0 : P->nd[0]) + 2 * P->cl[q];
}
static int comb_opos(const ot_plan_t *P, int q)
{
    return P->cpart[q] == 2 ? 0 : 2 * (P->cpart[q] == 0 ? 0 : P->nd[0]) + 2 * P->cout[q];
}
#define TT_P_RAND 0x140

typedef struct {
    uint32_t tab[24]; /* table rows */
    uint32_t tri[3];  /* triple bits, 5 per combine */
    uint64_t w[32];   /* dealer words of the word kind */
} ref_tt_key;

static int tt_mode(int kind)
{
    return kind == GATE_LRS_TT ? 2 : (kind == GATE_RELU_TTF || kind == GATE_RELU_ARS_TTF) ? 3 : 1;
}
static int tt_word_kind(int kind)
{
    switch (kind) {
    case GATE_RELU_TT: return GATE_RELU_SPLIT;
    case GATE_RELU_ARS_TT: return GATE_RELU_ARS_SPLIT;
    case GATE_RELU_TTF: return GATE_RELU;
    case GATE_RELU_ARS_TTF: return GATE_RELU_ARS;
    default: return GATE_LRS;
    }
}

int ref_tt_plan_info(int kind, int n, int s, int *out4)
{
    ot_plan_t P;
    if (!digit_plan_build(n, s, tt_mode(kind), &P)) return 0;
    out4[0] = P.D, out4[1] = P.rows, out4[2] = P.levels, out4[3] = P.ncomb;
    return 1;
}

/* the plan's triple-bit positions: out[0] = ncomb, out[1 + 2q] = tpa[q],
 * out[2 + 2q] = tpc[q] (q < ncomb), then mu_pos; returns 1, or 0 without a plan */
int ref_tt_tri_positions(int kind, int n, int s, int *out)
{
    ot_plan_t P;
    if (!digit_plan_build(n, s, tt_mode(kind), &P)) return 0;
    out[0] = P.ncomb;
    for (int q = 0; q < P.ncomb; q++) out[1 + 2 * q] = P.tpa[q], out[2 + 2 * q] = P.tpc[q];
    out[1 + 2 * P.ncomb] = P.mu_pos;
    return 1;
}

static uint32_t tt_stream_word(const aes_ks *dk, uint32_t op, uint64_t i, int w)
{
    uint8_t b[16];
    ref_prg(dk, op, TT_P_RAND + (uint32_t)(w / 4), i, b);
    const uint8_t *p = b + 4 * (w % 4);
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}
static int tt_stream_bit(const aes_ks *dk, uint32_t op, uint64_t i, int b)
{
    return (int)((tt_stream_word(dk, op, i, b / 32) >> (b % 32)) & 1);
}

uint64_t ref_tt_keygen(int kind, int n, int s, uint64_t seed, uint32_t op, uint64_t i, uint64_t r_in,
                       ref_tt_key *k0, ref_tt_key *k1)
{
    ot_plan_t P;
    memset(k0, 0, sizeof(*k0));
    memset(k1, 0, sizeof(*k1));
    if (!digit_plan_build(n, s, tt_mode(kind), &P)) return 0;
    static ref_gate_key g0, g1;
    uint64_t r_out = ref_gate_keygen(tt_word_kind(kind), n, s, seed, op, i, r_in, &g0, &g1);
    memcpy(k0->w, g0.w, sizeof(k0->w));
    memcpy(k1->w, g1.w, sizeof(k1->w));
    aes_ks dk;
    ref_dealer_key(seed, &dk);
    uint8_t blk[16];
    ref_prg(&dk, op, P_BITS, i, blk);
    int rho_c = (blk[0] ^ (blk[0] >> 1)) & 1, rho_L = ((blk[0] >> 2) ^ (blk[0] >> 3)) & 1,
        rho_e = ((blk[0] >> 4) ^ (blk[0] >> 5)) & 1;
    r_in &= nmask(n);
    uint64_t rhi = P.nd[0] ? (r_in >> s) & ((1ULL << P.bits[0]) - 1) : 0, rlo = r_in & ((1ULL << s) - 1);
    for (int g = 0; g < P.D; g++) {
        int part = ot_part(&P, g), w = ot_width(&P, g), W = 1 << w;
        uint32_t alpha = (uint32_t)(part == 0 ? rhi >> (P.wid[0] * g) : rlo >> (P.wid[1] * (g - P.nd[0]))) & (W - 1);
        /* truth bits: entry x -> lt at bit x, eq at bit W + x */
        uint32_t truth[4] = {0, 0, 0, 0};
        for (int x = 0; x < W; x++) {
            int lt = x < (int)alpha, eq = x == (int)alpha;
            if (P.nd[part] == 1 && P.mode != 3) {
                lt ^= part == 0 ? rho_c : rho_L;
                eq ^= part == 0 ? rho_e : 0;
            }
            truth[x / 32] |= (uint32_t)lt << (x % 32);
            if (P.deq[g]) truth[(W + x) / 32] |= (uint32_t)eq << ((W + x) % 32);
        }
        for (int k = 0; k < P.drows[g]; k++) {
            int row = P.drow0[g] + k;
            uint32_t s0 = tt_stream_word(&dk, op, i, row);
            k0->tab[row] = s0;
            k1->tab[row] = s0 ^ truth[k];
        }
    }
    int o0 = 32 * P.rows, o1 = o0 + 5 * P.ncomb;
    for (int q = 0; q < P.ncomb; q++) {
        int v0[5], v1[5];
        for (int k = 0; k < 5; k++) v0[k] = tt_stream_bit(&dk, op, i, o0 + 5 * q + k);
        for (int k = 0; k < 3; k++) v1[k] = tt_stream_bit(&dk, op, i, o1 + 3 * q + k);
        int a = v0[0] ^ v1[0], b = v0[1] ^ v1[1], b2 = v0[2] ^ v1[2];
        v1[3] = (a & b) ^ v0[3];
        v1[4] = (a & b2) ^ v0[4];
        if (P.croot[q]) {
            v1[3] ^= P.cpart[q] != 1 ? rho_c : rho_L;
            v1[4] ^= P.cpart[q] == 0 ? rho_e : 0;
        }
        if (!P.ceq[q]) v0[4] = v1[4] = 0;
        for (int k = 0; k < 5; k++) {
            if (!P.ceq[q] && (k == 2 || k == 4)) continue; /* no b', c' without an eq AND */
            int bit = tri_pos(&P, q, k);
            k0->tri[bit / 32] |= (uint32_t)v0[k] << (bit % 32);
            k1->tri[bit / 32] |= (uint32_t)v1[k] << (bit % 32);
        }
    }
    if (P.mode == 3) { /* each party's share of the lo compare's mask bit (P_BITS bits 2 and 3) */
        int b = P.mu_pos;
        k0->tri[b / 32] |= (uint32_t)((blk[0] >> 2) & 1) << (b % 32);
        k1->tri[b / 32] |= (uint32_t)((blk[0] >> 3) & 1) << (b % 32);
    }
    return r_out;
}

/*
 * Both parties' AND-tree protocol for one element, openings in place: each
 * party's masked comparison-bit shares in the round-1 encoding (bit0 hi lt,
 * bit1 lo lt, bit2 hi eq; the carry kind only bit1).
 */
#define TRI_BIT(k, b) ((int)(((k)->tri[(b) / 32] >> ((b) % 32)) & 1))
void ref_tt_eval_pair(int kind, int n, int s, uint64_t xhat, const ref_tt_key *k0, const ref_tt_key *k1, int *bits0,
                      int *bits1)
{
    ot_plan_t P;
    *bits0 = *bits1 = 0;
    if (!digit_plan_build(n, s, tt_mode(kind), &P)) return;
    const ref_tt_key *kk[2] = {k0, k1};
    xhat &= nmask(n);
    uint64_t st[2] = {0, 0};
    for (int p = 0; p < 2; p++)
        for (int g = 0; g < P.D; g++) {
            int W = 1 << ot_width(&P, g);
            uint32_t x = (uint32_t)(xhat >> ot_shift(&P, g)) & (uint32_t)(W - 1);
            const uint32_t *t = kk[p]->tab + P.drow0[g];
            uint64_t lt = (t[x / 32] >> (x % 32)) & 1, eq = 0;
            if (P.deq[g]) eq = (t[(W + x) / 32] >> ((W + x) % 32)) & 1;
            st[p] |= (lt << (2 * g)) | (eq << (2 * g + 1));
        }
#define TRI(p, b) ((int)((kk[p]->tri[(b) / 32] >> ((b) % 32)) & 1))
    for (int l = 1; l <= P.levels; l++) {
        int e_[OT_MAXC], f_[OT_MAXC], f2_[OT_MAXC];
        for (int q = 0; q < P.ncomb; q++) {
            if (P.clevel[q] != l) continue;
            int hp = comb_hpos(&P, q), lp = comb_lpos(&P, q);
            e_[q] = f_[q] = f2_[q] = 0;
            for (int p = 0; p < 2; p++) {
                e_[q] ^= (int)((st[p] >> (hp + 1)) & 1) ^ TRI(p, tri_pos(&P, q, 0));
                f_[q] ^= (int)((st[p] >> lp) & 1) ^ TRI(p, tri_pos(&P, q, 1));
                if (P.ceq[q]) f2_[q] ^= (int)((st[p] >> (lp + 1)) & 1) ^ TRI(p, tri_pos(&P, q, 2));
            }
        }
        for (int p = 0; p < 2; p++) {
            for (int q = 0; q < P.ncomb; q++) {
                if (P.clevel[q] != l) continue;
                int p0 = p == 0;
                int a = TRI(p, tri_pos(&P, q, 0)), b = TRI(p, tri_pos(&P, q, 1)), b2 = TRI(p, tri_pos(&P, q, 2)),
                    c = TRI(p, tri_pos(&P, q, 3)), c2 = TRI(p, tri_pos(&P, q, 4));
                int lt = (int)((st[p] >> comb_hpos(&P, q)) & 1) ^ c ^ (f_[q] & a) ^ (e_[q] & b) ^ (p0 & e_[q] & f_[q]);
                int eq = P.ceq[q] ? (c2 ^ (f2_[q] & a) ^ (e_[q] & b2) ^ (p0 & e_[q] & f2_[q])) : 0;
                int o = comb_opos(&P, q);
                st[p] = (st[p] & ~(3ULL << o)) | ((uint64_t)lt << o) | ((uint64_t)eq << (o + 1));
            }
            for (int pt = 0; pt < 2; pt++) {
                if (P.pfrom[l][pt] < 0) continue;
                int b = 2 * (pt == 0 ? 0 : P.nd[0]), o = b + 2 * P.pto[l][pt];
                uint64_t v = (st[p] >> (b + 2 * P.pfrom[l][pt])) & 3;
                st[p] = (st[p] & ~(3ULL << o)) | (v << o);
            }
        }
    }
#undef TRI
    int *out[2] = {bits0, bits1};
    for (int p = 0; p < 2; p++) {
        int hi = P.nd[0] ? (int)(st[p] & 1) | ((int)((st[p] >> 1) & 1) << 2) : 0;
        int lo = (int)((st[p] >> (2 * P.nd[0])) & 1);
        if (P.mode == 3) { /* full compare and the lo compare with the party's mask share; no equality */
            hi = (int)(st[p] & 1);
            lo ^= TRI_BIT(kk[p], P.mu_pos);
        }
        *out[p] = hi | (lo << 1);
    }
}

/* ------------------------------------------------------------ DPF-LUT */

typedef struct {
    uint8_t root[16];
    uint8_t cw[8][16];
    uint8_t cwv[16];
    uint64_t rout;
} ref_lut_key;

static int lut_epl(int n) { return 128 / n; }
static int lut_lb(int n) { return n == 32 ? 2 : 1; }

static uint64_t slot(const uint8_t b[16], int n, int k)
{
    uint64_t v = 0;
    int bytes = n / 8;
    for (int i = 0; i < bytes; i++) v |= (uint64_t)b[k * bytes + i] << (8 * i);
    return v;
}

static void set_slot(uint8_t b[16], int n, int k, uint64_t v)
{
    int bytes = n / 8;
    for (int i = 0; i < bytes; i++) b[k * bytes + i] = (uint8_t)(v >> (8 * i));
}

/* keys for the point function e_alpha over the 8-bit domain with payload 1 */
void ref_lut_keygen(int n, uint64_t seed, uint32_t op, uint64_t i, uint64_t alpha, uint64_t r_out,
                    ref_lut_key *k0, ref_lut_key *k1)
{
    if (!fixed_ready) fixed_init();
    aes_ks ks;
    ref_dealer_key(seed, &ks);
    uint64_t M = nmask(n);
    int lb = lut_lb(n), L = 8 - lb, epl = lut_epl(n);
    uint8_t s0[16], delta[16], cur[2][16], h[2][16], blk[16];
    memset(k0, 0, sizeof(*k0));
    memset(k1, 0, sizeof(*k1));
    alpha &= 255;
    ref_prg(&ks, op, P_HI_S0, i, s0);
    ref_prg(&ks, op, P_HI_DELTA, i, delta);
    delta[0] |= 1;
    memcpy(cur[0], s0, 16);
    memcpy(cur[1], s0, 16);
    xor16(cur[1], delta);
    memcpy(k0->root, cur[0], 16);
    memcpy(k1->root, cur[1], 16);
    for (int j = 0; j < L; j++) {
        int a = (int)((alpha >> (7 - j)) & 1);
        ccr(&ks_h, cur[0], h[0]);
        ccr(&ks_h, cur[1], h[1]);
        for (int q = 0; q < 16; q++) k0->cw[j][q] = (uint8_t)(h[0][q] ^ h[1][q] ^ (a ? 0 : delta[q]));
        for (int b = 0; b < 2; b++) {
            int t = cur[b][0] & 1;
            uint8_t cl[16];
            for (int q = 0; q < 16; q++) cl[q] = (uint8_t)(h[b][q] ^ (t ? k0->cw[j][q] : 0));
            if (a) xor16(cur[b], cl);
            else memcpy(cur[b], cl, 16);
        }
    }
    memcpy(k1->cw, k0->cw, sizeof(k0->cw));
    int t0 = cur[0][0] & 1;
    uint8_t g0[16], g1[16];
    ccr(&ks_c, cur[0], g0);
    ccr(&ks_c, cur[1], g1);
    int alo = (int)(alpha & (uint64_t)(epl - 1));
    for (int kk = 0; kk < epl; kk++) {
        uint64_t want = kk == alo ? 1 : 0;
        uint64_t v = (want - slot(g0, n, kk) + slot(g1, n, kk)) & M;
        if (!t0) v = (0 - v) & M; /* t0 - t1 = -1 */
        set_slot(k0->cwv, n, kk, v);
    }
    memcpy(k1->cwv, k0->cwv, 16);
    ref_prg(&ks, op, P_SHARE, i, blk);
    uint64_t a = ring_of(blk, n);
    k0->rout = a;
    k1->rout = (r_out - a) & M;
}

/* party's share of table[(xhat - alpha) mod 256] + r_out */
uint64_t ref_lut_eval(int n, int party, uint64_t xhat, const uint64_t *table, const ref_lut_key *k)
{
    if (!fixed_ready) fixed_init();
    uint64_t M = nmask(n);
    int lb = lut_lb(n), L = 8 - lb, epl = lut_epl(n);
    uint64_t acc = 0;
    for (int p = 0; p < (1 << L); p++) {
        uint8_t s[16], h[16], cl[16];
        memcpy(s, k->root, 16);
        for (int j = 0; j < L; j++) {
            int xj = (p >> (L - 1 - j)) & 1;
            int t = s[0] & 1;
            ccr(&ks_h, s, h);
            for (int q = 0; q < 16; q++) cl[q] = (uint8_t)(h[q] ^ (t ? k->cw[j][q] : 0));
            if (xj) xor16(s, cl);
            else memcpy(s, cl, 16);
        }
        int t = s[0] & 1;
        uint8_t g[16];
        ccr(&ks_c, s, g);
        for (int kk = 0; kk < epl; kk++) {
            uint64_t v = (slot(g, n, kk) + (t ? slot(k->cwv, n, kk) : 0)) & M;
            if (party) v = (0 - v) & M;
            uint64_t y = (uint64_t)(p * epl + kk);
            acc += v * table[(xhat - y) & 255];
        }
    }
    return (acc + k->rout) & M;
}

/* the public 8-bit degree table of secure_adj_norm.h:139-184 */
void ref_invsqrt_table(int scale, int nmax, uint64_t *table)
{
    for (int d = 0; d < 256; d++) table[d] = 0;
    double q = ldexp(1.0, scale);
    for (int d = 1; d <= nmax && d < 256; d++) table[d] = (uint64_t)llround(q / sqrt((double)d));
}
