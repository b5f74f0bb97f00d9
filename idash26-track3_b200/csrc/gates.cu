// Comparison gates (ReLU, ReLU o ARS, ARS, LRS of a non-negative value):
// dealer key generation, round 1 (DCF evaluation, one thread per element,
// bits packed by warp ballot) and round 2 (linear combination of the dealer
// words with the opened bits).
//
// Reference call sites replaced: DDGOrca::relu -> gpuRelu (gpu_mpc/ddg_orca.h:83-110,
// ddg_orca_batched.h:143-159) and DDGOrca::truncateForward -> gpuTruncate TrFloor
// (ddg_orca.h:112-123, ddg_orca_batched.h:161-200).
#include "dcf_dev.cuh"
#include "gates.cuh"
#include "ot.cuh"

namespace ddg {

// ------------------------------------------------- three-part split algebra
//
// DReLU bit d = q ^ eps ^ t with q = 1 ^ m_hat ^ c1_hat public, eps = r_m ^
// rho_c1 and t = e1*(c2 + e2*cL) in {0,1}.  Every true bit is b = b_hat +
// (1 - 2 b_hat) rho_b, so t is multilinear in (rho_e1, rho_c2, rho_e2, rho_L)
// over nine monomials, and
//   d = q + (1-2q) [tau_1 + (1 - 2 tau_1) eps + sum tau_m m - 2 sum tau_m eps m].
// The dealer shares the 19 monomials [eps, m (9), eps*m (9)]; m runs over
//   rho_c2, rho_L, rho_e2, rho_e2 rho_L, rho_e1, rho_e1 rho_c2, rho_e1 rho_L,
//   rho_e1 rho_e2, rho_e1 rho_e2 rho_L.

template <typename T>
__device__ __forceinline__ void split3_monomials(T ep, T pe1, T pc2, T pL, T pe2, T (&m)[SPLIT3_NMONO])
{
    const T t[9] = {pc2, pL, pe2, T(pe2 * pL), pe1, T(pe1 * pc2), T(pe1 * pL), T(pe1 * pe2), T(pe1 * pe2 * pL)};
    m[0] = ep;
#pragma unroll
    for (int k = 0; k < 9; k++) m[1 + k] = t[k], m[10 + k] = T(ep * t[k]);
}

// public coefficients of the 19 monomials; returns the constant term a0
template <typename T>
__device__ __forceinline__ T split3_coeffs(T q, T e1h, T c2h, T e2h, T cLh, T (&a)[SPLIT3_NMONO])
{
    const T su = T(1) - T(2) * q, se1 = T(1) - T(2) * e1h, sc2 = T(1) - T(2) * c2h, se2 = T(1) - T(2) * e2h,
            sL = T(1) - T(2) * cLh;
    // g = c2 + e2*cL = g0 + gc rho_c2 + gL rho_L + ge rho_e2 + geL rho_e2 rho_L
    const T g0 = c2h + e2h * cLh, gc = sc2, gL = e2h * sL, ge = cLh * se2, geL = se2 * sL;
    const T t1 = e1h * g0;
    const T tau[9] = {e1h * gc, e1h * gL, e1h * ge, e1h * geL, se1 * g0, se1 * gc, se1 * gL, se1 * ge, se1 * geL};
    a[0] = su * (T(1) - T(2) * t1);
#pragma unroll
    for (int k = 0; k < 9; k++) a[1 + k] = su * tau[k], a[10 + k] = T(0) - T(2) * su * tau[k];
    return q + su * t1;
}

// ---------------------------------------------------------------- keygen

template <typename T>
struct GateKeygenArgs {
    int kind, n, s;
    uint64_t N;
    uint32_t op;
    AesKey dk;
    const T *rin;
    T *rout;
    uint8_t *k0, *k1;
    GateLayout lay;
    OtPlan ot;          // OT / TT kinds: the digit plan (OT: and the two parties' keys K_0, K_1)
    AesKey prk0, prk1;
};

template <typename T, class E>
__global__ void __launch_bounds__(E::THREADS, E::CTAS) gate_keygen_kernel(const __grid_constant__ GateKeygenArgs<T> a)
{
    extern __shared__ uint32_t smem_tab[];
    E::stage(smem_tab);
    __syncthreads();
    E A(smem_tab);
    const GateLayout &L = a.lay;
    const int n = a.n, s = a.s;
    const uint64_t N = a.N;
    const uint64_t Npad = (N + 31) & ~uint64_t(31);
    for (uint64_t e = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < Npad; e += uint64_t(gridDim.x) * blockDim.x) {
        const bool valid = e < N;
        uint32_t bits = 0;
        if (valid) {
            const T r = a.rin[e];
            const T r_y = ring_of<T>(A.prg(a.dk.rk, a.op, P_ROUT, e));
            bits = A.prg(a.dk.rk, a.op, P_BITS, e).w[0];
            const T rho_c = T((bits ^ (bits >> 1)) & 1u);
            const T rho_L = T(((bits >> 2) ^ (bits >> 3)) & 1u);
            const T r_m = r >> (n - 1);
            const T r_H = r >> s;
            const T e_b = r_m ^ rho_c;
            if (L.hi) {
                // comparison threshold: bits [hi_shift, hi_shift + d) of the input mask
                const uint64_t alpha = uint64_t(r >> L.hi_shift) & ((uint64_t(1) << L.H.d) - 1);
                DcfOut o{a.k0 + L.H.root, a.k1 + L.H.root, a.k0 + L.H.cw, a.k1 + L.H.cw,
                         a.k0 + L.H.leaf, a.k1 + L.H.leaf, nullptr, nullptr};
                if (L.H.eq)
                    dcfeq_keygen(A, alpha, L.H.d, A.prg(a.dk.rk, a.op, P_HI_S0, e), A.prg(a.dk.rk, a.op, P_HI_DELTA, e),
                                 o, e, N);
                else
                    dcf_keygen(A, alpha, L.H.d, A.prg(a.dk.rk, a.op, P_HI_S0, e), A.prg(a.dk.rk, a.op, P_HI_DELTA, e),
                               o, e, N);
            }
            if (L.mid) {
                const uint64_t alpha = uint64_t(r >> s) & ((uint64_t(1) << SPLIT3_MID) - 1);
                DcfOut o{a.k0 + L.Mi.root, a.k1 + L.Mi.root, a.k0 + L.Mi.cw, a.k1 + L.Mi.cw,
                         a.k0 + L.Mi.leaf, a.k1 + L.Mi.leaf, nullptr, nullptr};
                dcfeq_keygen(A, alpha, SPLIT3_MID, A.prg(a.dk.rk, a.op, P_MID_S0, e),
                             A.prg(a.dk.rk, a.op, P_MID_DELTA, e), o, e, N);
            }
            if (L.ot) {
                const uint32_t rc = (bits ^ (bits >> 1)) & 1u, rl = ((bits >> 2) ^ (bits >> 3)) & 1u,
                               re = ((bits >> 4) ^ (bits >> 5)) & 1u;
                ot_keygen_elem(A, a.ot, a.prk0.rk, a.prk1.rk, e, N, uint64_t(r), rc, re, rl, a.k0 + L.ot_recv,
                               a.k1 + L.ot_recv, reinterpret_cast<uint32_t *>(a.k0 + L.ot_c0));
                reinterpret_cast<uint32_t *>(a.k1 + L.ot_c0)[e] = 0u;
                // party 0 receives D - G0 digits: its unused last slot is zeroed
                for (int t = a.ot.D - a.ot.G0; t < L.ot_gmax; t++) a.k0[L.ot_recv + uint64_t(t) * N + e] = 0;
                if (e == 0) {
                    for (int i = 0; i < 44; i++) {
                        reinterpret_cast<uint32_t *>(a.k0 + L.ot_ks)[i] = a.prk0.rk[i];
                        reinterpret_cast<uint32_t *>(a.k1 + L.ot_ks)[i] = a.prk1.rk[i];
                    }
                }
            }
            if (L.tt) {
                tt_keygen_elem(A, a.ot, a.dk.rk, a.op, e, N, uint64_t(r), bits,
                               reinterpret_cast<uint32_t *>(a.k0 + L.tt_tables),
                               reinterpret_cast<uint32_t *>(a.k1 + L.tt_tables),
                               reinterpret_cast<uint32_t *>(a.k0 + L.tt_tri),
                               reinterpret_cast<uint32_t *>(a.k1 + L.tt_tri));
            }
            if (L.lo) {
                const uint64_t alpha = uint64_t(r) & ((uint64_t(1) << L.Lo.d) - 1);
                DcfOut o{a.k0 + L.Lo.root, a.k1 + L.Lo.root, a.k0 + L.Lo.cw, a.k1 + L.Lo.cw,
                         a.k0 + L.Lo.leaf, a.k1 + L.Lo.leaf, nullptr, nullptr};
                dcf_keygen(A, alpha, L.Lo.d, A.prg(a.dk.rk, a.op, P_LO_S0, e), A.prg(a.dk.rk, a.op, P_LO_DELTA, e), o,
                           e, N);
            }
            T v[80];
            // split gates: monomials of the dealer bits the DReLU bit depends on,
            // eps = r_m ^ rho_c: eps, rho_L, rho_e, rho_e rho_L, eps rho_L, eps rho_e, eps rho_e rho_L
            const T rho_e = T(((bits >> 4) ^ (bits >> 5)) & 1u);
            const T mono[7] = {e_b, rho_L, rho_e, T(rho_e * rho_L), T(e_b * rho_L), T(e_b * rho_e),
                               T(e_b * rho_e * rho_L)};
            switch (gate_word_kind(a.kind)) {
            case GATE_RELU:
                v[0] = e_b, v[1] = r, v[2] = e_b * r, v[3] = r_y;
                break;
            case GATE_RELU_ARS:
                v[0] = e_b, v[1] = r_H, v[2] = e_b * r_H, v[3] = rho_L, v[4] = e_b * rho_L, v[5] = r_m, v[6] = e_b * r_m,
                v[7] = r_y;
                break;
            case GATE_ARS:
                v[0] = r_H, v[1] = rho_L, v[2] = rho_c, v[3] = r_m, v[4] = r_m * rho_c, v[5] = r_y;
                break;
            case GATE_RELU_SPLIT:
                for (int k = 0; k < 7; k++) v[k] = mono[k], v[8 + k] = mono[k] * r;
                v[7] = r, v[15] = r_y;
                break;
            case GATE_LRS_SPLIT:
                // carry = c1 + e1*c2 (exclusive terms); masks rho_c (c1), rho_e (e1), rho_L (c2)
                v[0] = r_H, v[1] = rho_c, v[2] = rho_e, v[3] = rho_L, v[4] = rho_e * rho_L, v[5] = r_m, v[6] = r_y;
                break;
            case GATE_RELU_SPLIT3:
            case GATE_RELU_ARS_SPLIT3: {
                const T rho_m = T(((bits >> 6) ^ (bits >> 7)) & 1u), rho_me = T(((bits >> 8) ^ (bits >> 9)) & 1u);
                T m3[SPLIT3_NMONO];
                split3_monomials<T>(e_b, rho_e, rho_m, rho_L, rho_me, m3);
                if (a.kind == GATE_RELU_SPLIT3) {
                    for (int k = 0; k < SPLIT3_NMONO; k++) v[k] = m3[k], v[20 + k] = m3[k] * r;
                    v[19] = r, v[39] = r_y;
                } else {
                    const T nj[3] = {r_H, rho_L, r_m};
                    for (int k = 0; k < SPLIT3_NMONO; k++) v[k] = m3[k];
                    for (int j = 0; j < 3; j++) v[19 + j] = nj[j];
                    for (int k = 0; k < SPLIT3_NMONO; k++)
                        for (int j = 0; j < 3; j++) v[22 + 3 * k + j] = m3[k] * nj[j];
                    v[79] = r_y;
                }
                break;
            }
            case GATE_RELU_ARS_SPLIT: {
                const T nj[3] = {r_H, rho_L, r_m};
                for (int k = 0; k < 7; k++) v[k] = mono[k];
                for (int j = 0; j < 3; j++) v[7 + j] = nj[j];
                for (int k = 0; k < 7; k++)
                    for (int j = 0; j < 3; j++) v[10 + 3 * k + j] = mono[k] * nj[j];
                v[31] = r_y;
                break;
            }
            default:
                v[0] = r_H, v[1] = rho_L, v[2] = r_m, v[3] = r_y;
                break;
            }
            T *w0 = reinterpret_cast<T *>(a.k0 + L.words);
            T *w1 = reinterpret_cast<T *>(a.k1 + L.words);
            for (int w = 0; w < L.nwords; w++) {
                T sh = ring_of<T>(A.prg(a.dk.rk, a.op, P_SHARE + w, e));
                w0[uint64_t(w) * N + e] = sh;
                w1[uint64_t(w) * N + e] = T(v[w] - sh);
            }
            a.rout[e] = r_y;
        }
        // pack the parties' output-mask bits, 32 elements per word
        const uint32_t m0h = __ballot_sync(0xFFFFFFFFu, valid && (bits & 1u));
        const uint32_t m1h = __ballot_sync(0xFFFFFFFFu, valid && (bits & 2u));
        const uint32_t m0l = __ballot_sync(0xFFFFFFFFu, valid && (bits & 4u));
        const uint32_t m1l = __ballot_sync(0xFFFFFFFFu, valid && (bits & 8u));
        const uint32_t m0e = __ballot_sync(0xFFFFFFFFu, valid && (bits & 16u));
        const uint32_t m1e = __ballot_sync(0xFFFFFFFFu, valid && (bits & 32u));
        const uint32_t m0m = __ballot_sync(0xFFFFFFFFu, valid && (bits & 64u));
        const uint32_t m1m = __ballot_sync(0xFFFFFFFFu, valid && (bits & 128u));
        const uint32_t m0me = __ballot_sync(0xFFFFFFFFu, valid && (bits & 256u));
        const uint32_t m1me = __ballot_sync(0xFFFFFFFFu, valid && (bits & 512u));
        if ((threadIdx.x & 31) == 0) {
            const uint64_t wi = e >> 5;
            if (L.hi) {
                reinterpret_cast<uint32_t *>(a.k0 + L.H.mu)[wi] = m0h;
                reinterpret_cast<uint32_t *>(a.k1 + L.H.mu)[wi] = m1h;
                if (L.H.eq) {
                    reinterpret_cast<uint32_t *>(a.k0 + L.H.mu_eq)[wi] = m0e;
                    reinterpret_cast<uint32_t *>(a.k1 + L.H.mu_eq)[wi] = m1e;
                }
            }
            if (L.mid) {
                reinterpret_cast<uint32_t *>(a.k0 + L.Mi.mu)[wi] = m0m;
                reinterpret_cast<uint32_t *>(a.k1 + L.Mi.mu)[wi] = m1m;
                reinterpret_cast<uint32_t *>(a.k0 + L.Mi.mu_eq)[wi] = m0me;
                reinterpret_cast<uint32_t *>(a.k1 + L.Mi.mu_eq)[wi] = m1me;
            }
            if (L.lo) {
                reinterpret_cast<uint32_t *>(a.k0 + L.Lo.mu)[wi] = m0l;
                reinterpret_cast<uint32_t *>(a.k1 + L.Lo.mu)[wi] = m1l;
            }
        }
    }
}

// ---------------------------------------------------------------- round 1

template <typename T>
struct Round1Args {
    int n, s, hi_d, hi_shift, lo_d;
    uint64_t N;
    const T *xhat;
    DcfView hi, mid, lo;
    bool has_hi, has_mid, has_lo, split;
    // split gates: bits_hi[0, nw) compare, [nw, 2nw) equality; with a middle
    // DCF also [2nw, 3nw) its compare and [3nw, 4nw) its equality
    uint32_t *bits_hi, *bits_lo;
};

template <typename T, class E>
__global__ void __launch_bounds__(E::THREADS, E::CTAS) gate_round1_kernel(const __grid_constant__ Round1Args<T> a)
{
    extern __shared__ uint32_t smem_tab[];
    E::stage(smem_tab);
    __syncthreads();
    E A(smem_tab);
    const uint64_t N = a.N;
    const uint64_t Npad = (N + 31) & ~uint64_t(31);
    const T hmask = (T(1) << a.hi_d) - 1;
    const T lmask = (T(1) << a.lo_d) - 1;
    for (uint64_t e = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < Npad; e += uint64_t(gridDim.x) * blockDim.x) {
        const bool valid = e < N;
        uint32_t bh = 0, bl = 0, be = 0, bm = 0, bme = 0;
        if (valid) {
            const T x = __ldcs(a.xhat + e);
            if (a.has_hi) {
                const uint64_t xh = uint64_t((x >> a.hi_shift) & hmask);
                if (a.split) {
                    const uint32_t b = dcfeq_eval(A, xh, a.hi_d, a.hi, e, N);
                    bh = b & 1u, be = b >> 1;
                } else {
                    bh = dcf_eval(A, xh, a.hi_d, a.hi, e, N);
                }
            }
            if (a.has_mid) {
                const uint32_t b =
                    dcfeq_eval(A, uint64_t((x >> a.s) & T((1u << SPLIT3_MID) - 1)), SPLIT3_MID, a.mid, e, N);
                bm = b & 1u, bme = b >> 1;
            }
            if (a.has_lo) bl = dcf_eval(A, uint64_t(x & lmask), a.lo_d, a.lo, e, N);
        }
        const uint32_t wh = __ballot_sync(0xFFFFFFFFu, bh);
        const uint32_t wl = __ballot_sync(0xFFFFFFFFu, bl);
        const uint32_t we = __ballot_sync(0xFFFFFFFFu, be);
        const uint32_t wm = __ballot_sync(0xFFFFFFFFu, bm);
        const uint32_t wme = __ballot_sync(0xFFFFFFFFu, bme);
        if ((threadIdx.x & 31) == 0) {
            const uint64_t wi = e >> 5, nw = (N + 31) >> 5;
            if (a.has_hi) a.bits_hi[wi] = wh ^ __ldcs(a.hi.mu + wi);
            if (a.split) a.bits_hi[nw + wi] = we ^ __ldcs(a.hi.mu_eq + wi);
            if (a.has_mid) {
                a.bits_hi[2 * nw + wi] = wm ^ __ldcs(a.mid.mu + wi);
                a.bits_hi[3 * nw + wi] = wme ^ __ldcs(a.mid.mu_eq + wi);
            }
            if (a.has_lo) a.bits_lo[wi] = wl ^ __ldcs(a.lo.mu + wi);
        }
    }
}

// ---------------------------------------------------------------- round 2

template <typename T>
struct Round2Args {
    int kind, n, s, party;
    uint64_t N, nw;
    const T *xhat, *xhat2;  // xhat2: second addend of the opened input (may be null)
    const uint32_t *hi_own, *hi_peer, *lo_own, *lo_peer;
    const T *words;
    T *share;
};

template <typename T, int KIND>
__global__ void gate_round2_kernel(const __grid_constant__ Round2Args<T> a)
{
    const uint64_t N = a.N;
    const int n = a.n, s = a.s;
    const T p0 = a.party == 0 ? T(1) : T(0);
    const T two_ns = T(1) << (n - s);
    for (uint64_t e = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < N; e += uint64_t(gridDim.x) * blockDim.x) {
        T x = a.xhat[e];
        if (a.xhat2) x += a.xhat2[e];
        const uint64_t wi = e >> 5;
        const uint32_t bi = uint32_t(e & 31);
        T ch = 0, cl = 0, eh = 0;
        if (KIND != GATE_LRS) ch = T(((a.hi_own[wi] ^ a.hi_peer[wi]) >> bi) & 1u);
        if (KIND != GATE_RELU) cl = T(((a.lo_own[wi] ^ a.lo_peer[wi]) >> bi) & 1u);
        if (KIND == GATE_RELU_SPLIT || KIND == GATE_RELU_ARS_SPLIT || KIND == GATE_LRS_SPLIT ||
            KIND == GATE_RELU_SPLIT3 || KIND == GATE_RELU_ARS_SPLIT3)
            eh = T(((a.hi_own[a.nw + wi] ^ a.hi_peer[a.nw + wi]) >> bi) & 1u);
        const T mh = x >> (n - 1);
        const T xH = x >> s;
        const T *w = a.words + e;
        auto W = [&](int k) { return __ldcs(w + uint64_t(k) * N); };
        const T q = T(1) ^ mh ^ ch;
        const T a1 = T(1) - T(2) * q;
        const T b1 = T(1) - T(2) * cl;
        T y;
        if (KIND == GATE_RELU) {
            y = p0 * q * x + a1 * x * W(0) - q * W(1) - a1 * W(2) + W(3);
        } else if (KIND == GATE_RELU_ARS) {
            y = p0 * (q * xH - q * cl) + W(0) * (a1 * xH - a1 * cl) - q * W(1) - a1 * W(2) - q * b1 * W(3) -
                a1 * b1 * W(4) + two_ns * (T(1) - mh) * (q * W(5) + a1 * W(6)) + W(7);
        } else if (KIND == GATE_RELU_SPLIT || KIND == GATE_RELU_ARS_SPLIT) {
            // every dealer word of the element in flight at once (the kernel is HBM-bound)
            constexpr int NWD = KIND == GATE_RELU_SPLIT ? 16 : 32;
            T wv[NWD];
#pragma unroll
            for (int k = 0; k < NWD; k++) wv[k] = W(k);
            auto W = [&](int k) { return wv[k]; };
            // DReLU = a0 + sum_k ak[k] * mono[k]  (mono: the dealer-bit monomials of the key words)
            const T se = T(1) - T(2) * eh, sc = b1;
            const T G0 = eh * cl, GL = eh * sc, Ge = cl * se, GeL = se * sc;
            const T a0 = q + a1 * G0;
            const T ak[7] = {a1 * (T(1) - T(2) * G0), a1 * GL, a1 * Ge, a1 * GeL, T(0) - T(2) * a1 * GL,
                             T(0) - T(2) * a1 * Ge, T(0) - T(2) * a1 * GeL};
            T sm = 0;
#pragma unroll
            for (int k = 0; k < 7; k++) sm += ak[k] * W(k);
            if (KIND == GATE_RELU_SPLIT) {
                T sr = 0;
#pragma unroll
                for (int k = 0; k < 7; k++) sr += ak[k] * W(8 + k);
                y = p0 * a0 * x + x * sm - a0 * W(7) - sr + W(15);
            } else {
                const T Y0 = xH - cl;
                const T yj[3] = {T(0) - T(1), T(0) - sc, two_ns * (T(1) - mh)};
                T sn = 0, smn = 0;
#pragma unroll
                for (int j = 0; j < 3; j++) sn += yj[j] * W(7 + j);
#pragma unroll
                for (int k = 0; k < 7; k++) {
                    T t = 0;
#pragma unroll
                    for (int j = 0; j < 3; j++) t += yj[j] * W(10 + 3 * k + j);
                    smn += ak[k] * t;
                }
                y = p0 * a0 * Y0 + Y0 * sm + a0 * sn + smn + W(31);
            }
        } else if (KIND == GATE_RELU_SPLIT3 || KIND == GATE_RELU_ARS_SPLIT3) {
            const T cm = T(((a.hi_own[2 * a.nw + wi] ^ a.hi_peer[2 * a.nw + wi]) >> bi) & 1u);
            const T em = T(((a.hi_own[3 * a.nw + wi] ^ a.hi_peer[3 * a.nw + wi]) >> bi) & 1u);
            T ak[SPLIT3_NMONO];
            const T a0 = split3_coeffs<T>(q, eh, cm, em, cl, ak);
            T sm = 0;
#pragma unroll
            for (int k = 0; k < SPLIT3_NMONO; k++) sm += ak[k] * W(k);
            if (KIND == GATE_RELU_SPLIT3) {
                T sr = 0;
#pragma unroll
                for (int k = 0; k < SPLIT3_NMONO; k++) sr += ak[k] * W(20 + k);
                y = p0 * a0 * x + x * sm - a0 * W(19) - sr + W(39);
            } else {
                const T Y0 = xH - cl;
                const T yj[3] = {T(0) - T(1), T(0) - b1, two_ns * (T(1) - mh)};
                T sn = 0, smn = 0;
#pragma unroll
                for (int j = 0; j < 3; j++) sn += yj[j] * W(19 + j);
#pragma unroll
                for (int k = 0; k < SPLIT3_NMONO; k++) {
                    T t = 0;
#pragma unroll
                    for (int j = 0; j < 3; j++) t += yj[j] * W(22 + 3 * k + j);
                    smn += ak[k] * t;
                }
                y = p0 * a0 * Y0 + Y0 * sm + a0 * sn + smn + W(79);
            }
        } else if (KIND == GATE_LRS_SPLIT) {
            // carry = c1 + e1*c2 with c1 = ch ^ rho_c, e1 = eh ^ rho_e, c2 = cl ^ rho_L
            const T sc1 = T(1) - T(2) * ch, se = T(1) - T(2) * eh;
            y = p0 * (xH - ch - eh * cl) - W(0) - sc1 * W(1) - cl * se * W(2) - eh * b1 * W(3) - se * b1 * W(4) +
                two_ns * (T(1) - mh) * W(5) + W(6);
        } else if (KIND == GATE_ARS) {
            const T pub = xH - cl + two_ns * (mh * ch - mh);
            y = p0 * pub - W(0) - b1 * W(1) +
                two_ns * (mh * (T(1) - T(2) * ch) * W(2) + ((T(1) - T(2) * mh) * ch + mh) * W(3) +
                          (T(1) - T(2) * mh) * (T(1) - T(2) * ch) * W(4)) +
                W(5);
        } else {
            y = p0 * (xH - cl) - W(0) - b1 * W(1) + two_ns * (T(1) - mh) * W(2) + W(3);
        }
        a.share[e] = y;
    }
}

// ---------------------------------------------------------------- launchers

int device_sms()
{
    int dev = 0;
    DDG_CUDA(cudaGetDevice(&dev));
    int sms = 0;
    DDG_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    return sms;
}

template <class E, typename K>
static int set_smem(K kernel)
{
    DDG_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, E::SMEM));
    return DDG_OK;
}

template <typename T, class E>
static int keygen_launch(const GateKeygenArgs<T> &a, cudaStream_t st)
{
    DDG_TRY(set_smem<E>(gate_keygen_kernel<T, E>));
    gate_keygen_kernel<T, E><<<aes_blocks<E>(a.N), E::THREADS, E::SMEM, st>>>(a);
    return DDG_OK;
}

template <typename T, class E>
static int round1_launch(const Round1Args<T> &a, cudaStream_t st)
{
    DDG_TRY(set_smem<E>(gate_round1_kernel<T, E>));
    gate_round1_kernel<T, E><<<aes_blocks<E>(a.N), E::THREADS, E::SMEM, st>>>(a);
    return DDG_OK;
}

template <typename T>
int gate_keygen_t(const GateLayout &L, uint64_t seed, uint32_t op, const void *rin, void *rout, void *k0, void *k1,
                  cudaStream_t st)
{
    DDG_TRY(aes_device_init());
    GateKeygenArgs<T> a;
    a.kind = L.kind, a.n = L.bw, a.s = L.s, a.N = L.n, a.op = op;
    a.dk = dealer_key(seed);
    a.rin = static_cast<const T *>(rin);
    a.rout = static_cast<T *>(rout);
    a.k0 = static_cast<uint8_t *>(k0);
    a.k1 = static_cast<uint8_t *>(k1);
    a.lay = L;
    if (L.ot) {
        a.ot = ot_plan_cached(L.bw, L.s);
        DDG_CHECK(a.ot.ok, DDG_ERR_ARG, "no OT-gate plan for bw %d, scale %d", L.bw, L.s);
        a.prk0 = ot_party_key(a.dk, op, 0);
        a.prk1 = ot_party_key(a.dk, op, 1);
    }
    if (L.tt) {
        a.ot = tt_plan_of(L.kind, L.bw, L.s);
        DDG_CHECK(a.ot.ok, DDG_ERR_ARG, "no truth-table plan for bw %d, scale %d", L.bw, L.s);
    }
    if (L.n == 0) return DDG_OK;
    DDG_TRY((aes_tables() == 4 ? keygen_launch<T, AesLane4>(a, st) : keygen_launch<T, AesLane2>(a, st)));
    note_launch();
    DDG_CUDA(cudaGetLastError());
    return DDG_OK;
}

template <typename T>
int gate_round1_t(const GateLayout &L, const void *xhat, const void *key, uint32_t *bits_hi, uint32_t *bits_lo,
                  cudaStream_t st)
{
    DDG_CHECK(!L.ot && !L.tt, DDG_ERR_ARG, "OT and TT gates have no one-shot round 1 (AND-tree levels)");
    DDG_TRY(aes_device_init());
    if (L.n == 0) return DDG_OK;
    Round1Args<T> a;
    a.n = L.bw, a.s = L.s, a.N = L.n, a.hi_d = L.H.d, a.hi_shift = L.hi_shift, a.lo_d = L.Lo.d;
    a.xhat = static_cast<const T *>(xhat);
    const uint8_t *k = static_cast<const uint8_t *>(key);
    a.has_hi = L.hi, a.has_mid = L.mid, a.has_lo = L.lo, a.split = L.hi && L.H.eq;
    a.hi = L.hi ? dcf_view(k, L.H) : DcfView{};
    a.mid = L.mid ? dcf_view(k, L.Mi) : DcfView{};
    a.lo = L.lo ? dcf_view(k, L.Lo) : DcfView{};
    a.bits_hi = bits_hi, a.bits_lo = bits_lo;
    TimedLaunch tl;
    DDG_TRY(tl.begin(st));
    DDG_TRY((aes_tables() == 4 ? round1_launch<T, AesLane4>(a, st) : round1_launch<T, AesLane2>(a, st)));
    note_launch();
    DDG_CUDA(cudaGetLastError());
    // algorithmic bytes: every key byte of the DCFs once, the input, the output bits
    const double n = double(L.n);
    double bytes = n * (L.bw / 8.0), aes = 0;
    if (L.hi) bytes += n * (16.0 * (L.H.L + 2) + (L.H.eq ? 0.5 : 0.25)), aes += n * (L.H.L + 1);
    if (L.mid) bytes += n * (16.0 * (L.Mi.L + 2) + 0.5), aes += n * (L.Mi.L + 1);
    if (L.lo) bytes += n * (16.0 * (L.Lo.L + 2) + 0.125 + 0.125), aes += n * (L.Lo.L + 1);
    DDG_TRY(tl.end(st, bytes, aes, n * ((L.hi ? 1 : 0) + (L.lo ? 1 : 0))));
    return DDG_OK;
}

template <typename T>
int gate_round2_t(const GateLayout &L, int party, const void *xhat, const uint32_t *hi_own, const uint32_t *hi_peer,
                  const uint32_t *lo_own, const uint32_t *lo_peer, const void *key, void *share, cudaStream_t st,
                  const void *xhat2)
{
    if (L.n == 0) return DDG_OK;
    Round2Args<T> a;
    a.kind = L.kind, a.n = L.bw, a.s = L.s, a.party = party, a.N = L.n, a.nw = (L.n + 31) / 32;
    a.xhat = static_cast<const T *>(xhat);
    a.xhat2 = static_cast<const T *>(xhat2);
    a.hi_own = hi_own, a.hi_peer = hi_peer, a.lo_own = lo_own, a.lo_peer = lo_peer;
    a.words = reinterpret_cast<const T *>(static_cast<const uint8_t *>(key) + L.words);
    a.share = static_cast<T *>(share);
    int sms = device_sms();
    uint64_t blocks = (L.n + 255) / 256;
    uint64_t cap = uint64_t(sms > 0 ? sms : 148) * 8;
    int grid = int(blocks < cap ? blocks : cap);
    switch (gate_word_kind(L.kind)) {
    case GATE_RELU: gate_round2_kernel<T, GATE_RELU><<<grid, 256, 0, st>>>(a); break;
    case GATE_RELU_ARS: gate_round2_kernel<T, GATE_RELU_ARS><<<grid, 256, 0, st>>>(a); break;
    case GATE_ARS: gate_round2_kernel<T, GATE_ARS><<<grid, 256, 0, st>>>(a); break;
    case GATE_RELU_SPLIT: gate_round2_kernel<T, GATE_RELU_SPLIT><<<grid, 256, 0, st>>>(a); break;
    case GATE_RELU_ARS_SPLIT: gate_round2_kernel<T, GATE_RELU_ARS_SPLIT><<<grid, 256, 0, st>>>(a); break;
    case GATE_LRS_SPLIT: gate_round2_kernel<T, GATE_LRS_SPLIT><<<grid, 256, 0, st>>>(a); break;
    case GATE_RELU_SPLIT3: gate_round2_kernel<T, GATE_RELU_SPLIT3><<<grid, 256, 0, st>>>(a); break;
    case GATE_RELU_ARS_SPLIT3: gate_round2_kernel<T, GATE_RELU_ARS_SPLIT3><<<grid, 256, 0, st>>>(a); break;
    default: gate_round2_kernel<T, GATE_LRS><<<grid, 256, 0, st>>>(a); break;
    }
    note_launch();
    DDG_CUDA(cudaGetLastError());
    return DDG_OK;
}

int gate_keygen(const GateLayout &L, uint64_t seed, uint32_t op, const void *rin, void *rout, void *k0, void *k1,
                cudaStream_t st)
{
    return L.bw == 32 ? gate_keygen_t<uint32_t>(L, seed, op, rin, rout, k0, k1, st)
                      : gate_keygen_t<uint64_t>(L, seed, op, rin, rout, k0, k1, st);
}

int gate_round1(const GateLayout &L, const void *xhat, const void *key, uint32_t *bits_hi, uint32_t *bits_lo,
                cudaStream_t st)
{
    return L.bw == 32 ? gate_round1_t<uint32_t>(L, xhat, key, bits_hi, bits_lo, st)
                      : gate_round1_t<uint64_t>(L, xhat, key, bits_hi, bits_lo, st);
}

int gate_round2(const GateLayout &L, int party, const void *xhat, const uint32_t *hi_own, const uint32_t *hi_peer,
                const uint32_t *lo_own, const uint32_t *lo_peer, const void *key, void *share, cudaStream_t st,
                const void *xhat2)
{
    return L.bw == 32
               ? gate_round2_t<uint32_t>(L, party, xhat, hi_own, hi_peer, lo_own, lo_peer, key, share, st, xhat2)
               : gate_round2_t<uint64_t>(L, party, xhat, hi_own, hi_peer, lo_own, lo_peer, key, share, st, xhat2);
}

}  // namespace ddg
