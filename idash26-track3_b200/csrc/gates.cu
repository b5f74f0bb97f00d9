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

namespace ddg {

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
            if (L.lo) {
                const uint64_t alpha = uint64_t(r) & ((uint64_t(1) << L.Lo.d) - 1);
                DcfOut o{a.k0 + L.Lo.root, a.k1 + L.Lo.root, a.k0 + L.Lo.cw, a.k1 + L.Lo.cw,
                         a.k0 + L.Lo.leaf, a.k1 + L.Lo.leaf, nullptr, nullptr};
                dcf_keygen(A, alpha, L.Lo.d, A.prg(a.dk.rk, a.op, P_LO_S0, e), A.prg(a.dk.rk, a.op, P_LO_DELTA, e), o,
                           e, N);
            }
            T v[32];
            // split gates: monomials of the dealer bits the DReLU bit depends on,
            // eps = r_m ^ rho_c: eps, rho_L, rho_e, rho_e rho_L, eps rho_L, eps rho_e, eps rho_e rho_L
            const T rho_e = T(((bits >> 4) ^ (bits >> 5)) & 1u);
            const T mono[7] = {e_b, rho_L, rho_e, T(rho_e * rho_L), T(e_b * rho_L), T(e_b * rho_e),
                               T(e_b * rho_e * rho_L)};
            switch (a.kind) {
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
    DcfView hi, lo;
    bool has_hi, has_lo, split;
    uint32_t *bits_hi, *bits_lo;  // split gates: bits_hi[0, nw) compare, [nw, 2nw) equality
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
        uint32_t bh = 0, bl = 0, be = 0;
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
            if (a.has_lo) bl = dcf_eval(A, uint64_t(x & lmask), a.lo_d, a.lo, e, N);
        }
        const uint32_t wh = __ballot_sync(0xFFFFFFFFu, bh);
        const uint32_t wl = __ballot_sync(0xFFFFFFFFu, bl);
        const uint32_t we = __ballot_sync(0xFFFFFFFFu, be);
        if ((threadIdx.x & 31) == 0) {
            const uint64_t wi = e >> 5;
            if (a.has_hi) a.bits_hi[wi] = wh ^ __ldcs(a.hi.mu + wi);
            if (a.split) a.bits_hi[((N + 31) >> 5) + wi] = we ^ __ldcs(a.hi.mu_eq + wi);
            if (a.has_lo) a.bits_lo[wi] = wl ^ __ldcs(a.lo.mu + wi);
        }
    }
}

// ---------------------------------------------------------------- round 2

template <typename T>
struct Round2Args {
    int kind, n, s, party;
    uint64_t N, nw;
    const T *xhat;
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
        const T x = a.xhat[e];
        const uint64_t wi = e >> 5;
        const uint32_t bi = uint32_t(e & 31);
        T ch = 0, cl = 0, eh = 0;
        if (KIND != GATE_LRS) ch = T(((a.hi_own[wi] ^ a.hi_peer[wi]) >> bi) & 1u);
        if (KIND != GATE_RELU) cl = T(((a.lo_own[wi] ^ a.lo_peer[wi]) >> bi) & 1u);
        if (KIND == GATE_RELU_SPLIT || KIND == GATE_RELU_ARS_SPLIT || KIND == GATE_LRS_SPLIT)
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
    DDG_TRY(aes_device_init());
    if (L.n == 0) return DDG_OK;
    Round1Args<T> a;
    a.n = L.bw, a.s = L.s, a.N = L.n, a.hi_d = L.H.d, a.hi_shift = L.hi_shift, a.lo_d = L.Lo.d;
    a.xhat = static_cast<const T *>(xhat);
    const uint8_t *k = static_cast<const uint8_t *>(key);
    a.has_hi = L.hi, a.has_lo = L.lo, a.split = L.hi && L.H.eq;
    a.hi = L.hi ? dcf_view(k, L.H) : DcfView{};
    a.lo = L.lo ? dcf_view(k, L.Lo) : DcfView{};
    a.bits_hi = bits_hi, a.bits_lo = bits_lo;
    DcfTiming *tm = dcf_timing_sink();
    DcfTiming::Rec *rec = nullptr;
    if (tm && tm->enabled && tm->nrec < int(sizeof(tm->recs) / sizeof(tm->recs[0]))) {
        rec = &tm->recs[tm->nrec];
        DDG_CUDA(cudaEventCreate(&rec->a));
        DDG_CUDA(cudaEventCreate(&rec->b));
        DDG_CUDA(cudaEventRecord(rec->a, st));
    }
    DDG_TRY((aes_tables() == 4 ? round1_launch<T, AesLane4>(a, st) : round1_launch<T, AesLane2>(a, st)));
    note_launch();
    DDG_CUDA(cudaGetLastError());
    if (rec) {
        DDG_CUDA(cudaEventRecord(rec->b, st));
        // algorithmic bytes: every key byte of the DCFs once, the input, the output bits
        const double n = double(L.n);
        double bytes = n * (L.bw / 8.0), aes = 0;
        if (L.hi) bytes += n * (16.0 * (L.H.L + 2) + (L.H.eq ? 0.5 : 0.25)), aes += n * (L.H.L + 1);
        if (L.lo) bytes += n * (16.0 * (L.Lo.L + 2) + 0.125 + 0.125), aes += n * (L.Lo.L + 1);
        rec->bytes = bytes, rec->aes = aes, rec->evals = n * ((L.hi ? 1 : 0) + (L.lo ? 1 : 0));
        tm->nrec++;
    }
    return DDG_OK;
}

template <typename T>
int gate_round2_t(const GateLayout &L, int party, const void *xhat, const uint32_t *hi_own, const uint32_t *hi_peer,
                  const uint32_t *lo_own, const uint32_t *lo_peer, const void *key, void *share, cudaStream_t st)
{
    if (L.n == 0) return DDG_OK;
    Round2Args<T> a;
    a.kind = L.kind, a.n = L.bw, a.s = L.s, a.party = party, a.N = L.n, a.nw = (L.n + 31) / 32;
    a.xhat = static_cast<const T *>(xhat);
    a.hi_own = hi_own, a.hi_peer = hi_peer, a.lo_own = lo_own, a.lo_peer = lo_peer;
    a.words = reinterpret_cast<const T *>(static_cast<const uint8_t *>(key) + L.words);
    a.share = static_cast<T *>(share);
    int sms = device_sms();
    uint64_t blocks = (L.n + 255) / 256;
    uint64_t cap = uint64_t(sms > 0 ? sms : 148) * 8;
    int grid = int(blocks < cap ? blocks : cap);
    switch (L.kind) {
    case GATE_RELU: gate_round2_kernel<T, GATE_RELU><<<grid, 256, 0, st>>>(a); break;
    case GATE_RELU_ARS: gate_round2_kernel<T, GATE_RELU_ARS><<<grid, 256, 0, st>>>(a); break;
    case GATE_ARS: gate_round2_kernel<T, GATE_ARS><<<grid, 256, 0, st>>>(a); break;
    case GATE_RELU_SPLIT: gate_round2_kernel<T, GATE_RELU_SPLIT><<<grid, 256, 0, st>>>(a); break;
    case GATE_RELU_ARS_SPLIT: gate_round2_kernel<T, GATE_RELU_ARS_SPLIT><<<grid, 256, 0, st>>>(a); break;
    case GATE_LRS_SPLIT: gate_round2_kernel<T, GATE_LRS_SPLIT><<<grid, 256, 0, st>>>(a); break;
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
                const uint32_t *lo_own, const uint32_t *lo_peer, const void *key, void *share, cudaStream_t st)
{
    return L.bw == 32 ? gate_round2_t<uint32_t>(L, party, xhat, hi_own, hi_peer, lo_own, lo_peer, key, share, st)
                      : gate_round2_t<uint64_t>(L, party, xhat, hi_own, hi_peer, lo_own, lo_peer, key, share, st);
}

}  // namespace ddg
