// DPF look-up table over an 8-bit domain, arithmetic payload in Z_2^n.
// Replaces gpuDpfLUT / gpuKeyGenLUT behind the secure adjacency normalisation
// (gpu_mpc/secure_adj_norm.h:270-279, 498-520): party b's share of
// table[(x_hat - alpha) mod 256] is  sum_y v_b(y) * table[(x_hat - y) mod 256]
// where v_0(y) + v_1(y) = [y == alpha] comes from a half-tree DPF whose
// 128-bit leaves hold 128/n slots (L = 8 - log2(128/n) tree levels).
// Evaluation: one warp per lookup; lane l expands the subtree under the
// depth-5 node with prefix l and the warp reduces the dot product.
#include "dcf_dev.cuh"
#include "gates.cuh"
#include "linear.cuh"

namespace ddg {

LutLayout lut_layout(int bw, uint64_t n, uint64_t base)
{
    LutLayout l;
    l.bw = bw;
    l.n = n;
    l.L = bw == 32 ? 6 : 7;
    l.root = align256(base);
    l.cw = align256(l.root + 16 * n);
    l.cwv = align256(l.cw + 16 * n * uint64_t(l.L));
    l.rout = align256(l.cwv + 16 * n);
    l.bytes = align256(l.rout + n * uint64_t(bw / 8)) - align256(base);
    return l;
}

template <typename T>
__device__ __forceinline__ T blk_slot(const Blk &b, int k)
{
    if constexpr (sizeof(T) == 4) {
        return k == 0 ? b.w[0] : k == 1 ? b.w[1] : k == 2 ? b.w[2] : b.w[3];
    } else {
        return k == 0 ? (uint64_t(b.w[0]) | (uint64_t(b.w[1]) << 32)) : (uint64_t(b.w[2]) | (uint64_t(b.w[3]) << 32));
    }
}

template <typename T>
__device__ __forceinline__ void blk_set_slot(Blk &b, int k, T v)
{
    if constexpr (sizeof(T) == 4) {
        if (k == 0) b.w[0] = v;
        else if (k == 1) b.w[1] = v;
        else if (k == 2) b.w[2] = v;
        else b.w[3] = v;
    } else {
        if (k == 0) b.w[0] = uint32_t(v), b.w[1] = uint32_t(v >> 32);
        else b.w[2] = uint32_t(v), b.w[3] = uint32_t(v >> 32);
    }
}

template <typename T>
struct LutKeygenArgs {
    LutLayout L;
    AesKey dk;
    uint32_t op;
    const T *alpha_mask;
    const T *rout;
    uint8_t *k0, *k1;
};

template <typename T, class E>
__global__ void __launch_bounds__(E::THREADS, E::CTAS) lut_keygen_kernel(const __grid_constant__ LutKeygenArgs<T> a)
{
    extern __shared__ uint32_t smem_tab[];
    E::stage(smem_tab);
    __syncthreads();
    E A(smem_tab);
    constexpr int EPL = 16 / sizeof(T);
    const uint64_t n = a.L.n;
    const int L = a.L.L;
    for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += uint64_t(gridDim.x) * blockDim.x) {
        const uint32_t alpha = uint32_t(a.alpha_mask[i]) & 255u;
        Blk s0 = A.prg(a.dk.rk, a.op, P_HI_S0, i);
        Blk delta = A.prg(a.dk.rk, a.op, P_HI_DELTA, i);
        delta.w[0] |= 1u;
        Blk cur0 = s0, cur1 = blk_xor(s0, delta);
        if (a.k0) st_blk(a.k0 + a.L.root + 16 * i, cur0);
        if (a.k1) st_blk(a.k1 + a.L.root + 16 * i, cur1);
        for (int j = 0; j < L; j++) {
            uint32_t bit = (alpha >> (7 - j)) & 1u;
            Blk h0 = A.hash_h(cur0), h1 = A.hash_h(cur1);
            Blk cw = blk_xor(blk_xor(h0, h1), blk_and_mask(delta, bit - 1u));
            if (a.k0) st_blk(a.k0 + a.L.cw + 16 * (uint64_t(j) * n + i), cw);
            if (a.k1) st_blk(a.k1 + a.L.cw + 16 * (uint64_t(j) * n + i), cw);
            Blk c0 = blk_xor(h0, blk_and_mask(cw, 0u - (cur0.w[0] & 1u)));
            Blk c1 = blk_xor(h1, blk_and_mask(cw, 0u - (cur1.w[0] & 1u)));
            cur0 = blk_xor(c0, blk_and_mask(cur0, 0u - bit));
            cur1 = blk_xor(c1, blk_and_mask(cur1, 0u - bit));
        }
        const bool t0 = cur0.w[0] & 1u;
        Blk g0 = A.hash_c(cur0), g1 = A.hash_c(cur1);
        Blk cwv;
        const int alo = int(alpha & (EPL - 1));
#pragma unroll
        for (int k = 0; k < EPL; k++) {
            T v = T(k == alo ? 1 : 0) - blk_slot<T>(g0, k) + blk_slot<T>(g1, k);
            blk_set_slot<T>(cwv, k, t0 ? v : T(0) - v);
        }
        if (a.k0) st_blk(a.k0 + a.L.cwv + 16 * i, cwv);
        if (a.k1) st_blk(a.k1 + a.L.cwv + 16 * i, cwv);
        T sh = ring_of<T>(A.prg(a.dk.rk, a.op, P_SHARE, i));
        if (a.k0) reinterpret_cast<T *>(a.k0 + a.L.rout)[i] = sh;
        if (a.k1) reinterpret_cast<T *>(a.k1 + a.L.rout)[i] = a.rout[i] - sh;
    }
}

template <typename T>
struct LutEvalArgs {
    LutLayout L;
    int party;
    const T *xhat;
    const T *table;
    const uint8_t *key;
    T *share;
};

template <typename T, class E>
__global__ void __launch_bounds__(E::THREADS, E::CTAS) lut_eval_kernel(const __grid_constant__ LutEvalArgs<T> a)
{
    extern __shared__ uint32_t smem_tab[];
    __shared__ T tab[256];
    E::stage(smem_tab);
    for (int i = threadIdx.x; i < 256; i += blockDim.x) tab[i] = a.table[i];
    __syncthreads();
    E A(smem_tab);
    constexpr int EPL = 16 / sizeof(T);
    const uint64_t n = a.L.n;
    const int L = a.L.L, Lr = L - 5;
    const int lane = threadIdx.x & 31;
    const uint64_t warps = (uint64_t(gridDim.x) * blockDim.x) >> 5;
    for (uint64_t i = (uint64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; i < n; i += warps) {
        const uint8_t *k = a.key;
        Blk s = ld_blk_stream(k + a.L.root + 16 * i);
        for (int j = 0; j < 5; j++) {
            uint32_t bit = (uint32_t(lane) >> (4 - j)) & 1u;
            Blk cw = ld_blk_stream(k + a.L.cw + 16 * (uint64_t(j) * n + i));
            Blk cl = blk_xor(A.hash_h(s), blk_and_mask(cw, 0u - (s.w[0] & 1u)));
            s = blk_xor(cl, blk_and_mask(s, 0u - bit));
        }
        const Blk cwv = ld_blk_stream(k + a.L.cwv + 16 * i);
        const T x = a.xhat[i];
        T acc = 0;
        // expand the remaining Lr levels of this lane's subtree: 2^Lr leaves
        for (int q = 0; q < (1 << Lr); q++) {
            Blk t = s;
            for (int j = 0; j < Lr; j++) {
                uint32_t bit = (uint32_t(q) >> (Lr - 1 - j)) & 1u;
                Blk cw = ld_blk_stream(k + a.L.cw + 16 * (uint64_t(5 + j) * n + i));
                Blk cl = blk_xor(A.hash_h(t), blk_and_mask(cw, 0u - (t.w[0] & 1u)));
                t = blk_xor(cl, blk_and_mask(t, 0u - bit));
            }
            const bool tb = t.w[0] & 1u;
            const Blk g = A.hash_c(t);
            const uint32_t leaf = (uint32_t(lane) << Lr) | uint32_t(q);
#pragma unroll
            for (int kk = 0; kk < EPL; kk++) {
                // arithmetic leaf: Conv(s) + t * CW_v, slot by slot in Z_2^n
                T v = blk_slot<T>(g, kk) + (tb ? blk_slot<T>(cwv, kk) : T(0));
                if (a.party) v = T(0) - v;
                const uint32_t y = leaf * EPL + kk;
                acc += v * tab[(uint32_t(x) - y) & 255u];
            }
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, o);
        if (lane == 0) a.share[i] = acc + reinterpret_cast<const T *>(k + a.L.rout)[i];
    }
}

template <typename T, class E>
static int lut_keygen_launch(const LutKeygenArgs<T> &a, cudaStream_t st)
{
    DDG_CUDA(cudaFuncSetAttribute(lut_keygen_kernel<T, E>, cudaFuncAttributeMaxDynamicSharedMemorySize, E::SMEM));
    lut_keygen_kernel<T, E><<<aes_blocks<E>(a.L.n), E::THREADS, E::SMEM, st>>>(a);
    return DDG_OK;
}

template <typename T, class E>
static int lut_eval_launch(const LutEvalArgs<T> &a, cudaStream_t st)
{
    DDG_CUDA(cudaFuncSetAttribute(lut_eval_kernel<T, E>, cudaFuncAttributeMaxDynamicSharedMemorySize, E::SMEM));
    lut_eval_kernel<T, E><<<aes_blocks<E>(a.L.n * 32), E::THREADS, E::SMEM, st>>>(a);  // a warp per lookup
    return DDG_OK;
}

template <typename T>
int lut_keygen(const LutLayout &L, const AesKey &dk, uint32_t op, const T *alpha_mask, const T *rout, uint8_t *k0,
               uint8_t *k1, cudaStream_t st)
{
    if (!L.n) return DDG_OK;
    DDG_TRY(aes_device_init());
    LutKeygenArgs<T> a{L, dk, op, alpha_mask, rout, k0, k1};
    DDG_TRY((aes_tables() == 4 ? lut_keygen_launch<T, AesLane4>(a, st) : lut_keygen_launch<T, AesLane2>(a, st)));
    note_launch();
    DDG_CUDA(cudaGetLastError());
    return DDG_OK;
}

template <typename T>
int lut_eval(const LutLayout &L, int party, const T *xhat, const T *table, const uint8_t *key, T *share,
             cudaStream_t st)
{
    if (!L.n) return DDG_OK;
    DDG_TRY(aes_device_init());
    LutEvalArgs<T> a{L, party, xhat, table, key, share};
    DDG_TRY((aes_tables() == 4 ? lut_eval_launch<T, AesLane4>(a, st) : lut_eval_launch<T, AesLane2>(a, st)));
    note_launch();
    DDG_CUDA(cudaGetLastError());
    return DDG_OK;
}

// ---------------------------------------------------------------- truth-table LUT

TtLutLayout tt_lut_layout(int bw, uint64_t n, uint64_t base)
{
    TtLutLayout l;
    l.bw = bw;
    l.n = n;
    l.tab = align256(base);
    l.rout = align256(l.tab + 256 * n * uint64_t(bw / 8));
    l.bytes = align256(l.rout + n * uint64_t(bw / 8)) - align256(base);
    return l;
}

template <typename T>
struct TtLutKeygenArgs {
    TtLutLayout L;
    AesKey dk;
    uint32_t op;
    const T *alpha_mask, *rout, *table;
    uint8_t *k0, *k1;
};

// dealer: party 0's entries from the PRG (4 or 2 words per block), party 1's
// = table[(u - alpha) mod 256] + r_out - party 0's
template <typename T, class E>
__global__ void __launch_bounds__(E::THREADS, E::CTAS) tt_lut_keygen_kernel(const __grid_constant__ TtLutKeygenArgs<T> a)
{
    extern __shared__ uint32_t smem_tab[];
    __shared__ T tab[256];
    E::stage(smem_tab);
    for (int i = threadIdx.x; i < 256; i += blockDim.x) tab[i] = a.table[i];
    __syncthreads();
    E A(smem_tab);
    constexpr int EPB = 16 / sizeof(T);
    const uint64_t n = a.L.n;
    for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += uint64_t(gridDim.x) * blockDim.x) {
        const uint32_t alpha = uint32_t(a.alpha_mask[i]) & 255u;
        const T ro = a.rout[i];
        T *t0 = reinterpret_cast<T *>(a.k0 + a.L.tab), *t1 = reinterpret_cast<T *>(a.k1 + a.L.tab);
        for (int b = 0; b < 256 / EPB; b++) {
            const Blk r = A.prg(a.dk.rk, a.op, P_TT_LUT, uint64_t(b) * n + i);
#pragma unroll
            for (int k = 0; k < EPB; k++) {
                const int u = b * EPB + k;
                const T s0 = blk_slot<T>(r, k);
                t0[uint64_t(u) * n + i] = s0;
                t1[uint64_t(u) * n + i] = T(tab[(uint32_t(u) - alpha) & 255u] + ro - s0);
            }
        }
        const T sh = ring_of<T>(A.prg(a.dk.rk, a.op, P_SHARE, i));
        reinterpret_cast<T *>(a.k0 + a.L.rout)[i] = sh;
        reinterpret_cast<T *>(a.k1 + a.L.rout)[i] = ro - sh;
    }
}

template <typename T>
__global__ void tt_lut_eval_kernel(const TtLutLayout L, const T *xhat, const uint8_t *key, T *share)
{
    const T *tab = reinterpret_cast<const T *>(key + L.tab);
    for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < L.n; i += uint64_t(gridDim.x) * blockDim.x)
        share[i] = __ldcs(tab + uint64_t(uint32_t(xhat[i]) & 255u) * L.n + i);
}

template <typename T>
int tt_lut_keygen(const TtLutLayout &L, const AesKey &dk, uint32_t op, const T *alpha_mask, const T *rout,
                  const T *table, uint8_t *k0, uint8_t *k1, cudaStream_t st)
{
    if (!L.n) return DDG_OK;
    DDG_CHECK(k0 && k1 && table, DDG_ERR_ARG, "truth-table LUT keygen needs both keys and the table");
    DDG_TRY(aes_device_init());
    TtLutKeygenArgs<T> a{L, dk, op, alpha_mask, rout, table, k0, k1};
    if (aes_tables() == 4) {
        DDG_CUDA(cudaFuncSetAttribute(tt_lut_keygen_kernel<T, AesLane4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      AesLane4::SMEM));
        tt_lut_keygen_kernel<T, AesLane4><<<aes_blocks<AesLane4>(L.n), AesLane4::THREADS, AesLane4::SMEM, st>>>(a);
    } else {
        DDG_CUDA(cudaFuncSetAttribute(tt_lut_keygen_kernel<T, AesLane2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      AesLane2::SMEM));
        tt_lut_keygen_kernel<T, AesLane2><<<aes_blocks<AesLane2>(L.n), AesLane2::THREADS, AesLane2::SMEM, st>>>(a);
    }
    note_launch();
    DDG_CUDA(cudaGetLastError());
    return DDG_OK;
}

template <typename T>
int tt_lut_eval(const TtLutLayout &L, const T *xhat, const uint8_t *key, T *share, cudaStream_t st)
{
    if (!L.n) return DDG_OK;
    const uint64_t blocks = (L.n + 255) / 256;
    tt_lut_eval_kernel<T><<<int(blocks < 4096 ? blocks : 4096), 256, 0, st>>>(L, xhat, key, share);
    note_launch();
    DDG_CUDA(cudaGetLastError());
    return DDG_OK;
}

template int tt_lut_keygen<uint32_t>(const TtLutLayout &, const AesKey &, uint32_t, const uint32_t *, const uint32_t *,
                                     const uint32_t *, uint8_t *, uint8_t *, cudaStream_t);
template int tt_lut_keygen<uint64_t>(const TtLutLayout &, const AesKey &, uint32_t, const uint64_t *, const uint64_t *,
                                     const uint64_t *, uint8_t *, uint8_t *, cudaStream_t);
template int tt_lut_eval<uint32_t>(const TtLutLayout &, const uint32_t *, const uint8_t *, uint32_t *, cudaStream_t);
template int tt_lut_eval<uint64_t>(const TtLutLayout &, const uint64_t *, const uint8_t *, uint64_t *, cudaStream_t);

template int lut_keygen<uint32_t>(const LutLayout &, const AesKey &, uint32_t, const uint32_t *, const uint32_t *,
                                  uint8_t *, uint8_t *, cudaStream_t);
template int lut_keygen<uint64_t>(const LutLayout &, const AesKey &, uint32_t, const uint64_t *, const uint64_t *,
                                  uint8_t *, uint8_t *, cudaStream_t);
template int lut_eval<uint32_t>(const LutLayout &, int, const uint32_t *, const uint32_t *, const uint8_t *,
                                uint32_t *, cudaStream_t);
template int lut_eval<uint64_t>(const LutLayout &, int, const uint64_t *, const uint64_t *, const uint8_t *,
                                uint64_t *, cudaStream_t);

}  // namespace ddg
