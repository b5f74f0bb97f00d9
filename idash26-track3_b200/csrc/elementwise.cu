// Elementwise kernels of the online graph and of the dealer: openings,
// Beaver products with row/column broadcast (secure_adj_norm.h:609-651 mul1 /
// mul2, deepdtagen.h:198 mask multiply), the max-pool tree level data movement
// (masked_maxpool_layer.h:72-126, fused into index arithmetic instead of
// cudaMemcpy2D + per-pair copies), the per-row concat (deepdtagen.h:45-100),
// degree row sums (secure_adj_norm.h:44-78) and the dealer's PRG fills.
#include "aes_dev.cuh"
#include "gates.cuh"
#include "linear.cuh"

namespace ddg {

static int ew_grid(uint64_t n)
{
    static int sms = 0;
    if (!sms) sms = device_sms();
    uint64_t blocks = (n + 255) / 256, cap = uint64_t(sms > 0 ? sms : 148) * 16;
    return int(blocks < cap ? (blocks ? blocks : 1) : cap);
}

#define GRID_STRIDE(i, n) \
    for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < (n); i += uint64_t(gridDim.x) * blockDim.x)

template <typename T>
__global__ void k_add(T *out, const T *a, const T *b, uint64_t n)
{
    GRID_STRIDE(i, n) out[i] = a[i] + b[i];
}

// the same on 16-byte vectors (all three pointers 16-byte aligned); the
// n % V tail elements go through k_add
template <typename T>
__global__ void k_add_v16(T *out, const T *a, const T *b, uint64_t nv)
{
    constexpr int V = 16 / sizeof(T);
    GRID_STRIDE(i, nv)
    {
        uint4 x = reinterpret_cast<const uint4 *>(a)[i], y = reinterpret_cast<const uint4 *>(b)[i];
        T *xs = reinterpret_cast<T *>(&x);
        const T *ys = reinterpret_cast<const T *>(&y);
#pragma unroll
        for (int k = 0; k < V; k++) xs[k] += ys[k];
        reinterpret_cast<uint4 *>(out)[i] = x;
    }
}

template <typename T>
__global__ void k_sub(T *out, const T *a, const T *b, uint64_t n)
{
    GRID_STRIDE(i, n) out[i] = a[i] - b[i];
}

template <typename T>
int ew_add(T *out, const T *a, const T *b, uint64_t n, cudaStream_t st)
{
    if (!n) return DDG_OK;
    constexpr uint64_t V = 16 / sizeof(T);
    const bool vec = ((uintptr_t(out) | uintptr_t(a) | uintptr_t(b)) & 15) == 0 && n >= V;
    if (vec) {
        const uint64_t nv = n / V;
        k_add_v16<T><<<ew_grid(nv), 256, 0, st>>>(out, a, b, nv);
        note_launch();
        DDG_CUDA(cudaGetLastError());
        if (n % V == 0) return DDG_OK;
        out += nv * V, a += nv * V, b += nv * V, n -= nv * V;
    }
    k_add<T><<<ew_grid(n), 256, 0, st>>>(out, a, b, n);
    note_launch();
    DDG_CUDA(cudaGetLastError());
    return DDG_OK;
}

template <typename T>
int ew_sub(T *out, const T *a, const T *b, uint64_t n, cudaStream_t st)
{
    if (!n) return DDG_OK;
    k_sub<T><<<ew_grid(n), 256, 0, st>>>(out, a, b, n);
    note_launch();
    DDG_CUDA(cudaGetLastError());
    return DDG_OK;
}

__device__ __forceinline__ uint64_t bc_index(uint64_t e, int bc, int R, int C)
{
    if (bc == BC_ROW) return e / uint64_t(C);                                   // (b*R + i)
    if (bc == BC_COL) return (e / (uint64_t(R) * C)) * uint64_t(C) + e % uint64_t(C);  // (b*C + j)
    return e;
}

template <typename T>
__global__ void k_beaver(T p0, uint64_t n, int bc, int R, int C, const T *xh, const T *yh, const T *msx, const T *msy,
                         const T *Z, T *out, const T *xh2, const T *yh2)
{
    GRID_STRIDE(e, n)
    {
        const uint64_t j = bc_index(e, bc, R, C);
        T x = xh[e], y = yh[j];
        if (xh2) x += xh2[e];
        if (yh2) y += yh2[j];
        out[e] = p0 * x * y - x * msy[j] - msx[e] * y + Z[e];
    }
}

template <typename T>
int beaver_ew(int party, const EwShape &sh, Bcast bc, const T *xh, const T *yh, const T *msx, const T *msy, const T *Z,
              T *out, cudaStream_t st, const T *xh2, const T *yh2)
{
    if (!sh.n) return DDG_OK;
    k_beaver<T><<<ew_grid(sh.n), 256, 0, st>>>(party == 0 ? T(1) : T(0), sh.n, int(bc), sh.R, sh.C, xh, yh, msx, msy,
                                               Z, out, xh2, yh2);
    note_launch();
    DDG_CUDA(cudaGetLastError());
    return DDG_OK;
}

template <typename T>
__global__ void k_beaver_z(uint64_t n, int bc, int R, int C, const T *rx, const T *ry, const T *rout, T *Z)
{
    GRID_STRIDE(e, n) Z[e] = rx[e] * ry[bc_index(e, bc, R, C)] + rout[e];
}

template <typename T>
int beaver_ew_z(const EwShape &sh, Bcast bc, const T *rx, const T *ry, const T *rout, T *Z, cudaStream_t st)
{
    if (!sh.n) return DDG_OK;
    k_beaver_z<T><<<ew_grid(sh.n), 256, 0, st>>>(sh.n, int(bc), sh.R, sh.C, rx, ry, rout, Z);
    note_launch();
    DDG_CUDA(cudaGetLastError());
    return DDG_OK;
}

// one warp per row: lanes stride over the columns, shuffle reduction
template <typename T>
__global__ void k_rowsum(const T *a, const T *m, T *out, uint64_t rows, int cols)
{
    const uint64_t warp = (uint64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const uint64_t nwarps = (uint64_t(gridDim.x) * blockDim.x) >> 5;
    for (uint64_t r = warp; r < rows; r += nwarps) {
        T s = 0;
        for (int j = lane; j < cols; j += 32) s += a[r * cols + j];
#pragma unroll
        for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, o);
        if (lane == 0) out[r] = s + (m ? m[r] : T(0));
    }
}

template <typename T>
int rowsum_plus(const T *a, const T *m, T *out, uint64_t rows, int cols, cudaStream_t st)
{
    if (!rows) return DDG_OK;
    k_rowsum<T><<<ew_grid(rows * 32), 256, 0, st>>>(a, m, out, rows, cols);
    note_launch();
    DDG_CUDA(cudaGetLastError());
    return DDG_OK;
}

template <typename T>
__global__ void k_pool_split(const T *cur, const T *cur2, T *even, T *diff, int B, int cnt, int F)
{
    const int pairs = cnt / 2;
    const uint64_t n = uint64_t(B) * pairs * F;
    GRID_STRIDE(e, n)
    {
        const int f = int(e % F);
        const uint64_t bp = e / F;
        const int p = int(bp % pairs);
        const uint64_t b = bp / pairs;
        const uint64_t base = (b * cnt + 2 * p) * uint64_t(F) + f;
        T ev = cur[base], od = cur[base + F];
        if (cur2) ev += cur2[base], od += cur2[base + F];
        even[e] = ev;
        diff[e] = od - ev;
    }
}

// 16-byte vector forms of the max-pool level kernels: a row of F ring words is
// F / L vectors (L = 4 for Z_2^32, 2 for Z_2^64), and a thread finds its row
// and vector with two 32-bit divisions per 16 bytes instead of 64-bit
// divisions per element.  Used when F is a multiple of L, the buffers are
// 16-byte aligned and the vector count fits 32 bits.
template <typename T>
struct Vec16;
template <>
struct Vec16<uint32_t> {
    using V = uint4;
    static constexpr int L = 4;
    __device__ static V add(V a, V b) { return make_uint4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w); }
    __device__ static V sub(V a, V b) { return make_uint4(a.x - b.x, a.y - b.y, a.z - b.z, a.w - b.w); }
};
template <>
struct Vec16<uint64_t> {
    using V = ulonglong2;
    static constexpr int L = 2;
    __device__ static V add(V a, V b) { return make_ulonglong2(a.x + b.x, a.y + b.y); }
    __device__ static V sub(V a, V b) { return make_ulonglong2(a.x - b.x, a.y - b.y); }
};

template <typename T>
__global__ void k_pool_split_v(const typename Vec16<T>::V *cur, const typename Vec16<T>::V *cur2,
                               typename Vec16<T>::V *even, typename Vec16<T>::V *diff, uint32_t pairs, uint32_t cnt,
                               uint32_t fv, uint32_t nvec)
{
    using W = Vec16<T>;
    for (uint32_t t = blockIdx.x * blockDim.x + threadIdx.x; t < nvec; t += gridDim.x * blockDim.x) {
        const uint32_t row = t / fv, c = t - row * fv;
        const uint32_t b = row / pairs, p = row - b * pairs;
        const uint64_t src = (uint64_t(b) * cnt + 2 * p) * fv + c;
        typename W::V ev = cur[src], od = cur[src + fv];
        if (cur2) ev = W::add(ev, cur2[src]), od = W::add(od, cur2[src + fv]);
        even[t] = ev;
        diff[t] = W::sub(od, ev);
    }
}

template <typename T>
__global__ void k_pool_merge_v(const typename Vec16<T>::V *even, const typename Vec16<T>::V *relu,
                               const typename Vec16<T>::V *relu2, const typename Vec16<T>::V *cur,
                               const typename Vec16<T>::V *cur2, typename Vec16<T>::V *next, uint32_t pairs,
                               uint32_t cnt, uint32_t fv, uint32_t nvec)
{
    using W = Vec16<T>;
    const uint32_t nxt = pairs + (cnt & 1);
    for (uint32_t t = blockIdx.x * blockDim.x + threadIdx.x; t < nvec; t += gridDim.x * blockDim.x) {
        const uint32_t row = t / fv, c = t - row * fv;
        const uint32_t b = row / nxt, q = row - b * nxt;
        typename W::V v;
        if (q < pairs) {
            const uint64_t i = (uint64_t(b) * pairs + q) * fv + c;
            v = W::add(even[i], relu[i]);
            if (relu2) v = W::add(v, relu2[i]);
        } else {
            const uint64_t i = (uint64_t(b) * cnt + (cnt - 1)) * fv + c;
            v = cur[i];
            if (cur2) v = W::add(v, cur2[i]);
        }
        next[t] = v;
    }
}

inline bool al16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

template <typename T>
int pool_split(const T *cur, T *even, T *diff, int B, int cnt, int F, cudaStream_t st, const T *cur2)
{
    const uint64_t n = uint64_t(B) * (cnt / 2) * F;
    if (!n) return DDG_OK;
    constexpr int L = Vec16<T>::L;
    if (F % L == 0 && n / L < (1ull << 31) && al16(cur) && al16(cur2) && al16(even) && al16(diff)) {
        using V = typename Vec16<T>::V;
        const uint32_t nvec = uint32_t(n / L);
        k_pool_split_v<T><<<ew_grid(nvec), 256, 0, st>>>(
            reinterpret_cast<const V *>(cur), reinterpret_cast<const V *>(cur2), reinterpret_cast<V *>(even),
            reinterpret_cast<V *>(diff), uint32_t(cnt / 2), uint32_t(cnt), uint32_t(F / L), nvec);
    } else {
        k_pool_split<T><<<ew_grid(n), 256, 0, st>>>(cur, cur2, even, diff, B, cnt, F);
    }
    note_launch();
    DDG_CUDA(cudaGetLastError());
    return DDG_OK;
}

template <typename T>
__global__ void k_pool_merge(const T *even, const T *relu, const T *relu2, const T *cur, const T *cur2, T *next,
                             int B, int cnt, int F)
{
    const int pairs = cnt / 2, nxt = pairs + (cnt & 1);
    const uint64_t n = uint64_t(B) * nxt * F;
    GRID_STRIDE(e, n)
    {
        const int f = int(e % F);
        const uint64_t bq = e / F;
        const int q = int(bq % nxt);
        const uint64_t b = bq / nxt;
        T v;
        if (q < pairs) {
            const uint64_t s = (b * pairs + q) * uint64_t(F) + f;
            v = even[s] + relu[s];
            if (relu2) v += relu2[s];
        } else {
            const uint64_t s = (b * cnt + (cnt - 1)) * uint64_t(F) + f;
            v = cur[s];
            if (cur2) v += cur2[s];
        }
        next[e] = v;
    }
}

template <typename T>
int pool_merge(const T *even, const T *relu, const T *cur, T *next, int B, int cnt, int F, cudaStream_t st,
               const T *relu2, const T *cur2)
{
    const uint64_t n = uint64_t(B) * (cnt / 2 + (cnt & 1)) * F;
    if (!n) return DDG_OK;
    constexpr int L = Vec16<T>::L;
    if (F % L == 0 && n / L < (1ull << 31) && al16(even) && al16(relu) && al16(relu2) && al16(cur) && al16(cur2) &&
        al16(next)) {
        using V = typename Vec16<T>::V;
        const uint32_t nvec = uint32_t(n / L);
        k_pool_merge_v<T><<<ew_grid(nvec), 256, 0, st>>>(
            reinterpret_cast<const V *>(even), reinterpret_cast<const V *>(relu), reinterpret_cast<const V *>(relu2),
            reinterpret_cast<const V *>(cur), reinterpret_cast<const V *>(cur2), reinterpret_cast<V *>(next),
            uint32_t(cnt / 2), uint32_t(cnt), uint32_t(F / L), nvec);
    } else {
        k_pool_merge<T><<<ew_grid(n), 256, 0, st>>>(even, relu, relu2, cur, cur2, next, B, cnt, F);
    }
    note_launch();
    DDG_CUDA(cudaGetLastError());
    return DDG_OK;
}

template <typename T>
__global__ void k_concat(const T *a, const T *b, T *out, int B, int wa, int wb)
{
    const int w = wa + wb;
    const uint64_t n = uint64_t(B) * w;
    GRID_STRIDE(e, n)
    {
        const uint64_t r = e / w;
        const int c = int(e % w);
        out[e] = c < wa ? a[r * wa + c] : (b ? b[r * wb + (c - wa)] : T(0));
    }
}

template <typename T>
int concat_rows(const T *a, const T *b, T *out, int B, int wa, int wb, cudaStream_t st)
{
    const uint64_t n = uint64_t(B) * (wa + wb);
    if (!n) return DDG_OK;
    k_concat<T><<<ew_grid(n), 256, 0, st>>>(a, b, out, B, wa, wb);
    note_launch();
    DDG_CUDA(cudaGetLastError());
    return DDG_OK;
}

template <typename T>
__global__ void k_unmask_ars(const T *xh, const T *r, T *out, uint64_t n, int s)
{
    using S = typename std::conditional<sizeof(T) == 4, int32_t, int64_t>::type;
    GRID_STRIDE(i, n) out[i] = T(S(T(xh[i] - r[i])) >> s);
}

template <typename T>
int unmask_ars(const T *xh, const T *r, T *out, uint64_t n, int s, cudaStream_t st)
{
    if (!n) return DDG_OK;
    k_unmask_ars<T><<<ew_grid(n), 256, 0, st>>>(xh, r, out, n, s);
    note_launch();
    DDG_CUDA(cudaGetLastError());
    return DDG_OK;
}

template <typename T>
__global__ void k_i64_to_ring(const int64_t *in, T *out, uint64_t n, int shl)
{
    GRID_STRIDE(i, n) out[i] = T(uint64_t(in[i]) << shl);
}

template <typename T>
int i64_to_ring(const int64_t *in, T *out, uint64_t n, int shl, cudaStream_t st)
{
    if (!n) return DDG_OK;
    k_i64_to_ring<T><<<ew_grid(n), 256, 0, st>>>(in, out, n, shl);
    note_launch();
    DDG_CUDA(cudaGetLastError());
    return DDG_OK;
}

// ------------------------------------------------------------ dealer PRG

template <typename T, class E>
__global__ void __launch_bounds__(E::THREADS, E::CTAS) k_prg_split(const T *v, uint64_t n,
                                                                   const __grid_constant__ AesKey dk, uint32_t op,
                                                                   uint32_t purpose, T *s0, T *s1)
{
    extern __shared__ uint32_t smem_tab[];
    E::stage(smem_tab);
    __syncthreads();
    E A(smem_tab);
    GRID_STRIDE(i, n)
    {
        Blk b = A.prg(dk.rk, op, purpose, i);
        T r;
        if constexpr (sizeof(T) == 4) r = b.w[0];
        else r = uint64_t(b.w[0]) | (uint64_t(b.w[1]) << 32);
        if (s0) s0[i] = r;
        if (s1) s1[i] = (v ? v[i] : T(0)) - r;
    }
}

template <typename T>
static int prg_launch(const T *v, uint64_t n, const AesKey &dk, uint32_t op, uint32_t purpose, T *s0, T *s1,
                      cudaStream_t st)
{
    if (!n) return DDG_OK;
    DDG_TRY(aes_device_init());
    if (aes_tables() == 4) {
        using E = AesLane4;
        DDG_CUDA(cudaFuncSetAttribute(k_prg_split<T, E>, cudaFuncAttributeMaxDynamicSharedMemorySize, E::SMEM));
        k_prg_split<T, E><<<aes_blocks<E>(n), E::THREADS, E::SMEM, st>>>(v, n, dk, op, purpose, s0, s1);
    } else {
        using E = AesLane2;
        DDG_CUDA(cudaFuncSetAttribute(k_prg_split<T, E>, cudaFuncAttributeMaxDynamicSharedMemorySize, E::SMEM));
        k_prg_split<T, E><<<aes_blocks<E>(n), E::THREADS, E::SMEM, st>>>(v, n, dk, op, purpose, s0, s1);
    }
    note_launch();
    DDG_CUDA(cudaGetLastError());
    return DDG_OK;
}

template <typename T>
int prg_fill(T *out, uint64_t n, const AesKey &dk, uint32_t op, uint32_t purpose, cudaStream_t st)
{
    return prg_launch<T>(nullptr, n, dk, op, purpose, out, nullptr, st);
}

template <typename T>
int split_shares(const T *v, uint64_t n, const AesKey &dk, uint32_t op, uint32_t purpose, T *s0, T *s1, cudaStream_t st)
{
    return prg_launch<T>(v, n, dk, op, purpose, s0, s1, st);
}

#define INST(T)                                                                                                  \
    template int ew_add<T>(T *, const T *, const T *, uint64_t, cudaStream_t);                                   \
    template int ew_sub<T>(T *, const T *, const T *, uint64_t, cudaStream_t);                                   \
    template int beaver_ew<T>(int, const EwShape &, Bcast, const T *, const T *, const T *, const T *, const T *, \
                              T *, cudaStream_t, const T *, const T *);                                                                \
    template int beaver_ew_z<T>(const EwShape &, Bcast, const T *, const T *, const T *, T *, cudaStream_t);     \
    template int rowsum_plus<T>(const T *, const T *, T *, uint64_t, int, cudaStream_t);                         \
    template int pool_split<T>(const T *, T *, T *, int, int, int, cudaStream_t, const T *);                     \
    template int pool_merge<T>(const T *, const T *, const T *, T *, int, int, int, cudaStream_t, const T *,       \
                               const T *);                                                                        \
    template int concat_rows<T>(const T *, const T *, T *, int, int, int, cudaStream_t);                         \
    template int unmask_ars<T>(const T *, const T *, T *, uint64_t, int, cudaStream_t);                          \
    template int i64_to_ring<T>(const int64_t *, T *, uint64_t, int, cudaStream_t);                              \
    template int prg_fill<T>(T *, uint64_t, const AesKey &, uint32_t, uint32_t, cudaStream_t);                   \
    template int split_shares<T>(const T *, uint64_t, const AesKey &, uint32_t, uint32_t, T *, T *, cudaStream_t);
INST(uint32_t)
INST(uint64_t)

}  // namespace ddg
