// Ring GEMMs over Z_2^32 / Z_2^64 on the CUDA cores (integer multiply-add
// wraps modulo 2^bits natively).  The tensor-core kernel (ring_gemm_tc.cu) is
// the default; this one serves reduction lengths beyond its exactness bound
// and the comparison tests.  One kernel serves every linear layer:
//
//   C[b] = sign * ( A1[b] . (s1*B1[b] - B1m[b])  -  A2[b] . B2[b] ) + bias + Add[b]
//
// * FC, secret x public weight (FC<T> behind DDGOrcaBase::matmul 4-arg,
//   gpu_mpc/ddg_orca_base.h:208-271): party 0: A1 = x_hat, B1 = W, bias, Add =
//   its key words; dealer: sign = -1, A1 = r_x, B1 = W, Add = r_y.
// * Beaver, secret x secret per sample (DDGOrcaBase::matmul 3-arg,
//   ddg_orca_base.h:170-205, batched loop of sytorch/layers/layers.h:67-90):
//   A1 = A_hat, B1 = H_hat (s1 = 1 for party 0, 0 for party 1), B1m = [r_H],
//   A2 = [r_A], B2 = H_hat, Add = [r_A r_H + r_P]; all B samples in one launch.
// Tiles: 64x64 outputs per 256-thread CTA, 4x4 per thread, K step 16,
// operands staged through shared memory.
#include "common.cuh"
#include "linear.cuh"

namespace ddg {

constexpr int GT = 64, GK = 16;

template <typename T>
__global__ void __launch_bounds__(256) ring_gemm_kernel(const __grid_constant__ GemmArgs<T> a)
{
    __shared__ T As[GK][GT + 1];
    __shared__ T Bs[GK][GT];
    const int b = blockIdx.z;
    const int m0 = blockIdx.y * GT, n0 = blockIdx.x * GT;
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    T acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = 0;

    for (int phase = 0; phase < 2; phase++) {
        const T *A = phase == 0 ? a.A1 : a.A2;
        const T *B = phase == 0 ? a.B1 : a.B2;
        if (A == nullptr) continue;
        const T *Bm = phase == 0 ? a.B1m : nullptr;
        const T s1 = phase == 0 ? a.s1 : T(1);
        const int64_t lda = phase == 0 ? a.lda1 : a.lda2, ldb = phase == 0 ? a.ldb1 : a.ldb2;
        A += int64_t(b) * (phase == 0 ? a.sA1 : a.sA2);
        if (B) B += int64_t(b) * (phase == 0 ? a.sB1 : a.sB2);
        if (Bm) Bm += int64_t(b) * a.sB1m;
        T sub[4][4];
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) sub[i][j] = 0;
        for (int k0 = 0; k0 < a.K; k0 += GK) {
            // A tile GT x GK: 1024 elements, 4 per thread
#pragma unroll
            for (int q = 0; q < 4; q++) {
                int idx = threadIdx.x + q * 256;
                int r = idx / GK, c = idx % GK;
                int gm = m0 + r, gk = k0 + c;
                As[c][r] = (gm < a.M && gk < a.K) ? A[int64_t(gm) * lda + gk] : T(0);
            }
            // B tile GK x GT
#pragma unroll
            for (int q = 0; q < 4; q++) {
                int idx = threadIdx.x + q * 256;
                int r = idx / GT, c = idx % GT;
                int gk = k0 + r, gn = n0 + c;
                T v = 0;
                if (gk < a.K && gn < a.N) {
                    int64_t o = int64_t(gk) * ldb + gn;
                    if (B) v = s1 * B[o];
                    if (Bm) v -= Bm[o];
                }
                Bs[r][c] = v;
            }
            __syncthreads();
#pragma unroll
            for (int kk = 0; kk < GK; kk++) {
                T av[4], bv[4];
#pragma unroll
                for (int i = 0; i < 4; i++) av[i] = As[kk][ty * 4 + i];
#pragma unroll
                for (int j = 0; j < 4; j++) bv[j] = Bs[kk][tx * 4 + j];
#pragma unroll
                for (int i = 0; i < 4; i++)
#pragma unroll
                    for (int j = 0; j < 4; j++) sub[i][j] += av[i] * bv[j];
            }
            __syncthreads();
        }
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) acc[i][j] = phase == 0 ? sub[i][j] : acc[i][j] - sub[i][j];
    }
    const T *Add = a.Add ? a.Add + int64_t(b) * a.sAdd : nullptr;
    T *C = a.C + int64_t(b) * a.sC;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        int gm = m0 + ty * 4 + i;
        if (gm >= a.M) continue;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            int gn = n0 + tx * 4 + j;
            if (gn >= a.N) continue;
            T v = a.sign * acc[i][j];
            if (a.bias) v += a.bias[gn];
            if (Add) v += Add[int64_t(gm) * a.ldAdd + gn];
            C[int64_t(gm) * a.ldc + gn] = v;
        }
    }
}

template <typename T>
int ring_gemm_simt(const GemmArgs<T> &a, cudaStream_t st)
{
    if (a.M == 0 || a.N == 0 || a.batch == 0) return DDG_OK;
    dim3 grid((a.N + GT - 1) / GT, (a.M + GT - 1) / GT, a.batch);
    DDG_CHECK(grid.y <= 65535 && grid.z <= 65535, DDG_ERR_ARG, "gemm grid too large (M=%d batch=%d)", a.M, a.batch);
    ring_gemm_kernel<T><<<grid, 256, 0, st>>>(a);
    note_launch();
    DDG_CUDA(cudaGetLastError());
    return DDG_OK;
}

template int ring_gemm_simt<uint32_t>(const GemmArgs<uint32_t> &, cudaStream_t);
template int ring_gemm_simt<uint64_t>(const GemmArgs<uint64_t> &, cudaStream_t);

// Thin row blocks: the last M % 128 rows of a GEMM whose other rows run on the
// tensor cores in whole 128-row tiles (the per-sample Beaver products have
// 138 rows: a second 128-row tile would do 10 rows of work).  16 rows x 64
// columns per 256-thread CTA; a thread owns one column of four consecutive
// rows, so per k step a warp reads its four A values with one broadcast
// 16-byte shared load (A is staged transposed) and 32 consecutive B values.
// Same formula as ring_gemm_kernel, with the two products run as one sequence
// of K-chunks: the second product's B enters negated, and the next chunk is
// loaded into registers while the current one is multiplied.
constexpr int TR = 16, TN = 64, TK = 32;
constexpr int TQA = TR * TK / 256, TQB = TK * TN / 256;

// chunk `it` of the product sequence into registers: A rows m0.. (TR x TK),
// B' = s1*B1 - B1m for the first product, -B2 for the second (TK x TN)
template <typename T>
__device__ __forceinline__ void thin_load(const GemmArgs<T> &a, int it, int nk, int b, int m0, int n0, T (&ra)[TQA],
                                          T (&rb)[TQB])
{
    const bool second = it >= nk;
    const int k0 = (second ? it - nk : it) * TK;
    const T *A = (second ? a.A2 : a.A1) + int64_t(b) * (second ? a.sA2 : a.sA1);
    const int64_t lda = second ? a.lda2 : a.lda1, ldb = second ? a.ldb2 : a.ldb1;
    const T *B = second ? a.B2 : a.B1;
    const T *Bm = second ? nullptr : a.B1m;
    if (B) B += int64_t(b) * (second ? a.sB2 : a.sB1);
    if (Bm) Bm += int64_t(b) * a.sB1m;
    const T s1 = second ? T(0) - T(1) : a.s1;
#pragma unroll
    for (int q = 0; q < TQA; q++) {
        const int idx = threadIdx.x + q * 256, r = idx / TK, c = idx % TK;
        const int gm = m0 + r, gk = k0 + c;
        ra[q] = (gm < a.M && gk < a.K) ? A[int64_t(gm) * lda + gk] : T(0);
    }
#pragma unroll
    for (int q = 0; q < TQB; q++) {
        const int idx = threadIdx.x + q * 256, r = idx / TN, c = idx % TN;
        const int gk = k0 + r, gn = n0 + c;
        T v = 0;
        if (gk < a.K && gn < a.N) {
            const int64_t o = int64_t(gk) * ldb + gn;
            if (B) v = s1 * B[o];
            if (Bm) v -= Bm[o];
        }
        rb[q] = v;
    }
}

template <typename T>
__global__ void __launch_bounds__(256) ring_gemm_thin_kernel(const __grid_constant__ GemmArgs<T> a)
{
    // A transposed, rows padded to 20 elements: 16-byte aligned row starts,
    // 4-way bank conflicts at most on the transposing stores
    __shared__ __align__(16) T As[TK][TR + 4];
    __shared__ T Bs[TK][TN];
    const int b = blockIdx.z;
    const int m0 = blockIdx.y * TR, n0 = blockIdx.x * TN;
    const int col = threadIdx.x % TN, rg = threadIdx.x / TN;
    const int nk = (a.K + TK - 1) / TK, nit = a.A2 ? 2 * nk : nk;
    T acc[4] = {0, 0, 0, 0};
    T ra[TQA], rb[TQB];
    if (nit > 0) thin_load<T>(a, 0, nk, b, m0, n0, ra, rb);
    for (int it = 0; it < nit; it++) {
#pragma unroll
        for (int q = 0; q < TQA; q++) {
            const int idx = threadIdx.x + q * 256;
            As[idx % TK][idx / TK] = ra[q];
        }
#pragma unroll
        for (int q = 0; q < TQB; q++) {
            const int idx = threadIdx.x + q * 256;
            Bs[idx / TN][idx % TN] = rb[q];
        }
        __syncthreads();
        if (it + 1 < nit) thin_load<T>(a, it + 1, nk, b, m0, n0, ra, rb);
#pragma unroll 8
        for (int kk = 0; kk < TK; kk++) {
            const T bv = Bs[kk][col];
            T av[4];
            if constexpr (sizeof(T) == 4) {
                const uint4 v = *reinterpret_cast<const uint4 *>(&As[kk][4 * rg]);
                av[0] = v.x, av[1] = v.y, av[2] = v.z, av[3] = v.w;
            } else {
                const ulonglong2 v0 = *reinterpret_cast<const ulonglong2 *>(&As[kk][4 * rg]);
                const ulonglong2 v1 = *reinterpret_cast<const ulonglong2 *>(&As[kk][4 * rg + 2]);
                av[0] = v0.x, av[1] = v0.y, av[2] = v1.x, av[3] = v1.y;
            }
#pragma unroll
            for (int i = 0; i < 4; i++) acc[i] += av[i] * bv;
        }
        __syncthreads();
    }
    const int gn = n0 + col;
    if (gn >= a.N) return;
    const T *Add = a.Add ? a.Add + int64_t(b) * a.sAdd : nullptr;
    T *C = a.C + int64_t(b) * a.sC;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int gm = m0 + 4 * rg + i;
        if (gm >= a.M) continue;
        T v = a.sign * acc[i];
        if (a.bias) v += a.bias[gn];
        if (Add) v += Add[int64_t(gm) * a.ldAdd + gn];
        C[int64_t(gm) * a.ldc + gn] = v;
    }
}

template <typename T>
int ring_gemm_rows(const GemmArgs<T> &a, int m0, cudaStream_t st)
{
    DDG_CHECK(m0 >= 0 && m0 <= a.M && a.A1 && a.C, DDG_ERR_ARG, "gemm rows: bad row offset or operand");
    if (m0 == a.M || a.N == 0 || a.batch == 0) return DDG_OK;
    GemmArgs<T> t = a;
    t.M = a.M - m0;
    t.A1 = a.A1 + int64_t(m0) * a.lda1;
    if (a.A2) t.A2 = a.A2 + int64_t(m0) * a.lda2;
    if (a.Add) t.Add = a.Add + int64_t(m0) * a.ldAdd;
    t.C = a.C + int64_t(m0) * a.ldc;
    dim3 grid((t.N + TN - 1) / TN, (t.M + TR - 1) / TR, t.batch);
    DDG_CHECK(grid.y <= 65535 && grid.z <= 65535, DDG_ERR_ARG, "gemm grid too large (M=%d batch=%d)", t.M, t.batch);
    ring_gemm_thin_kernel<T><<<grid, 256, 0, st>>>(t);
    note_launch();
    DDG_CUDA(cudaGetLastError());
    return DDG_OK;
}

template int ring_gemm_rows<uint32_t>(const GemmArgs<uint32_t> &, int, cudaStream_t);
template int ring_gemm_rows<uint64_t>(const GemmArgs<uint64_t> &, int, cudaStream_t);

}  // namespace ddg
