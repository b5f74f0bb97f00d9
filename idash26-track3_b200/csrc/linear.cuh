// Linear / elementwise building blocks of the online graph and the dealer.
#pragma once
#include "aes_dev.cuh"
#include "common.cuh"

namespace ddg {

template <typename T>
struct GemmArgs {
    int M = 0, N = 0, K = 0, batch = 1;
    const T *A1 = nullptr, *B1 = nullptr, *B1m = nullptr;
    int64_t lda1 = 0, ldb1 = 0, sA1 = 0, sB1 = 0, sB1m = 0;
    T s1 = 1;
    const T *A2 = nullptr, *B2 = nullptr;
    int64_t lda2 = 0, ldb2 = 0, sA2 = 0, sB2 = 0;
    T sign = 1;
    const T *bias = nullptr;
    const T *Add = nullptr;
    int64_t ldAdd = 0, sAdd = 0;
    T *C = nullptr;
    int64_t ldc = 0, sC = 0;
    // optional second addends of A1, B1, B2 (same strides): the operand is
    // A1 + A1b etc., an opened value still held as the two parties' shares
    const T *A1b = nullptr, *B1b = nullptr, *B2b = nullptr;
    // packed engine only: a caller-owned buffer (ring_gemm_a_pack_bytes) for the
    // A operand's byte planes, kept after the call; apk_ready: it already holds
    // this A operand (the packing is skipped).  Other engines ignore both.
    uint8_t *apk_keep = nullptr;
    int apk_ready = 0;
};

// tensor-core limb GEMM where the shape allows (ring_gemm_tc.cu), else the CUDA-core kernel
template <typename T>
int ring_gemm(const GemmArgs<T> &a, cudaStream_t st);
// bytes of the packed A operand when the packed engine takes this GEMM, else 0
template <typename T>
uint64_t ring_gemm_a_pack_bytes(const GemmArgs<T> &a);
// the CUDA-core kernel (ring_gemm.cu)
template <typename T>
int ring_gemm_simt(const GemmArgs<T> &a, cudaStream_t st);
// rows [m0, M) of a on the CUDA cores, 16-row blocks (ring_gemm.cu): the
// ragged last rows of a tensor-core GEMM
template <typename T>
int ring_gemm_rows(const GemmArgs<T> &a, int m0, cudaStream_t st);
// DDG_OK unless a tensor-core GEMM launch gave up on one of its bounded waits
// since the last clear (reads a device word: synchronises with the device)
int ring_gemm_tc_error(bool clear);
// the same check ordered on stream st (waits for st only; does not clear)
int ring_gemm_tc_check(cudaStream_t st);
// 0: tensor cores where the shape allows (default), 1: CUDA cores only
void set_gemm_path(int path);
int gemm_path();

// broadcast pattern of the second operand of an elementwise product over
// (B, R, C) = (batch, rows, cols):  none (same shape), row (index b*R + i),
// col (index b*C + j)
enum Bcast { BC_NONE = 0, BC_ROW = 1, BC_COL = 2 };

struct EwShape {
    uint64_t n = 0;     // elements of the output
    int R = 1, C = 1;   // rows/cols for the broadcast patterns
};

template <typename T>
int ew_add(T *out, const T *a, const T *b, uint64_t n, cudaStream_t st);
template <typename T>
int ew_sub(T *out, const T *a, const T *b, uint64_t n, cudaStream_t st);

// party share of x*y: p0*xh*yh - xh*[r_y] - [r_x]*yh + Z (xh2, yh2: second
// addends of the opened inputs, or null)
template <typename T>
int beaver_ew(int party, const EwShape &sh, Bcast bc, const T *xh, const T *yh, const T *msx, const T *msy, const T *Z,
              T *out, cudaStream_t st, const T *xh2 = nullptr, const T *yh2 = nullptr);
// dealer: Z = r_x * r_y + r_out
template <typename T>
int beaver_ew_z(const EwShape &sh, Bcast bc, const T *rx, const T *ry, const T *rout, T *Z, cudaStream_t st);

// out[row] = sum_j a[row, j] + m[row]   (rows x cols)
template <typename T>
int rowsum_plus(const T *a, const T *m, T *out, uint64_t rows, int cols, cudaStream_t st);

// max-pool tree level over cur (B, cnt, F): even[b,p,f] = cur[b,2p,f],
// diff[b,p,f] = cur[b,2p+1,f] - cur[b,2p,f] for p < cnt/2.  A non-null second
// addend (cur2, relu2) is added on load: an opened value still held as the
// two parties' shares.
template <typename T>
int pool_split(const T *cur, T *even, T *diff, int B, int cnt, int F, cudaStream_t st, const T *cur2 = nullptr);
// next[b,p,f] = even[b,p,f] + relu[b,p,f] (p < cnt/2), carried cur[b,cnt-1,f] if cnt odd
template <typename T>
int pool_merge(const T *even, const T *relu, const T *cur, T *next, int B, int cnt, int F, cudaStream_t st,
               const T *relu2 = nullptr, const T *cur2 = nullptr);

// out (B, wa+wb) = [a (B, wa) | b (B, wb)] per row
template <typename T>
int concat_rows(const T *a, const T *b, T *out, int B, int wa, int wb, cudaStream_t st);

// out[i] = arithmetic shift of (xh[i] - r[i]) by s  (revealed output)
template <typename T>
int unmask_ars(const T *xh, const T *r, T *out, uint64_t n, int s, cudaStream_t st);

// dealer randomness: out[i] = ring(AES_K(i || op || purpose))
template <typename T>
int prg_fill(T *out, uint64_t n, const AesKey &dk, uint32_t op, uint32_t purpose, cudaStream_t st);
// dealer sharing: s0[i] = ring(AES_K(i || op || purpose)), s1 = v - s0 (either output may be null)
template <typename T>
int split_shares(const T *v, uint64_t n, const AesKey &dk, uint32_t op, uint32_t purpose, T *s0, T *s1,
                 cudaStream_t st);
// widen an int64 host-layout array to ring elements, optionally shifted left
template <typename T>
int i64_to_ring(const int64_t *in, T *out, uint64_t n, int shl, cudaStream_t st);

// ------------------------------------------------------------------ DPF LUT (lut.cu)

// key layout of n lookups: root[n] 16 B | cw[L][n] 16 B | cwv[n] 16 B | rout share[n] words
struct LutLayout {
    int bw = 0, L = 0;
    uint64_t n = 0, root = 0, cw = 0, cwv = 0, rout = 0, bytes = 0;
};
LutLayout lut_layout(int bw, uint64_t n, uint64_t base = 0);

template <typename T>
int lut_keygen(const LutLayout &L, const AesKey &dk, uint32_t op, const T *alpha_mask, const T *rout, uint8_t *k0,
               uint8_t *k1, cudaStream_t st);
template <typename T>
int lut_eval(const LutLayout &L, int party, const T *xhat, const T *table, const uint8_t *key, T *share,
             cudaStream_t st);

// ------------------------------------------------------------------ truth-table LUT (lut.cu)
//
// The same 8-bit look-up for the truth-table backend: the dealer gives party
// p a table T_p[256] per lookup with T_0[u] + T_1[u] = table[(u - alpha) mod
// 256] + r_out (alpha the input mask), and party p's share is T_p[x_hat mod
// 256]: one word read, no AES.  Layout of n lookups: tab[256][n] words |
// rout share[n] words (as the DPF layout, for the masks of later products).
struct TtLutLayout {
    int bw = 0;
    uint64_t n = 0, tab = 0, rout = 0, bytes = 0;
};
TtLutLayout tt_lut_layout(int bw, uint64_t n, uint64_t base = 0);

template <typename T>
int tt_lut_keygen(const TtLutLayout &L, const AesKey &dk, uint32_t op, const T *alpha_mask, const T *rout,
                  const T *table, uint8_t *k0, uint8_t *k1, cudaStream_t st);
template <typename T>
int tt_lut_eval(const TtLutLayout &L, const T *xhat, const uint8_t *key, T *share, cudaStream_t st);

}  // namespace ddg
