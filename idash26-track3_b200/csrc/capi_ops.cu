// extern "C" per-op entry points of the linear layers and the DPF LUT: one
// party's share computation, no communication (the caller opens).
#include "aes_dev.cuh"
#include "common.cuh"
#include "linear.cuh"

using namespace ddg;

static int check_bw(int bw)
{
    DDG_CHECK(bw == 32 || bw == 64, DDG_ERR_ARG, "bw must be 32 or 64 (got %d)", bw);
    return DDG_OK;
}

template <typename T>
static int matmul_t(int party, int batch, int M, int K, int N, const void *A, const void *Bm, const void *msA,
                    const void *msB, const void *Z, void *out, cudaStream_t st)
{
    GemmArgs<T> g;
    g.M = M, g.N = N, g.K = K, g.batch = batch;
    g.A1 = (const T *)A, g.lda1 = K, g.sA1 = int64_t(M) * K;
    g.B1 = (const T *)Bm, g.ldb1 = N, g.sB1 = int64_t(K) * N, g.s1 = party == 0 ? T(1) : T(0);
    g.B1m = (const T *)msB, g.sB1m = int64_t(K) * N;
    g.A2 = (const T *)msA, g.lda2 = K, g.sA2 = int64_t(M) * K;
    g.B2 = (const T *)Bm, g.ldb2 = N, g.sB2 = int64_t(K) * N;
    g.Add = (const T *)Z, g.ldAdd = N, g.sAdd = int64_t(M) * N;
    g.C = (T *)out, g.ldc = N, g.sC = int64_t(M) * N;
    return ring_gemm<T>(g, st);
}

template <typename T>
static int fc_t(int party, int M, int K, int N, const void *x, const void *W, const void *b2s, const void *C, void *out,
                cudaStream_t st)
{
    if (party == 1) {
        if (uint64_t(M) * N)
            DDG_CUDA(cudaMemcpyAsync(out, C, uint64_t(M) * N * sizeof(T), cudaMemcpyDeviceToDevice, st));
        return DDG_OK;
    }
    GemmArgs<T> g;
    g.M = M, g.N = N, g.K = K;
    g.A1 = (const T *)x, g.lda1 = K;
    g.B1 = (const T *)W, g.ldb1 = N;
    g.bias = (const T *)b2s;
    g.Add = (const T *)C, g.ldAdd = N;
    g.C = (T *)out, g.ldc = N;
    return ring_gemm<T>(g, st);
}

extern "C" {

uint64_t ddg_lut_key_bytes(int bw, uint64_t n)
{
    if (check_bw(bw) != DDG_OK) return 0;
    return lut_layout(bw, n).bytes;
}

int ddg_lut_keygen(int bw, uint64_t n, uint64_t seed, uint32_t op_id, const void *d_alpha_mask, const void *d_rout,
                   void *d_key0, void *d_key1, void *stream)
{
    DDG_TRY(check_bw(bw));
    DDG_CHECK(n == 0 || (d_alpha_mask && d_rout && (d_key0 || d_key1)), DDG_ERR_ARG, "null pointer");
    LutLayout L = lut_layout(bw, n);
    AesKey dk = dealer_key(seed);
    auto st = static_cast<cudaStream_t>(stream);
    auto *k0 = static_cast<uint8_t *>(d_key0), *k1 = static_cast<uint8_t *>(d_key1);
    return bw == 32 ? lut_keygen<uint32_t>(L, dk, op_id, static_cast<const uint32_t *>(d_alpha_mask),
                                           static_cast<const uint32_t *>(d_rout), k0, k1, st)
                    : lut_keygen<uint64_t>(L, dk, op_id, static_cast<const uint64_t *>(d_alpha_mask),
                                           static_cast<const uint64_t *>(d_rout), k0, k1, st);
}

uint64_t ddg_tt_lut_key_bytes(int bw, uint64_t n)
{
    if (check_bw(bw) != DDG_OK) return 0;
    return tt_lut_layout(bw, n).bytes;
}

int ddg_tt_lut_keygen(int bw, uint64_t n, uint64_t seed, uint32_t op_id, const void *d_alpha_mask, const void *d_rout,
                      const void *d_table, void *d_key0, void *d_key1, void *stream)
{
    DDG_TRY(check_bw(bw));
    DDG_CHECK(n == 0 || (d_alpha_mask && d_rout && d_table && d_key0 && d_key1), DDG_ERR_ARG, "null pointer");
    TtLutLayout L = tt_lut_layout(bw, n);
    AesKey dk = dealer_key(seed);
    auto st = static_cast<cudaStream_t>(stream);
    auto *k0 = static_cast<uint8_t *>(d_key0), *k1 = static_cast<uint8_t *>(d_key1);
    return bw == 32 ? tt_lut_keygen<uint32_t>(L, dk, op_id, static_cast<const uint32_t *>(d_alpha_mask),
                                              static_cast<const uint32_t *>(d_rout),
                                              static_cast<const uint32_t *>(d_table), k0, k1, st)
                    : tt_lut_keygen<uint64_t>(L, dk, op_id, static_cast<const uint64_t *>(d_alpha_mask),
                                              static_cast<const uint64_t *>(d_rout),
                                              static_cast<const uint64_t *>(d_table), k0, k1, st);
}

int ddg_tt_lut_eval(int bw, uint64_t n, const void *d_xhat, const void *d_key, void *d_share, void *stream)
{
    DDG_TRY(check_bw(bw));
    DDG_CHECK(n == 0 || (d_xhat && d_key && d_share), DDG_ERR_ARG, "null pointer");
    TtLutLayout L = tt_lut_layout(bw, n);
    auto st = static_cast<cudaStream_t>(stream);
    auto *k = static_cast<const uint8_t *>(d_key);
    return bw == 32 ? tt_lut_eval<uint32_t>(L, static_cast<const uint32_t *>(d_xhat), k,
                                            static_cast<uint32_t *>(d_share), st)
                    : tt_lut_eval<uint64_t>(L, static_cast<const uint64_t *>(d_xhat), k,
                                            static_cast<uint64_t *>(d_share), st);
}

int ddg_lut_eval(int bw, uint64_t n, int party, const void *d_xhat, const void *d_table, const void *d_key,
                 void *d_share, void *stream)
{
    DDG_TRY(check_bw(bw));
    DDG_CHECK(party == 0 || party == 1, DDG_ERR_ARG, "party must be 0 or 1");
    DDG_CHECK(n == 0 || (d_xhat && d_table && d_key && d_share), DDG_ERR_ARG, "null pointer");
    LutLayout L = lut_layout(bw, n);
    auto st = static_cast<cudaStream_t>(stream);
    auto *k = static_cast<const uint8_t *>(d_key);
    return bw == 32 ? lut_eval<uint32_t>(L, party, static_cast<const uint32_t *>(d_xhat),
                                         static_cast<const uint32_t *>(d_table), k, static_cast<uint32_t *>(d_share), st)
                    : lut_eval<uint64_t>(L, party, static_cast<const uint64_t *>(d_xhat),
                                         static_cast<const uint64_t *>(d_table), k, static_cast<uint64_t *>(d_share), st);
}

int ddg_mul_share(int bw, int party, uint64_t n, int bcast, int rows, int cols, const void *d_xhat, const void *d_yhat,
                  const void *d_msx, const void *d_msy, const void *d_z, void *d_out, void *stream)
{
    DDG_TRY(check_bw(bw));
    DDG_CHECK(party == 0 || party == 1, DDG_ERR_ARG, "party must be 0 or 1");
    DDG_CHECK(bcast >= 0 && bcast <= 2 && rows > 0 && cols > 0, DDG_ERR_ARG, "bad broadcast shape");
    DDG_CHECK(n == 0 || (d_xhat && d_yhat && d_msx && d_msy && d_z && d_out), DDG_ERR_ARG, "null pointer");
    EwShape sh;
    sh.n = n, sh.R = rows, sh.C = cols;
    auto st = static_cast<cudaStream_t>(stream);
    if (bw == 32)
        return beaver_ew<uint32_t>(party, sh, Bcast(bcast), (const uint32_t *)d_xhat, (const uint32_t *)d_yhat,
                                   (const uint32_t *)d_msx, (const uint32_t *)d_msy, (const uint32_t *)d_z,
                                   (uint32_t *)d_out, st);
    return beaver_ew<uint64_t>(party, sh, Bcast(bcast), (const uint64_t *)d_xhat, (const uint64_t *)d_yhat,
                               (const uint64_t *)d_msx, (const uint64_t *)d_msy, (const uint64_t *)d_z,
                               (uint64_t *)d_out, st);
}

int ddg_matmul_share(int bw, int party, int batch, int M, int K, int N, const void *d_ahat, const void *d_bhat,
                     const void *d_msa, const void *d_msb, const void *d_z, void *d_out, void *stream)
{
    DDG_TRY(check_bw(bw));
    DDG_CHECK(party == 0 || party == 1, DDG_ERR_ARG, "party must be 0 or 1");
    DDG_CHECK(batch >= 0 && M >= 0 && K >= 0 && N >= 0, DDG_ERR_ARG, "negative size");
    DDG_CHECK(batch == 0 || M == 0 || N == 0 || (d_ahat && d_bhat && d_msa && d_msb && d_z && d_out), DDG_ERR_ARG,
              "null pointer");
    auto st = static_cast<cudaStream_t>(stream);
    return bw == 32 ? matmul_t<uint32_t>(party, batch, M, K, N, d_ahat, d_bhat, d_msa, d_msb, d_z, d_out, st)
                    : matmul_t<uint64_t>(party, batch, M, K, N, d_ahat, d_bhat, d_msa, d_msb, d_z, d_out, st);
}

int ddg_fc_share(int bw, int party, int M, int K, int N, const void *d_xhat, const void *d_w, const void *d_bias2s,
                 const void *d_c, void *d_out, void *stream)
{
    DDG_TRY(check_bw(bw));
    DDG_CHECK(party == 0 || party == 1, DDG_ERR_ARG, "party must be 0 or 1");
    DDG_CHECK(M >= 0 && K >= 0 && N >= 0, DDG_ERR_ARG, "negative size");
    DDG_CHECK(M == 0 || N == 0 || (d_c && d_out && (party == 1 || (d_xhat && d_w))), DDG_ERR_ARG, "null pointer");
    auto st = static_cast<cudaStream_t>(stream);
    return bw == 32 ? fc_t<uint32_t>(party, M, K, N, d_xhat, d_w, d_bias2s, d_c, d_out, st)
                    : fc_t<uint64_t>(party, M, K, N, d_xhat, d_w, d_bias2s, d_c, d_out, st);
}

int ddg_gemm_path(int path)
{
    DDG_CHECK(path >= 0 && path <= 5, DDG_ERR_ARG, "gemm path must be 0..5 (got %d)", path);
    set_gemm_path(path);
    return DDG_OK;
}

int ddg_gemm_status(void) { return ring_gemm_tc_error(true); }

}  // extern "C"
