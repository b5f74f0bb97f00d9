/*
 * ddg_fss.h -- C ABI of the B200 two-party online inference library
 * (libddg.so) for the DeepDTAGen affinity branch.
 *
 * Every entry point takes plain pointers and sizes.  Device pointers are
 * prefixed d_, host pointers h_.  `stream` is a cudaStream_t passed as void*
 * (NULL = legacy default stream).  Every function returns a status code
 * (DDG_OK = 0); ddg_last_error() gives the message of the last failure on the
 * calling thread.  No entry point aborts the process.
 *
 * Ring: bw in {32, 64}; ring elements are uint32_t / uint64_t little-endian,
 * fixed-point scale `scale` (12 in the reference).
 */
#ifndef DDG_FSS_H
#define DDG_FSS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes (the reference aborts instead: checkCudaErrors / assert / exit) */
#define DDG_OK 0
#define DDG_ERR_ARG 1       /* bad argument (size, bit width, kind, null pointer) */
#define DDG_ERR_CUDA 2      /* CUDA runtime error */
#define DDG_ERR_KEY 3       /* key region exhausted, wrong size or layout mismatch */
#define DDG_ERR_PEER 4      /* the channel to the other party failed or timed out */
#define DDG_ERR_STATE 5     /* object used in the wrong state (no keys bound, no channel) */
#define DDG_ERR_OVERFLOW 6  /* input violates a documented range precondition */

/* gate kinds of the comparison-based nonlinear layers */
#define DDG_GATE_RELU 0      /* y = ReLU(x)                                   */
#define DDG_GATE_RELU_ARS 1  /* y = ReLU(floor(x / 2^scale))   (FC + ReLU)     */
#define DDG_GATE_ARS 2       /* y = floor(x / 2^scale), signed  (FC, no ReLU)  */
#define DDG_GATE_LRS 3       /* y = floor(x / 2^scale) for x in [0, 2^(bw-1))   */

const char *ddg_last_error(void);
int ddg_version(void);

/* ------------------------------------------------------------------------
 * Gate kernels, one party, no communication.
 *
 * Replaces the per-op key readers and FSS kernels behind
 *   DDGOrca::relu            gpu_mpc/ddg_orca.h:83-110 (readReluKey + gpuRelu),
 *   DDGOrcaBatched::relu     gpu_mpc/ddg_orca_batched.h:143-159,
 *   DDGOrca::truncateForward gpu_mpc/ddg_orca.h:112-123 (TrFloor),
 *   DDGOrcaBatched::truncateForward gpu_mpc/ddg_orca_batched.h:161-200.
 * x_hat = x + r_in (mod 2^bw) is the masked-public input; the output is the
 * party's additive share of y_hat = f(x) + r_out.  A gate is two rounds:
 *   round 1: DCF evaluation -> packed bits (1 bit/element for each DCF) that
 *            both parties exchange and XOR;
 *   round 2: local combination -> additive share that both parties exchange
 *            and add.
 * ---------------------------------------------------------------------- */

/* bytes of one party's key for n elements */
uint64_t ddg_gate_key_bytes(int kind, int bw, int scale, uint64_t n);

/* byte offsets of one party's key for n elements, written to out[12]:
 *   0 hi_root 1 hi_cw 2 hi_leaf 3 hi_mu 4 lo_root 5 lo_cw 6 lo_leaf 7 lo_mu
 *   8 words 9 total bytes 10 high-DCF tree levels 11 low-DCF tree levels
 * Each DCF is structure-of-arrays: root[n] 16 B, cw[levels][n] 16 B
 * (level-major), leaf[n] 16 B, mu[ceil(n/32)] u32 mask bits; then
 * nwords x n ring words.  Every array starts on a 256-byte boundary. */
int ddg_gate_key_layout(int kind, int bw, int scale, uint64_t n, uint64_t *out);

/* dealer: both parties' keys for n elements with input masks d_rin (n ring
 * elements); writes the output masks d_rout.  Deterministic in (seed, op_id). */
int ddg_gate_keygen(int kind, int bw, int scale, uint64_t n, uint64_t seed, uint32_t op_id, const void *d_rin,
                    void *d_rout, void *d_key0, void *d_key1, void *stream);

/* round 1: d_bits_hi / d_bits_lo hold ceil(n/32) words each (a gate without
 * the high DCF (LRS) or the low DCF (RELU) leaves that array untouched). */
int ddg_gate_round1(int kind, int bw, int scale, uint64_t n, const void *d_xhat, const void *d_key,
                    uint32_t *d_bits_hi, uint32_t *d_bits_lo, void *stream);

/* round 2: own and peer round-1 bits, party's key -> party's share */
int ddg_gate_round2(int kind, int bw, int scale, uint64_t n, int party, const void *d_xhat,
                    const uint32_t *d_hi_own, const uint32_t *d_hi_peer, const uint32_t *d_lo_own,
                    const uint32_t *d_lo_peer, const void *d_key, void *d_share, void *stream);

/* Diagnostics: `threads` independent chains of `iters` fixed-key tree
 * hashes (one AES-128 each), one word per chain written to d_out.  Gives the
 * AES-blocks/s ceiling of the DCF kernels. */
int ddg_aes_chain(uint64_t threads, int iters, uint32_t *d_out, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* DDG_FSS_H */
