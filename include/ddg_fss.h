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
/* Same functions as RELU / RELU_ARS with the (bw-1)-bit comparison split into a
 * DCF with equality output over the upper bw-1-scale bits and the scale-bit low
 * DCF: 1{x<a} = 1{U<A} ^ (1{U==A} & 1{V<B}).  20 instead of 25 / 31 AES-128 per
 * element at bw=32; round 1 emits three bit arrays (see ddg_gate_round1). */
#define DDG_GATE_RELU_SPLIT 4
#define DDG_GATE_RELU_ARS_SPLIT 5
/* Same function as LRS with the scale-bit carry comparison 1{x_low < r_low}
 * split into a DCF with equality output over its upper scale-s2 bits and a
 * plain DCF over its low s2 = min(7, scale-1) bits: carry = c1 + e1*c2 (the
 * two terms are exclusive).  2 instead of scale-6 AES-128 per element (2 vs 6
 * at scale 12) for 7 key words instead of 4; scale >= 2.  Round 1 emits three
 * bit arrays like the other split kinds. */
#define DDG_GATE_LRS_SPLIT 6
/* Same functions as RELU / RELU_ARS with the (bw-1)-bit comparison split in
 * three: the upper bits U1 and the 6 bits U2 above the low scale bits V, each
 * of U1, U2 a DCF with equality output, V the scale-bit DCF:
 * 1{x<a} = c1 + e1*(c2 + e2*cL).  15 instead of 20 AES-128 per element at
 * bw=32 for 40 / 80 key words instead of 16 / 32; scale + 6 < bw - 1.  Round 1
 * emits five bit arrays (see ddg_gate_round1). */
#define DDG_GATE_RELU_SPLIT3 7
#define DDG_GATE_RELU_ARS_SPLIT3 8
/* Same functions (and the same dealer words and round 2) as RELU_SPLIT /
 * RELU_ARS_SPLIT, with the comparison bits computed interactively instead of
 * from DCF keys, after the reference's LSS ReLU backend
 * (gpu_mpc/lss/lss_compare.cpp, lss_protocol.md sections 1-2, 5): the
 * (bw-1-scale)- and scale-bit parts are cut into radix-16 digits, each digit
 * garbled by one party as a 16-entry (lt, eq) table the other party reads at
 * its dealer-given index, and the digits are combined by a tree of Beaver AND
 * gates, one round per level (3 levels at bw=32, 4 at bw=64).  Each party
 * regenerates its own randomness from a per-gate AES key: about 4 AES-128
 * and 9 key bytes per element and party at bw=32 besides the 16 / 32 words,
 * against 15-20 AES and 160-290 DCF key bytes.  Round 1 is interactive: run
 * these kinds through the forward or ddg_gate_eval_pair; ddg_gate_round1
 * refuses them.  Round 2 is that of the SPLIT kinds (three bit arrays). */
#define DDG_GATE_RELU_OT 9
#define DDG_GATE_RELU_ARS_OT 10

/* Same functions (and the same dealer words and round 2) as RELU_SPLIT /
 * RELU_ARS_SPLIT / LRS, with the comparison bits from dealer truth tables:
 * every radix-2^w digit of the compared part of x_hat (public) indexes a
 * table of 2^w (lt, eq) bit pairs that the dealer XOR-shares between the
 * parties, and the digits are combined by the Beaver AND tree of the OT
 * kinds (2 levels at bw=32, 4 at bw=64; 1 for the truncation carry, two
 * 6-bit digits).  No AES and no table message online; the tables are key
 * bytes (40 per element and party for the bw=32 ReLU, 24 for the carry).
 * Round 2 is that of the SPLIT kinds (three bit arrays) or of LRS (one). */
#define DDG_GATE_RELU_TT 11
#define DDG_GATE_RELU_ARS_TT 12
#define DDG_GATE_LRS_TT 13
/* RELU_TT / RELU_ARS_TT with one more AND combining the two part roots into
 * the full (bw-1)-bit comparison: only the full compare bit and the lo
 * compare bit are opened, and round 2 is that of RELU / RELU_ARS (4 / 8
 * words instead of 16 / 32).  One more opening per gate, a quarter of the
 * dealer words; the forward's default ReLU kinds.  Round 2 reads two bit
 * arrays: [full compare | lo compare]. */
#define DDG_GATE_RELU_TTF 14
#define DDG_GATE_RELU_ARS_TTF 15

/* ReLU comparison backends of the forward (ddg_relu_backend) */
#define DDG_RELU_DCF 0
#define DDG_RELU_OT 1
#define DDG_RELU_TT 2

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

/* byte offsets of one party's key for n elements, written to out[22]:
 *   0 hi_root 1 hi_cw 2 hi_leaf 3 hi_mu 4 lo_root 5 lo_cw 6 lo_leaf 7 lo_mu
 *   8 words 9 total bytes 10 high-DCF tree levels 11 low-DCF tree levels
 *   12 hi_mu_eq (split kinds) 13 high-DCF domain bits 14 position of the
 *   high DCF's lowest input bit in x_hat 15 low-DCF domain bits
 *   16 mid_root 17 mid_cw 18 mid_leaf 19 mid_mu 20 mid_mu_eq 21 middle-DCF
 *   tree levels (three-part split kinds; 0 otherwise)
 * Each DCF is structure-of-arrays: root[n] 16 B, cw[levels][n] 16 B
 * (level-major), leaf[n] 16 B, mu[ceil(n/32)] u32 mask bits; then
 * nwords x n ring words.  Every array starts on a 256-byte boundary. */
int ddg_gate_key_layout(int kind, int bw, int scale, uint64_t n, uint64_t *out);
/* OT kinds: byte offsets of one party's key for n elements, written to out[10]:
 *   0 round keys of the party's AES key (44 u32) 1 receiver records (slots x n
 *   bytes: choice | pad_lt << 4 | pad_eq << 5) 2 party 0's triple c bits (n u32;
 *   zero in party 1's key) 3 words 4 total bytes 5 receiver slots 6 digits
 *   7 digits garbled by party 0 8 AND-tree levels 9 AND-tree combines */
int ddg_ot_key_layout(int kind, int bw, int scale, uint64_t n, uint64_t *out);
/* TT kinds: one party's key for n elements, written to out[8]:
 *   0 offset of the digit tables (rows x n u32, row-major: a digit's lt bits
 *   over its 2^w values, then its eq bits, packed from bit 0 of its first row)
 *   1 table rows 2 offset of the triple words (words x n u32: bits 5q..5q+4 =
 *   a, b, b', c, c' of combine q) 3 triple words 4 words 5 total bytes
 *   6 digits 7 AND-tree levels */
int ddg_tt_key_layout(int kind, int bw, int scale, uint64_t n, uint64_t *out);

/* dealer: both parties' keys for n elements with input masks d_rin (n ring
 * elements); writes the output masks d_rout.  Deterministic in (seed, op_id). */
int ddg_gate_keygen(int kind, int bw, int scale, uint64_t n, uint64_t seed, uint32_t op_id, const void *d_rin,
                    void *d_rout, void *d_key0, void *d_key1, void *stream);

/* round 1: d_bits_hi / d_bits_lo hold ceil(n/32) words each (a gate without
 * the high DCF (LRS) or the low DCF (RELU) leaves that array untouched); for
 * the split kinds d_bits_hi holds 2*ceil(n/32) words: the compare bits, then
 * the equality bits; for the three-part split kinds 4*ceil(n/32) words: then
 * the middle DCF's compare and equality bits.  Round 2 reads its own and the
 * peer's arrays in the same layout. */
int ddg_gate_round1(int kind, int bw, int scale, uint64_t n, const void *d_xhat, const void *d_key,
                    uint32_t *d_bits_hi, uint32_t *d_bits_lo, void *stream);

/* round 2: own and peer round-1 bits, party's key -> party's share */
int ddg_gate_round2(int kind, int bw, int scale, uint64_t n, int party, const void *d_xhat,
                    const uint32_t *d_hi_own, const uint32_t *d_hi_peer, const uint32_t *d_lo_own,
                    const uint32_t *d_lo_peer, const void *d_key, void *d_share, void *stream);

/* Both parties' evaluation of one gate on one device with no device
 * allocation (no counterpart in the reference, whose GPU code allocates per
 * op through gpuMalloc).  For callers that cannot call cudaMalloc -- code
 * inside a host framework that owns all device memory, code that must not hit
 * the implicit synchronisation of cudaMalloc/cudaFree mid-pipeline, fixed
 * memory budgets.  Same result as, per party, ddg_gate_round1 + the bit
 * exchange + ddg_gate_round2 followed by adding the two shares: d_yhat[n] =
 * f(x) + r_out (masked-public), from d_xhat and both parties' keys.  The
 * round-1 bits and round-2 shares live in one file-scope device array of
 * 4,325,376 bytes (4.125 MiB) held by every GPU that loads the library until exit; at most
 * DDG_NOALLOC_MAX_N elements per call, larger n is rejected with DDG_ERR_ARG.
 * Calls share that array: calls that overlap on the GPU race.  The first call
 * on a device looks up the array's address and uploads the AES tables; make
 * it before any stream capture. */
#define DDG_NOALLOC_MAX_N 262144
int ddg_gate_eval_pair_noalloc(int kind, int bw, int scale, uint64_t n, const void *d_xhat, const void *d_key0,
                               const void *d_key1, void *d_yhat, void *stream);

/* ------------------------------------------------------------------------
 * Parties and the full online forward.
 *
 * A ddg_party is one evaluator of the online phase: it replaces the
 * reference's DDGOrcaBatched backend object together with its GpuPeer
 * (gpu_mpc/ddg_orca_batched.h:87-141, ddg_orca_base.h:93-116) and the
 * resident evaluation loop of deepdtagen_inference.cu:422-607.  Its key region
 * is a device buffer holding one forward's keys in graph order (the reference
 * reads a key file into a GPU arena, patch:608-686); every op consumes the next
 * section, as the reference's keyBuf cursor does.
 * ---------------------------------------------------------------------- */
typedef struct ddg_party ddg_party;

int ddg_party_create(ddg_party **out, int party, int bw, int scale, int device);
int ddg_party_destroy(ddg_party *party);
/* public weights: the int64 weights.bin blob of reference/export_weights.py
 * (nine layers in forward order, W as (in,out) row-major then b, scale `scale`;
 * loadWeightsI64 at deepdtagen_inference.cu:121-181 shifts b to 2*scale) */
int ddg_party_set_weights(ddg_party *party, const int64_t *h_blob, uint64_t n_int64);
/* bind a device key region (not copied; must outlive the forwards) */
int ddg_party_bind_keys(ddg_party *party, const void *d_keys, uint64_t bytes);
/* the party's CUDA stream (all its kernels and copies run on it) */
int ddg_party_stream(ddg_party *party, void **stream);
/* last forward: out3 = {bytes sent, openings (rounds), key bytes consumed} */
int ddg_party_stats(ddg_party *party, uint64_t *out3);
/* channel between two parties of this process (same or different devices);
 * zero-copy openings when both live on one device */
int ddg_pair_local(ddg_party *p0, ddg_party *p1);
/* channel to the peer in another process: both ranks pass the same 128-byte
 * NCCL unique id (ddg_nccl_unique_id on one rank, broadcast by the caller) */
int ddg_nccl_unique_id(void *out128);
int ddg_party_connect_nccl(ddg_party *party, const void *unique_id128, int nranks, int rank, int peer_rank);
/* The two parties as two processes on one node (one GPU each): openings go
 * through CUDA IPC.  Each party exports four send slots of slot_bytes (at
 * least ddg_forward_max_exchange_bytes) and interprocess events; a POSIX
 * shared-memory block `name` (no slash, the same for both parties, unused on
 * the node; party 0 creates and removes it) carries the handles and the
 * generation counters.  A party reads the peer's slot in place over NVLink.
 * Waits on the peer are bounded by the party's timeout (ddg_party_set_timeout
 * before connecting, default 60 s) and end in DDG_ERR_PEER. */
int ddg_party_connect_ipc(ddg_party *party, const char *name, uint64_t slot_bytes);
/* The same two-process channel with the handoff on the device (push mode):
 * each party's kernels write its share into the peer's receive slot with
 * peer stores over NVLink and raise a flag in the peer's memory; the
 * consumer's one-thread kernel waits for that flag and the consumers read
 * their own HBM.  No host thread waits per opening, so a party's host thread
 * enqueues the whole forward ahead of the GPU.  Needs the two parties on
 * different GPUs of one node (refused otherwise: kernels that wait on each
 * other never share a GPU).  A device-side wait that exceeds the party's
 * timeout ends the forward with DDG_ERR_PEER.  Both parties must connect in
 * the same mode. */
int ddg_party_connect_ipc_push(ddg_party *party, const char *name, uint64_t slot_bytes);
/* Diagnostics: `iters` openings of `bytes` through the party's channel (a
 * memset as producer, a one-thread read of the peer's bytes as consumer),
 * both parties calling it together; ms per opening from CUDA events on the
 * party's stream. */
int ddg_party_exchange_probe(ddg_party *party, uint64_t bytes, int iters, double *ms_per_exchange);
/* the largest single exchange of one forward of `batch` samples, in bytes
 * (with the OT ReLU backend selected: its garbled tables) */
uint64_t ddg_forward_max_exchange_bytes(int bw, int scale, int batch);
/* give up (DDG_ERR_PEER) when the peer does not reach an opening in time */
int ddg_party_set_timeout(ddg_party *party, int timeout_ms);

/* key bytes of one forward of `batch` samples (per party) */
uint64_t ddg_forward_key_bytes(int bw, int scale, int batch);
/* One online forward of `batch` samples (replaces DeepDTAGenAffinity::_forward,
 * gpu_mpc/deepdtagen.h:183-222, with ddgSecureAdjNormEval in front,
 * secure_adj_norm.h:394-659).  Inputs: this party's additive shares of
 *   x (batch,138,94) at scale, adj (batch,138,138) raw 0/1 at scale 0,
 *   mask (batch,138,376) at scale, protein (batch,128) at scale (party 0 holds
 *   zeros, party 1 the public value; deepdtagen_inference.cu:426-432),
 * as device pointers, or host pointers when on_host != 0 (copied in).
 * Outputs (either may be NULL): h_out_raw[batch] = revealed output at scale
 * (signed), h_affinity[batch] = int32(value) / 2^scale, the reference's
 * AFFINITY[i] (deepdtagen_inference.cu:594-606). */
int ddg_forward_eval(ddg_party *party, int batch, const void *x_share, const void *adj_share, const void *mask_share,
                     const void *protein_share, int on_host, int64_t *h_out_raw, double *h_affinity);
/* both parties of an in-process pair, party 1 on an internal thread;
 * in0/in1 = {x, adj, mask, protein} share pointers of party 0 / party 1 */
int ddg_forward_eval_pair(ddg_party *p0, ddg_party *p1, int batch, const void *const *in0, const void *const *in1,
                          int on_host, int64_t *h_out_raw, double *h_affinity);
/* The same pair forward captured once into a CUDA graph and replayed (no
 * counterpart in the reference, whose forward is a host loop of per-layer
 * calls): ddg_forward_graph_create records both parties' launches, openings
 * and allocations of one forward of device-resident inputs in0/in1 (the
 * same pointers at every replay, the same key region: a replay re-reads the
 * keys, as the reference's benchmark loop rewinds keyBuf) without running
 * it; ddg_forward_graph_launch replays it on party 0's stream, waits for it
 * and returns the revealed output like ddg_forward_eval_pair.  Make one
 * ordinary ddg_forward_eval_pair of the pair first (one-time set-up of the
 * kernels and tables happens there, not inside a capture).  With DCF timing
 * enabled on the parties when the graph is created, the graph owns the
 * events of the timed launches it captured and every replay re-records them;
 * each ddg_parties_dcf_union / ddg_party_dcf_timing then adds the launches of
 * the last replay (once, if a replay ran since the previous read-out) to the
 * party's totals, beside those of its host-launched forwards.  One graph per
 * party at a time; destroy the graph before its parties. */
typedef struct ddg_forward_graph ddg_forward_graph;
int ddg_forward_graph_create(ddg_party *p0, ddg_party *p1, int batch, const void *const *in0, const void *const *in1,
                             ddg_forward_graph **out);
/* The same with on_host != 0: in0 / in1 are pinned host buffers (page-locked,
 * cudaHostAlloc or registered; the same addresses at every replay), and every
 * replay copies them host -> device on each party's copy stream, each input
 * ahead of its first use, as ddg_forward_eval_pair with on_host does; the
 * staging buffers are allocated before the capture. */
int ddg_forward_graph_create_ex(ddg_party *p0, ddg_party *p1, int batch, const void *const *in0,
                                const void *const *in1, int on_host, ddg_forward_graph **out);
/* One party's forward captured on its own stream, for a party whose peer is
 * another process (the split deployment, one party per GPU): the channel must
 * hand off on the device (ddg_party_connect_ipc_push; DDG_ERR_STATE for other
 * channels, and while another push-mode party lives on the same device in
 * this process).  The peer replays its own graph of the same forward, or runs
 * the same forward host-launched: the exchange sequences match either way.
 * ddg_forward_graph_launch replays it on the party's stream and returns the
 * revealed output like ddg_forward_eval; a device-side wait for the peer that
 * gave up is reported as DDG_ERR_PEER.  The rest as ddg_forward_graph_create_ex
 * (one host-launched ddg_forward_eval first; `in` device or, with on_host,
 * pinned host buffers). */
int ddg_party_graph_create(ddg_party *party, int batch, const void *const *in, int on_host,
                           ddg_forward_graph **out);
int ddg_forward_graph_launch(ddg_forward_graph *graph, int64_t *h_out_raw, double *h_affinity);
/* ddg_forward_graph_enqueue: one replay queued on the (first) party's stream
 * without waiting or reading back, so that replays follow each other with no
 * host round trip; ddg_forward_graph_sync waits for every replay enqueued and
 * returns the last one's output like ddg_forward_graph_launch (either output
 * may be NULL).  DCF timing read-outs come after a sync. */
int ddg_forward_graph_enqueue(ddg_forward_graph *graph);
int ddg_forward_graph_sync(ddg_forward_graph *graph, int64_t *h_out_raw, double *h_affinity);
int ddg_forward_graph_destroy(ddg_forward_graph *graph);
/* Pipelined forwards of an in-process pair on host-resident input shares (the
 * overlap of the reference's streaming loop, deepdtagen_inference.cu:608-826,
 * applied to the inputs): two CUDA graphs of the pair's forward, each reading
 * its own device staging set; ddg_forward_pipeline_submit copies one step's
 * input shares (in0 / in1: {x, adj, mask, protein}, pinned host buffers that
 * stay untouched until the step's outputs are delivered) into the next
 * staging set on a copy stream, which overlaps the previous step's forward,
 * then replays that set's graph and reads its revealed output back, all
 * without waiting.  Outputs reach h_out_raw / h_affinity (either may be NULL;
 * kept until then) when a later submit reuses the set (two steps in flight)
 * or at ddg_forward_pipeline_wait, which delivers every submitted step.
 * Create after one ordinary ddg_forward_eval_pair of the pair, with DCF timing
 * off on both parties; destroy before the parties.  The keys are re-read by
 * every step, as for ddg_forward_graph_create. */
typedef struct ddg_forward_pipeline ddg_forward_pipeline;
int ddg_forward_pipeline_create(ddg_party *p0, ddg_party *p1, int batch, ddg_forward_pipeline **out);
int ddg_forward_pipeline_submit(ddg_forward_pipeline *pipeline, const void *const *in0, const void *const *in1,
                                int64_t *h_out_raw, double *h_affinity);
int ddg_forward_pipeline_wait(ddg_forward_pipeline *pipeline);
int ddg_forward_pipeline_destroy(ddg_forward_pipeline *pipeline);
/* GPU dealer (replaces DDGOrcaKeygenBatched + ddgSecureAdjNormKeygen,
 * deepdtagen_inference.cu:283-342): both parties' keys of one forward, fresh
 * masks from `seed`, into d_key0 / d_key1 (ddg_forward_key_bytes each) */
int ddg_dealer_forward(int bw, int scale, int batch, uint64_t seed, const int64_t *h_weights, uint64_t n_weights,
                       int device, void *d_key0, void *d_key1, void *stream);

/* ------------------------------------------------------------------------
 * The caller's own transport, and the forward layer by layer.
 *
 * The reference's graph calls its backend one layer or op at a time, each
 * reading the next key section through the caller's keyBuf cursor and
 * opening through the backend's GpuPeer: ddgSecureAdjNorm{Keygen,Eval}
 * (gpu_mpc/secure_adj_norm.h:204-213, 394-405), GCNLayer::forward
 * (gcn_layer.h:99-103), MaskedMaxPoolLayer(B,Nmax,F)::_forward
 * (masked_maxpool_layer.h:23-47) and the Backend<T> ops matmul (4-arg),
 * mul, relu, truncateForward and output (ddg_orca_base.h:170-323,
 * ddg_orca.h:43-123).  The entry points below are that interface.  Each
 * runs the same layer function as the fused forward on a cursor the caller
 * holds; called in the graph's order (adjnorm, input x, GCN 0..2, input
 * mask, mul with truncation, maxpool, FC 3 (ReLU), FC 4 (floor), concat
 * protein, FC 5..7 (ReLU), FC 8, output) they read exactly the key region of
 * ddg_forward_key_bytes / ddg_dealer_forward and reveal exactly what
 * ddg_forward_eval reveals.  Evaluator calls use the party's keys, weights
 * and channel (any: ddg_pair_local, NCCL, IPC or ddg_party_connect_callback)
 * and return once the party's stream has drained; both parties make the same
 * calls in the same order.  Outputs go into caller-provided device buffers.
 * Gate kinds follow ddg_relu_backend (the TT kinds by default).
 * ---------------------------------------------------------------------- */

/* A transport for the openings supplied by the caller (replaces the
 * reference's GpuPeer::reconstructInPlace, gpu_mpc/utils/gpu_comms.h:291-302,
 * over its TCP SigmaPeer, sigma_comms.cpp:106-150).  For every opening the
 * library calls exchange(user, party, d_send, d_recv, bytes, stream) on the
 * thread that called it: d_send holds this party's `bytes` bytes once the
 * work already queued on `stream` has run; the callback must make the
 * peer's bytes of the same opening available in the device buffer d_recv to
 * work queued on `stream` after it returns (for example: synchronise the
 * stream, copy d_send to the host, send, receive, copy into d_recv).  Both
 * parties see the same sequence of openings.  A nonzero return fails the op
 * with DDG_ERR_PEER. */
typedef struct ddg_comm {
    void *user;
    int (*exchange)(void *user, int party, const void *d_send, void *d_recv, uint64_t bytes, void *stream);
} ddg_comm;
int ddg_party_connect_callback(ddg_party *party, const ddg_comm *comm);

/* Key cursor (the reference's u8* keyBuf, advanced by every op,
 * ddg_orca_base.h:41-50): offset = bytes of the bound key region consumed
 * (evaluators) or written (dealer) so far; ops = dealer ops so far (it seeds
 * each op's randomness; evaluators leave it alone).  A forward starts at
 * {0, 0}; a call that fails leaves the cursor where it was. */
typedef struct ddg_cursor {
    uint64_t offset;
    uint32_t ops;
    uint32_t reserved;
} ddg_cursor;

/* A masked-public wire held by one evaluator: d_value = x + r (n ring
 * elements on the device) and d_mask_share, the party's additive share of r
 * (a pointer into its key region), NULL until an op needs it, which then
 * reads it at the cursor and stores it here, as the reference's leaf
 * registry keeps one mask share per tensor (ddg_orca_base.h:72-80).  Pass
 * the same wire to every later op that uses the tensor.  For an output the
 * caller provides d_value with room for the stated size; the call sets n and
 * d_mask_share. */
typedef struct ddg_wire {
    void *d_value;
    uint64_t n;
    const void *d_mask_share;
} ddg_wire;
/* The dealer's view of a wire: the mask r (device) and both parties' shares
 * of it in their key regions (NULL until an op needs them). */
typedef struct ddg_mask_wire {
    void *d_mask;
    uint64_t n;
    const void *d_share0;
    const void *d_share1;
} ddg_mask_wire;

/* activation of ddg_op_fc_*: none (the output layer), ReLU(floor(y / 2^scale))
 * (dfc1, ffc1-3 and the GCN FCs), floor(y / 2^scale) (dfc2) */
#define DDG_ACT_NONE 0
#define DDG_ACT_RELU 1
#define DDG_ACT_TRUNC 2

/* evaluator, one party.  Sizes: adjacency (batch,138,138), features
 * (batch,138,94), GCN layer l output (batch,138,{188,282,376}[l]), max-pool
 * input (batch,138,376) and output (batch,376), FC layer l (rows x in) ->
 * (rows x out) with (in,out) of weights.bin layer l, concat (batch,128) ->
 * (batch,256). */
/* a secret-shared input leaf: own share + own mask share, opened
 * (registerLeaf + revealIfLeaf, ddg_orca_base.h:72-80) */
int ddg_op_input_eval(ddg_party *party, ddg_cursor *cur, uint64_t n, const void *d_share, ddg_wire *out);
/* ddgSecureAdjNormEval (secure_adj_norm.h:394-659): A_hat at scale from the
 * party's share of the raw 0/1 adjacency */
int ddg_adjnorm_eval(ddg_party *party, ddg_cursor *cur, int batch, const void *d_adj_share, ddg_wire *out_ahat);
/* GCNLayer::forward (gcn_layer.h:99-116), layer 0..2, aggregate first */
int ddg_gcn_layer_eval(ddg_party *party, ddg_cursor *cur, int layer, int batch, ddg_wire *ahat, ddg_wire *x,
                       ddg_wire *out);
/* Backend<T>::matmul 3-arg (ddg_orca_base.h:170-205, looped per sample in
 * sytorch/layers/layers.h:67-90): the Beaver product A_hat . x per sample,
 * ahat (batch,138,138), x (batch,138,k) -> (batch,138,k), no truncation */
int ddg_op_matmul_eval(ddg_party *party, ddg_cursor *cur, int batch, int k, ddg_wire *ahat, ddg_wire *x,
                       ddg_wire *out);
/* Backend<T>::mul (ddg_orca.h:43-63): Beaver product a*b, b broadcast per
 * bcast (0 none, 1 by row, 2 by column of a (., rows, cols) tensor); trunc != 0
 * adds the exact floor by 2^scale, valid for products in [0, 2^(bw-1)) */
int ddg_op_mul_eval(ddg_party *party, ddg_cursor *cur, int bcast, int rows, int cols, ddg_wire *a, ddg_wire *b,
                    int trunc, ddg_wire *out);
/* Backend<T>::relu / truncateForward (ddg_orca.h:83-123): one gate of any kind
 * (DDG_GATE_*), with its comparison rounds over the party's channel */
int ddg_op_gate_eval(ddg_party *party, ddg_cursor *cur, int kind, ddg_wire *x, ddg_wire *out);
/* MaskedMaxPoolLayer(batch,138,376)::_forward (masked_maxpool_layer.h:47-166)
 * on the masked features */
int ddg_maxpool_eval(ddg_party *party, ddg_cursor *cur, int batch, ddg_wire *masked, ddg_wire *out);
/* FC<T> through Backend<T>::matmul 4-arg (ddg_orca_base.h:208-271), then act */
int ddg_op_fc_eval(ddg_party *party, ddg_cursor *cur, int layer, int rows, int act, ddg_wire *x, ddg_wire *out);
/* GPUConcat (deepdtagen.h:45-100): [d2 | protein], the protein revealed from
 * the parties' shares (party 0 holds zeros) */
int ddg_op_concat_protein_eval(ddg_party *party, ddg_cursor *cur, int batch, ddg_wire *d2,
                               const void *d_protein_share, ddg_wire *out);
/* Backend<T>::output (ddg_orca_base.h:296-302): unmask, shift by scale; the
 * same outputs as ddg_forward_eval */
int ddg_op_output_eval(ddg_party *party, ddg_cursor *cur, int batch, ddg_wire *o, int64_t *h_out_raw,
                       double *h_affinity);

/* dealer (the keygen mirror, DDGOrcaBaseKeygen / ddgSecureAdjNormKeygen,
 * ddg_orca_base.h:326-525, secure_adj_norm.h:204-374): both parties' keys,
 * written at the cursor into the bound key regions; masks from `seed`.
 * Called in the graph's order it writes the keys of ddg_dealer_forward with
 * the same seed, byte for byte. */
typedef struct ddg_dealer ddg_dealer;
int ddg_dealer_create(ddg_dealer **out, int bw, int scale, int device, uint64_t seed, const int64_t *h_weights,
                      uint64_t n_weights);
int ddg_dealer_bind_keys(ddg_dealer *dealer, void *d_key0, void *d_key1, uint64_t bytes);
int ddg_dealer_stream(ddg_dealer *dealer, void **stream);
int ddg_dealer_destroy(ddg_dealer *dealer);
int ddg_op_input_keygen(ddg_dealer *dealer, ddg_cursor *cur, uint64_t n, ddg_mask_wire *out);
int ddg_adjnorm_keygen(ddg_dealer *dealer, ddg_cursor *cur, int batch, ddg_mask_wire *out_ahat);
int ddg_gcn_layer_keygen(ddg_dealer *dealer, ddg_cursor *cur, int layer, int batch, ddg_mask_wire *ahat,
                         ddg_mask_wire *x, ddg_mask_wire *out);
int ddg_op_matmul_keygen(ddg_dealer *dealer, ddg_cursor *cur, int batch, int k, ddg_mask_wire *ahat,
                         ddg_mask_wire *x, ddg_mask_wire *out);
int ddg_op_mul_keygen(ddg_dealer *dealer, ddg_cursor *cur, int bcast, int rows, int cols, ddg_mask_wire *a,
                      ddg_mask_wire *b, int trunc, ddg_mask_wire *out);
int ddg_op_gate_keygen(ddg_dealer *dealer, ddg_cursor *cur, int kind, ddg_mask_wire *x, ddg_mask_wire *out);
int ddg_maxpool_keygen(ddg_dealer *dealer, ddg_cursor *cur, int batch, ddg_mask_wire *masked, ddg_mask_wire *out);
int ddg_op_fc_keygen(ddg_dealer *dealer, ddg_cursor *cur, int layer, int rows, int act, ddg_mask_wire *x,
                     ddg_mask_wire *out);
int ddg_op_concat_protein_keygen(ddg_dealer *dealer, ddg_cursor *cur, int batch, ddg_mask_wire *d2,
                                 ddg_mask_wire *out);
int ddg_op_output_keygen(ddg_dealer *dealer, ddg_cursor *cur, ddg_mask_wire *o);

/* ------------------------------------------------------------------------
 * Key chunks and streaming (replaces the chunked key file and the streaming
 * evaluation of deepdtagen_inference.cu:344-416 and :608-826: 4 KiB-padded
 * chunks, 2 pinned + 2 device slots, a copy stream and events).
 *
 * A chunk is one forward's key region + zero padding + a 64-byte trailer
 * (magic "DDGKEY01", bw, scale, batch, chunk index, key bytes, checksum),
 * ddg_key_chunk_bytes long (a multiple of 4 KiB).  A key file is chunks
 * back to back; chunk k starts at k * ddg_key_chunk_bytes.
 * ---------------------------------------------------------------------- */
uint64_t ddg_key_chunk_bytes(int bw, int scale, int batch);
/* position-keyed 64-bit sum of the 8-byte words of a device buffer */
int ddg_key_checksum(const void *d_key, uint64_t bytes, uint64_t *out, void *stream);
/* write the trailer (with the checksum) into a device chunk whose first
 * ddg_forward_key_bytes hold a dealer's key region */
int ddg_key_chunk_seal(void *d_chunk, int bw, int scale, int batch, uint64_t chunk_index, void *stream);
/* DDG_ERR_KEY if the trailer is missing, for other parameters, or the checksum differs */
int ddg_key_chunk_verify(const void *d_chunk, int bw, int scale, int batch, uint64_t *chunk_index, void *stream);

/* A key stream feeds one party's forwards from chunks outside HBM: two
 * device slots; before forward k the copy of chunk k+1 is queued on the
 * stream's own copy stream, behind the forward that last used its slot, so it
 * runs during forward k.  Sources: pinned host chunks (used cyclically in the
 * order added) or a key file of nchunks chunks read cyclically by an I/O
 * thread (pread into two pinned staging buffers). */
typedef struct ddg_keystream ddg_keystream;
int ddg_keystream_create(ddg_keystream **out, ddg_party *party, int batch);
int ddg_keystream_destroy(ddg_keystream *ks);
int ddg_keystream_add_host_chunk(ddg_keystream *ks, const void *h_chunk);
int ddg_keystream_open_file(ddg_keystream *ks, const char *path, int nchunks);
/* verify every chunk's trailer and checksum on the GPU before use */
int ddg_keystream_set_verify(ddg_keystream *ks, int on);
/* out5 = {chunks consumed, bytes copied, summed H2D copy ms, summed file read ms, ms waited for the reader} */
int ddg_keystream_stats(ddg_keystream *ks, double *out5);
/* ddg_forward_eval / ddg_forward_eval_pair with the keys of the next chunk */
int ddg_forward_eval_streamed(ddg_keystream *ks, int batch, const void *x_share, const void *adj_share,
                              const void *mask_share, const void *protein_share, int on_host, int64_t *h_out_raw,
                              double *h_affinity);
int ddg_forward_eval_pair_streamed(ddg_keystream *ks0, ddg_keystream *ks1, int batch, const void *const *in0,
                                   const void *const *in1, int on_host, int64_t *h_out_raw, double *h_affinity);

/* ------------------------------------------------------------------------
 * Linear layers and the DPF look-up table, one party, no communication.
 * ---------------------------------------------------------------------- */

/* DPF LUT over an 8-bit domain (replaces gpuKeyGenLUT / gpuDpfLUT of
 * gpu_mpc/secure_adj_norm.h:270-279, 498-520).  Dealer: point alpha = low 8
 * bits of d_alpha_mask[i]; output mask d_rout[i] (shared into the keys).
 * Eval: party's share of table[(x_hat - alpha) mod 256] + r_out; d_table holds
 * 256 ring elements.  Either key pointer may be NULL (that party is skipped). */
uint64_t ddg_lut_key_bytes(int bw, uint64_t n);
int ddg_lut_keygen(int bw, uint64_t n, uint64_t seed, uint32_t op_id, const void *d_alpha_mask, const void *d_rout,
                   void *d_key0, void *d_key1, void *stream);
int ddg_lut_eval(int bw, uint64_t n, int party, const void *d_xhat, const void *d_table, const void *d_key,
                 void *d_share, void *stream);
/* Truth-table form of the same look-up (the truth-table backend's, used by
 * the forward with ddg_relu_backend(DDG_RELU_TT)): the dealer gives party p
 * a table T_p[256] per lookup with T_0[u] + T_1[u] = table[(u - alpha) mod
 * 256] + r_out, so party p's share of table[(x_hat - alpha) mod 256] + r_out
 * is T_p[x_hat mod 256] (one word read, no AES).  Key layout: 256 x n ring
 * words (entry-major), then n words of the party's share of r_out.  The
 * dealer needs the public table (256 ring words on the device). */
uint64_t ddg_tt_lut_key_bytes(int bw, uint64_t n);
int ddg_tt_lut_keygen(int bw, uint64_t n, uint64_t seed, uint32_t op_id, const void *d_alpha_mask, const void *d_rout,
                      const void *d_table, void *d_key0, void *d_key1, void *stream);
int ddg_tt_lut_eval(int bw, uint64_t n, const void *d_xhat, const void *d_key, void *d_share, void *stream);

/* Beaver elementwise product (replaces gpuMul of DDGOrca::mul,
 * gpu_mpc/ddg_orca.h:43-63, and of secure_adj_norm.h:609-651):
 *   out = [party==0] x_hat*y_hat - x_hat*[r_y] - [r_x]*y_hat + [r_x r_y + r_z]
 * bcast: 0 none, 1 y indexed by row (b*rows + i), 2 by column (b*cols + j)
 * of an element (b, i, j) of a (batch, rows, cols) tensor. */
int ddg_mul_share(int bw, int party, uint64_t n, int bcast, int rows, int cols, const void *d_xhat, const void *d_yhat,
                  const void *d_msx, const void *d_msy, const void *d_z, void *d_out, void *stream);

/* Beaver matrix product per sample, secret x secret (replaces gpuMatmul of
 * DDGOrcaBase::matmul 3-arg, gpu_mpc/ddg_orca_base.h:170-205, looped per
 * sample in sytorch/layers/layers.h:67-90): for b < batch,
 *   out[b] = A_hat[b] . ([party==0] B_hat[b] - [r_B][b]) - [r_A][b] . B_hat[b] + Z[b]
 * A (M x K), B (K x N), out (M x N), row-major, contiguous per sample. */
int ddg_matmul_share(int bw, int party, int batch, int M, int K, int N, const void *d_ahat, const void *d_bhat,
                     const void *d_msa, const void *d_msb, const void *d_z, void *d_out, void *stream);

/* Fully connected layer, secret x public weight (replaces FC<T> through
 * DDGOrcaBase::matmul 4-arg, gpu_mpc/ddg_orca_base.h:208-271):
 *   party 0: out = x_hat . W + bias2s + C0;  party 1: out = C1
 * W (K x N) ring, bias2s (N) = bias << scale (may be NULL), C = key words
 * [r_y - r_x . W]. */
int ddg_fc_share(int bw, int party, int M, int K, int N, const void *d_xhat, const void *d_w, const void *d_bias2s,
                 const void *d_c, void *d_out, void *stream);

/* Ring GEMM engine of ddg_matmul_share / ddg_fc_share and the forward.
 * path 0 (default): tcgen05 tensor cores, 8-bit limb products with int32
 * accumulation recombined modulo 2^bw; at bw 32 the operands are first split
 * into byte planes in the tensor cores' shared-memory layout by two streaming
 * kernels (scratch from the device's stream-ordered pool) and the GEMM moves
 * them with bulk copies through a 4-stage warp-specialised pipeline, a
 * 16-row tail tile covering ragged last rows (M % 128 <= 16); at bw 64
 * operand B MN-major in shared memory with 128 x 32 tiles; 1: CUDA cores
 * (integer multiply-add); 2: tensor cores with B K-major; 3: tensor cores
 * with 128 x 128 (bw 32) or 128 x 32 (bw 64) tiles; 4: tensor cores, 128 x 64
 * tiles, synchronous staging; 5: at bw 32 the in-kernel operand split (with
 * cp.async staging and 128 x 128 tiles where the operands allow it), ragged
 * last rows on the CUDA cores.  Reduction lengths beyond the limb sums' exactness bound
 * (K > 8192 at bw 32, K > 4096 at bw 64, counting both Beaver products) always
 * use the CUDA cores.  Process-wide setting.
 * ddg_gemm_status: DDG_OK, or DDG_ERR_CUDA when a tensor-core GEMM gave up on
 * one of its bounded internal waits since the last call (and clears the
 * flag); synchronises with the device. */
int ddg_gemm_path(int path);
int ddg_gemm_status(void);

/* Kernel accounting.  ddg_launch_count: kernels this library has launched
 * (process-wide).  DCF timing: when enabled on a party, every gate round-1
 * (DCF) launch is bracketed by CUDA events on the party's stream; out6 gets
 * {launches, algorithmic bytes (key bytes + input + output bits), AES blocks,
 * summed launch ms, ms of the union of this party's launches, ms of the union
 * of both parties' launches of an in-process pair (party 0, as of the last
 * ddg_parties_dcf_union)}, accumulated since enabling.  Enabling pre-creates
 * the events of about 28 forwards. */
uint64_t ddg_launch_count(void);
int ddg_party_enable_dcf_timing(ddg_party *party, int on);
int ddg_party_dcf_timing(ddg_party *party, double *out6);
/* several parties on one device (the two parties of an in-process pair, or
 * half-batch lanes): set parties[0]'s pair-union total (out6[5]) to the union
 * of all their DCF launch intervals since timing was enabled.  Launch events
 * are read back here and in ddg_party_dcf_timing, not at the end of each
 * forward. */
int ddg_parties_dcf_union(ddg_party *const *parties, int n);

/* Diagnostics: `threads` independent chains of `iters` fixed-key tree
 * hashes (one AES-128 each), one word per chain written to d_out.  Gives the
 * AES-blocks/s ceiling of the DCF kernels. */
int ddg_aes_chain(uint64_t threads, int iters, uint32_t *d_out, void *stream);
/* the same with the AES engine chosen: 0 = the one in use (ddg_aes_tables),
 * 2 or 4 = that many staged round tables */
int ddg_aes_chain_variant(uint64_t threads, int iters, int variant, uint32_t *d_out, void *stream);
/* AES engine of every FSS kernel (DCF evaluation and key generation, DPF
 * LUT, dealer PRG), process-wide: 4 (default) stages T0..T3 in 128 KiB of
 * shared memory, one 768-thread CTA per SM, 6 integer-pipe instructions per
 * round column; 2 stages T0 and T2 in 64 KiB, three 256-thread CTAs per SM,
 * 8 instructions per column (T1 ^ T3 as an 8-bit rotation).  Same outputs. */
int ddg_aes_tables(int tables);
/* Comparison split of the forward's ReLU gates under the DCF backend
 * (ddg_relu_backend(DDG_RELU_DCF)), process-wide: 3 (default,
 * DDG_GATE_RELU*_SPLIT3: fewest AES) or 2 (DDG_GATE_RELU*_SPLIT: smaller
 * keys).  It changes the key layout: the dealer
 * (ddg_dealer_forward, ddg_forward_key_bytes) and both evaluators must run
 * with the same setting. */
int ddg_relu_split(int parts);
/* Comparison backend of the forward's ReLU gates, process-wide:
 * DDG_RELU_TT (default; DDG_GATE_RELU*_TTF, and DDG_GATE_LRS_TT at the
 * truncation sites), DDG_RELU_OT (DDG_GATE_RELU*_OT) or DDG_RELU_DCF (the
 * split chosen by ddg_relu_split).  It changes the key layout like
 * ddg_relu_split. */
int ddg_relu_backend(int backend);

/* Test and measurement helper: both parties of one gate on one device, every
 * opening done in place (the peer's buffers read directly).  d_bits0/1
 * (optional, ddg_gate_round1_arrays() x ceil(n/32) words each) receive each
 * party's masked comparison-bit shares in the round-1 layout of the kind (for
 * the OT kinds that of the SPLIT kinds: [hi lt | hi eq | lo lt]); d_share0/1
 * each party's additive share of the masked output y + r_out. */
int ddg_gate_eval_pair(int kind, int bw, int scale, uint64_t n, const void *d_xhat, const void *d_key0,
                       const void *d_key1, uint32_t *d_bits0, uint32_t *d_bits1, void *d_share0, void *d_share1,
                       void *stream);
/* number of ceil(n/32)-word bit arrays of a kind's comparison bits (0 on bad arguments) */
int ddg_gate_round1_arrays(int kind, int bw, int scale);

#ifdef __cplusplus
}
#endif
#endif /* DDG_FSS_H */
