// Per-layer and per-op entry points (extern "C", include/ddg_fss.h): the
// reference's layer interface -- ddgSecureAdjNorm{Keygen,Eval}
// (gpu_mpc/secure_adj_norm.h:204-213, 394-405), GCNLayer::forward
// (gcn_layer.h:99-103), MaskedMaxPoolLayer::_forward
// (masked_maxpool_layer.h:23-47) and the Backend<T> ops the graph calls
// one at a time (ddg_orca_base.h:170-323, ddg_orca.h:43-123) -- over a key
// cursor that every call advances, as the reference's u8* keyBuf is.
//
// Every call runs one layer function of graph.cuh on a fresh executor whose
// key cursor (and, for the dealer, op counter) starts where the caller's
// ddg_cursor says, so a forward driven call by call in the order of
// affinity_graph reads and writes exactly the key sections of the fused
// forward: the dealer's keys are byte for byte those of ddg_dealer_forward,
// and the revealed outputs those of ddg_forward_eval.  A call's temporaries
// come from the device's stream-ordered pool and are released before it
// returns; its output is copied into the caller's buffer.  Each call drains
// the party's (dealer's) stream before returning.
#include <string>

#include "aes_dev.cuh"
#include "graph.cuh"

using namespace ddg;

struct ddg_dealer {
    int bw = 32, s = 12, device = 0;
    uint64_t seed = 0;
    DevWeights w;
    uint8_t *k0 = nullptr, *k1 = nullptr;
    uint64_t key_bytes = 0;
    cudaStream_t st = nullptr;
};

namespace {

template <typename T>
Tn<T> tn_of(const ddg_wire *w)
{
    Tn<T> t;
    t.v = static_cast<T *>(w->d_value);
    t.n = w->n;
    t.ms0 = static_cast<const T *>(w->d_mask_share);
    return t;
}

template <typename T>
Tn<T> tn_of(const ddg_mask_wire *w)
{
    Tn<T> t;
    t.v = static_cast<T *>(w->d_mask);
    t.n = w->n;
    t.ms0 = static_cast<const T *>(w->d_share0);
    t.ms1 = static_cast<const T *>(w->d_share1);
    return t;
}

// an op may have taken an input's mask share from the keys: hand it back
template <typename T>
void back(ddg_wire *w, const Tn<T> &t)
{
    w->d_mask_share = t.ms0;
}
template <typename T>
void back(ddg_mask_wire *w, const Tn<T> &t)
{
    w->d_share0 = t.ms0, w->d_share1 = t.ms1;
}

template <typename T, class E>
void put(E &e, ddg_wire *out, const Tn<T> &t)
{
    if (e.err != DDG_OK) return;
    e.ok(cudaMemcpyAsync(out->d_value, t.v, t.n * sizeof(T), cudaMemcpyDeviceToDevice, e.st) == cudaSuccess
             ? DDG_OK : DDG_ERR_CUDA);
    out->n = t.n;
    out->d_mask_share = t.ms0;
}
template <typename T, class E>
void put(E &e, ddg_mask_wire *out, const Tn<T> &t)
{
    if (e.err != DDG_OK) return;
    e.ok(cudaMemcpyAsync(out->d_mask, t.v, t.n * sizeof(T), cudaMemcpyDeviceToDevice, e.st) == cudaSuccess
             ? DDG_OK : DDG_ERR_CUDA);
    out->n = t.n;
    out->d_share0 = t.ms0, out->d_share1 = t.ms1;
}

int check_wires(std::initializer_list<const void *> ptrs)
{
    for (const void *p : ptrs) DDG_CHECK(p, DDG_ERR_ARG, "null wire or wire buffer");
    return DDG_OK;
}

// one evaluator's call: body(EvalExec<T>&) runs layer functions and puts the output
template <typename T, class F>
int run_eval(ddg_party *h, ddg_cursor *cur, int batch, F &&body)
{
    Party &P = h->P;
    EvalExec<T> e;
    e.B = batch, e.bw = P.bw, e.s = P.s, e.st = P.stream, e.P = &P, e.p = P.party, e.off = cur->offset;
    body(e);
    if (e.err == DDG_OK) {
        // the peer may still read buffers this party allocated (zero-copy pairs): join before freeing
        e.err = P.chan->barrier(P.party, P.stream);
    } else if (auto *lp = dynamic_cast<LocalPairChannel *>(P.chan)) {
        lp->fail();  // the peer stops waiting for this party's openings
    }
    e.free_all();
    const cudaError_t ce = cudaStreamSynchronize(P.stream);
    if (e.err == DDG_OK && ce != cudaSuccess) {
        set_last_error("layer call: %s", cudaGetErrorString(ce));
        e.err = DDG_ERR_CUDA;
    }
    if (e.err == DDG_OK) e.err = ring_gemm_tc_check(P.stream);
    if (e.err == DDG_OK) e.err = P.chan->status(P.party);
    if (e.err != DDG_OK) {
        if (auto *lp = dynamic_cast<LocalPairChannel *>(P.chan)) lp->fail();
        return e.err;
    }
    cur->offset = e.off;
    return DDG_OK;
}

int eval_ready(ddg_party *h, ddg_cursor *cur, int batch)
{
    DDG_CHECK(h && cur, DDG_ERR_ARG, "null party or cursor");
    DDG_CHECK(batch > 0, DDG_ERR_ARG, "batch must be positive (got %d)", batch);
    Party &P = h->P;
    DDG_CHECK(P.chan, DDG_ERR_STATE, "party %d has no channel", P.party);
    DDG_CHECK(P.keys, DDG_ERR_STATE, "party %d has no keys bound", P.party);
    DDG_CHECK(P.w.table, DDG_ERR_STATE, "party %d has no weights", P.party);
    DDG_CUDA(cudaSetDevice(P.device));
    DDG_TRY(keep_pool_memory(P.device));
    return aes_device_init();
}

template <typename T, class F>
int run_keygen(ddg_dealer *d, ddg_cursor *cur, int batch, F &&body)
{
    DealerExec<T> e;
    e.B = batch, e.bw = d->bw, e.s = d->s, e.st = d->st, e.seed = d->seed, e.dk = dealer_key(d->seed);
    e.k0 = d->k0, e.k1 = d->k1, e.w = &d->w;
    e.off = cur->offset, e.op = 1 + cur->ops, e.limit = d->key_bytes;
    body(e);
    const cudaError_t ce = cudaStreamSynchronize(d->st);
    if (e.err == DDG_OK && ce != cudaSuccess) {
        set_last_error("layer keygen: %s", cudaGetErrorString(ce));
        e.err = DDG_ERR_CUDA;
    }
    if (e.err == DDG_OK) e.err = ring_gemm_tc_check(d->st);
    e.free_all();
    cudaStreamSynchronize(d->st);
    if (e.err != DDG_OK) return e.err;
    cur->offset = e.off;
    cur->ops = e.op - 1;
    return DDG_OK;
}

int keygen_ready(ddg_dealer *d, ddg_cursor *cur, int batch)
{
    DDG_CHECK(d && cur, DDG_ERR_ARG, "null dealer or cursor");
    DDG_CHECK(batch > 0, DDG_ERR_ARG, "batch must be positive (got %d)", batch);
    DDG_CHECK(d->k0 && d->k1, DDG_ERR_STATE, "dealer has no key regions bound");
    DDG_CUDA(cudaSetDevice(d->device));
    DDG_TRY(keep_pool_memory(d->device));
    return aes_device_init();
}

bool act_ok(int act) { return act == FC_ACT_NONE || act == FC_ACT_RELU || act == FC_ACT_TRUNC; }

int check_gate_kind(int kind, int bw, int s)
{
    DDG_CHECK(kind >= GATE_RELU && kind < GATE_KIND_END, DDG_ERR_ARG, "gate kind %d out of range", kind);
    DDG_CHECK(!gate_is_tt(kind) || tt_plan_of(kind, bw, s).ok, DDG_ERR_ARG, "no truth-table plan for bw %d scale %d",
              bw, s);
    DDG_CHECK(!gate_is_ot(kind) || ot_plan_cached(bw, s).ok, DDG_ERR_ARG, "no OT-gate plan for bw %d scale %d", bw,
              s);
    return DDG_OK;
}

}  // namespace

// ------------------------------------------------------------------ evaluators

#define DDG_DISPATCH_EVAL(h, cur, batch, BODY)                                                  \
    (h)->P.bw == 32 ? run_eval<uint32_t>(h, cur, batch, [&](EvalExec<uint32_t> &e) { BODY(uint32_t); }) \
                    : run_eval<uint64_t>(h, cur, batch, [&](EvalExec<uint64_t> &e) { BODY(uint64_t); })
#define DDG_DISPATCH_KEYGEN(d, cur, batch, BODY)                                                        \
    (d)->bw == 32 ? run_keygen<uint32_t>(d, cur, batch, [&](DealerExec<uint32_t> &e) { BODY(uint32_t); }) \
                  : run_keygen<uint64_t>(d, cur, batch, [&](DealerExec<uint64_t> &e) { BODY(uint64_t); })

extern "C" {

int ddg_op_input_eval(ddg_party *h, ddg_cursor *cur, uint64_t n, const void *d_share, ddg_wire *out)
{
    DDG_TRY(eval_ready(h, cur, 1));
    DDG_TRY(check_wires({d_share, out, out ? out->d_value : nullptr}));
#define BODY(T)                                     \
    e.in[IN_X] = static_cast<const T *>(d_share);   \
    Tn<T> y = e.reveal_input(IN_X, n);              \
    put<T>(e, out, y);
    return DDG_DISPATCH_EVAL(h, cur, 1, BODY);
#undef BODY
}

int ddg_adjnorm_eval(ddg_party *h, ddg_cursor *cur, int batch, const void *d_adj_share, ddg_wire *out)
{
    DDG_TRY(eval_ready(h, cur, batch));
    DDG_TRY(check_wires({d_adj_share, out, out ? out->d_value : nullptr}));
#define BODY(T)                                       \
    e.in[IN_ADJ] = static_cast<const T *>(d_adj_share); \
    Tn<T> y = adjnorm_layer<T>(e);                    \
    put<T>(e, out, y);
    return DDG_DISPATCH_EVAL(h, cur, batch, BODY);
#undef BODY
}

int ddg_gcn_layer_eval(ddg_party *h, ddg_cursor *cur, int layer, int batch, ddg_wire *ahat, ddg_wire *x,
                       ddg_wire *out)
{
    DDG_TRY(eval_ready(h, cur, batch));
    DDG_TRY(check_wires({ahat, x, out, out ? out->d_value : nullptr}));
    DDG_CHECK(layer >= 0 && layer < 3, DDG_ERR_ARG, "GCN layer %d out of range (0..2)", layer);
    DDG_CHECK(ahat->n == uint64_t(batch) * NMAX * NMAX && x->n == uint64_t(batch) * NMAX * LAYER_IN[layer],
              DDG_ERR_ARG, "GCN layer %d: wire sizes do not match batch %d", layer, batch);
#define BODY(T)                                   \
    Tn<T> A = tn_of<T>(ahat), H = tn_of<T>(x);     \
    Tn<T> y = gcn_layer<T>(e, A, H, layer);        \
    back<T>(ahat, A), back<T>(x, H);               \
    put<T>(e, out, y);
    return DDG_DISPATCH_EVAL(h, cur, batch, BODY);
#undef BODY
}

int ddg_op_matmul_eval(ddg_party *h, ddg_cursor *cur, int batch, int k, ddg_wire *ahat, ddg_wire *x, ddg_wire *out)
{
    DDG_TRY(eval_ready(h, cur, batch));
    DDG_TRY(check_wires({ahat, x, out, out ? out->d_value : nullptr}));
    DDG_CHECK(k > 0 && ahat->n == uint64_t(batch) * NMAX * NMAX && x->n == uint64_t(batch) * NMAX * k, DDG_ERR_ARG,
              "matmul: wires are not (%d, %d, %d) and (%d, %d, %d)", batch, NMAX, NMAX, batch, NMAX, k);
#define BODY(T)                                   \
    Tn<T> A = tn_of<T>(ahat), H = tn_of<T>(x);     \
    Tn<T> y = e.matmul(A, H, k);                   \
    back<T>(ahat, A), back<T>(x, H);               \
    put<T>(e, out, y);
    return DDG_DISPATCH_EVAL(h, cur, batch, BODY);
#undef BODY
}

int ddg_op_mul_eval(ddg_party *h, ddg_cursor *cur, int bcast, int rows, int cols, ddg_wire *a, ddg_wire *b,
                    int trunc, ddg_wire *out)
{
    DDG_TRY(eval_ready(h, cur, 1));
    DDG_TRY(check_wires({a, b, out, out ? out->d_value : nullptr}));
    DDG_CHECK(bcast >= BC_NONE && bcast <= BC_COL, DDG_ERR_ARG, "bcast %d out of range", bcast);
    DDG_CHECK(bcast == BC_NONE || (rows > 0 && cols > 0 && a->n % (uint64_t(rows) * cols) == 0), DDG_ERR_ARG,
              "broadcast shape (%d x %d) does not divide %llu elements", rows, cols, (unsigned long long)a->n);
#define BODY(T)                                                          \
    Tn<T> A = tn_of<T>(a), Bw = tn_of<T>(b);                             \
    EwShape sh;                                                          \
    sh.n = A.n, sh.R = rows, sh.C = cols;                                \
    Tn<T> y = e.mul(A, Bw, Bcast(bcast), sh);                            \
    if (trunc) y = e.gate(graph_kinds().lrs, y);                         \
    back<T>(a, A), back<T>(b, Bw);                                       \
    put<T>(e, out, y);
    return DDG_DISPATCH_EVAL(h, cur, 1, BODY);
#undef BODY
}

int ddg_op_gate_eval(ddg_party *h, ddg_cursor *cur, int kind, ddg_wire *x, ddg_wire *out)
{
    DDG_TRY(eval_ready(h, cur, 1));
    DDG_TRY(check_wires({x, out, out ? out->d_value : nullptr}));
    DDG_TRY(check_gate_kind(kind, h->P.bw, h->P.s));
#define BODY(T)                         \
    Tn<T> X = tn_of<T>(x);              \
    Tn<T> y = e.gate(kind, X);          \
    put<T>(e, out, y);
    return DDG_DISPATCH_EVAL(h, cur, 1, BODY);
#undef BODY
}

int ddg_maxpool_eval(ddg_party *h, ddg_cursor *cur, int batch, ddg_wire *masked, ddg_wire *out)
{
    DDG_TRY(eval_ready(h, cur, batch));
    DDG_TRY(check_wires({masked, out, out ? out->d_value : nullptr}));
    DDG_CHECK(masked->n == uint64_t(batch) * NMAX * POOL, DDG_ERR_ARG, "max-pool input is not (%d, %d, %d)", batch,
              NMAX, POOL);
#define BODY(T)                                 \
    Tn<T> y = maxpool_layer<T>(e, tn_of<T>(masked)); \
    put<T>(e, out, y);
    return DDG_DISPATCH_EVAL(h, cur, batch, BODY);
#undef BODY
}

int ddg_op_fc_eval(ddg_party *h, ddg_cursor *cur, int layer, int rows, int act, ddg_wire *x, ddg_wire *out)
{
    DDG_TRY(eval_ready(h, cur, 1));
    DDG_TRY(check_wires({x, out, out ? out->d_value : nullptr}));
    DDG_CHECK(layer >= 0 && layer < NLAYERS && rows > 0 && act_ok(act), DDG_ERR_ARG, "bad FC layer, rows or act");
    DDG_CHECK(x->n == uint64_t(rows) * LAYER_IN[layer], DDG_ERR_ARG, "FC layer %d input is not %d x %d", layer, rows,
              LAYER_IN[layer]);
#define BODY(T)                                         \
    Tn<T> X = tn_of<T>(x);                              \
    Tn<T> y = fc_layer<T>(e, X, layer, rows, act);      \
    put<T>(e, out, y);
    return DDG_DISPATCH_EVAL(h, cur, 1, BODY);
#undef BODY
}

int ddg_op_concat_protein_eval(ddg_party *h, ddg_cursor *cur, int batch, ddg_wire *d2, const void *d_protein_share,
                               ddg_wire *out)
{
    DDG_TRY(eval_ready(h, cur, batch));
    DDG_TRY(check_wires({d2, d_protein_share, out, out ? out->d_value : nullptr}));
    DDG_CHECK(d2->n == uint64_t(batch) * PROT, DDG_ERR_ARG, "concat input is not (%d, %d)", batch, PROT);
#define BODY(T)                                               \
    e.in[IN_PROT] = static_cast<const T *>(d_protein_share);  \
    Tn<T> y = concat_protein_layer<T>(e, tn_of<T>(d2));       \
    put<T>(e, out, y);
    return DDG_DISPATCH_EVAL(h, cur, batch, BODY);
#undef BODY
}

int ddg_op_output_eval(ddg_party *h, ddg_cursor *cur, int batch, ddg_wire *o, int64_t *h_out_raw, double *h_affinity)
{
    DDG_TRY(eval_ready(h, cur, batch));
    DDG_TRY(check_wires({o}));
    DDG_CHECK(o->n == uint64_t(batch), DDG_ERR_ARG, "output wire holds %llu values for batch %d",
              (unsigned long long)o->n, batch);
    std::vector<uint64_t> h64(batch);
    std::vector<uint32_t> h32(batch);
#define BODY(T)                                                                                                \
    e.output(tn_of<T>(o));                                                                                     \
    if (e.err == DDG_OK)                                                                                       \
        e.ok(cudaMemcpyAsync(sizeof(T) == 4 ? (void *)h32.data() : (void *)h64.data(), e.out, batch * sizeof(T), \
                             cudaMemcpyDeviceToHost, e.st) == cudaSuccess ? DDG_OK : DDG_ERR_CUDA);
    const int st = DDG_DISPATCH_EVAL(h, cur, batch, BODY);
#undef BODY
    if (st != DDG_OK) return st;
    for (int i = 0; i < batch; i++) {
        // the revealed value is signed at the ring width; AFFINITY = int32(value) / 2^s (deepdtagen_inference.cu:594-606)
        const int64_t v = h->P.bw == 32 ? int64_t(int32_t(h32[i])) : int64_t(h64[i]);
        if (h_out_raw) h_out_raw[i] = v;
        if (h_affinity) h_affinity[i] = double(int32_t(uint32_t(uint64_t(v)))) / double(1ull << h->P.s);
    }
    return DDG_OK;
}

// ------------------------------------------------------------------ dealer

int ddg_dealer_create(ddg_dealer **out, int bw, int scale, int device, uint64_t seed, const int64_t *h_weights,
                      uint64_t n_weights)
{
    DDG_CHECK(out && h_weights, DDG_ERR_ARG, "null argument");
    DDG_CHECK(bw == 32 || bw == 64, DDG_ERR_ARG, "bw must be 32 or 64 (got %d)", bw);
    DDG_CHECK(scale >= 1 && scale < bw - 1, DDG_ERR_ARG, "scale %d out of range for bw %d", scale, bw);
    *out = nullptr;
    DDG_CUDA(cudaSetDevice(device));
    auto *d = new ddg_dealer();
    d->bw = bw, d->s = scale, d->device = device, d->seed = seed;
    int st = d->w.load(h_weights, n_weights, bw, scale, device);
    if (st == DDG_OK && cudaStreamCreateWithFlags(&d->st, cudaStreamNonBlocking) != cudaSuccess) {
        set_last_error("cudaStreamCreate failed");
        st = DDG_ERR_CUDA;
    }
    if (st != DDG_OK) {
        d->w.release();
        delete d;
        return st;
    }
    *out = d;
    return DDG_OK;
}

int ddg_dealer_bind_keys(ddg_dealer *d, void *d_key0, void *d_key1, uint64_t bytes)
{
    DDG_CHECK(d && d_key0 && d_key1, DDG_ERR_ARG, "null argument");
    d->k0 = static_cast<uint8_t *>(d_key0), d->k1 = static_cast<uint8_t *>(d_key1), d->key_bytes = bytes;
    return DDG_OK;
}

int ddg_dealer_stream(ddg_dealer *d, void **stream)
{
    DDG_CHECK(d && stream, DDG_ERR_ARG, "null argument");
    *stream = d->st;
    return DDG_OK;
}

int ddg_dealer_destroy(ddg_dealer *d)
{
    if (!d) return DDG_OK;
    cudaSetDevice(d->device);
    if (d->st) cudaStreamSynchronize(d->st), cudaStreamDestroy(d->st);
    d->w.release();
    delete d;
    return DDG_OK;
}

int ddg_op_input_keygen(ddg_dealer *d, ddg_cursor *cur, uint64_t n, ddg_mask_wire *out)
{
    DDG_TRY(keygen_ready(d, cur, 1));
    DDG_TRY(check_wires({out, out ? out->d_mask : nullptr}));
#define BODY(T)                               \
    Tn<T> y = e.reveal_input(IN_X, n);        \
    put<T>(e, out, y);
    return DDG_DISPATCH_KEYGEN(d, cur, 1, BODY);
#undef BODY
}

int ddg_adjnorm_keygen(ddg_dealer *d, ddg_cursor *cur, int batch, ddg_mask_wire *out)
{
    DDG_TRY(keygen_ready(d, cur, batch));
    DDG_TRY(check_wires({out, out ? out->d_mask : nullptr}));
#define BODY(T)                               \
    Tn<T> y = adjnorm_layer<T>(e);            \
    put<T>(e, out, y);
    return DDG_DISPATCH_KEYGEN(d, cur, batch, BODY);
#undef BODY
}

int ddg_gcn_layer_keygen(ddg_dealer *d, ddg_cursor *cur, int layer, int batch, ddg_mask_wire *ahat,
                         ddg_mask_wire *x, ddg_mask_wire *out)
{
    DDG_TRY(keygen_ready(d, cur, batch));
    DDG_TRY(check_wires({ahat, x, out, out ? out->d_mask : nullptr}));
    DDG_CHECK(layer >= 0 && layer < 3, DDG_ERR_ARG, "GCN layer %d out of range (0..2)", layer);
    DDG_CHECK(ahat->n == uint64_t(batch) * NMAX * NMAX && x->n == uint64_t(batch) * NMAX * LAYER_IN[layer],
              DDG_ERR_ARG, "GCN layer %d: wire sizes do not match batch %d", layer, batch);
#define BODY(T)                                   \
    Tn<T> A = tn_of<T>(ahat), H = tn_of<T>(x);     \
    Tn<T> y = gcn_layer<T>(e, A, H, layer);        \
    back<T>(ahat, A), back<T>(x, H);               \
    put<T>(e, out, y);
    return DDG_DISPATCH_KEYGEN(d, cur, batch, BODY);
#undef BODY
}

int ddg_op_matmul_keygen(ddg_dealer *d, ddg_cursor *cur, int batch, int k, ddg_mask_wire *ahat, ddg_mask_wire *x,
                         ddg_mask_wire *out)
{
    DDG_TRY(keygen_ready(d, cur, batch));
    DDG_TRY(check_wires({ahat, x, out, out ? out->d_mask : nullptr}));
    DDG_CHECK(k > 0 && ahat->n == uint64_t(batch) * NMAX * NMAX && x->n == uint64_t(batch) * NMAX * k, DDG_ERR_ARG,
              "matmul: wires are not (%d, %d, %d) and (%d, %d, %d)", batch, NMAX, NMAX, batch, NMAX, k);
#define BODY(T)                                   \
    Tn<T> A = tn_of<T>(ahat), H = tn_of<T>(x);     \
    Tn<T> y = e.matmul(A, H, k);                   \
    back<T>(ahat, A), back<T>(x, H);               \
    put<T>(e, out, y);
    return DDG_DISPATCH_KEYGEN(d, cur, batch, BODY);
#undef BODY
}

int ddg_op_mul_keygen(ddg_dealer *d, ddg_cursor *cur, int bcast, int rows, int cols, ddg_mask_wire *a,
                      ddg_mask_wire *b, int trunc, ddg_mask_wire *out)
{
    DDG_TRY(keygen_ready(d, cur, 1));
    DDG_TRY(check_wires({a, b, out, out ? out->d_mask : nullptr}));
    DDG_CHECK(bcast >= BC_NONE && bcast <= BC_COL, DDG_ERR_ARG, "bcast %d out of range", bcast);
    DDG_CHECK(bcast == BC_NONE || (rows > 0 && cols > 0 && a->n % (uint64_t(rows) * cols) == 0), DDG_ERR_ARG,
              "broadcast shape (%d x %d) does not divide %llu elements", rows, cols, (unsigned long long)a->n);
#define BODY(T)                                                          \
    Tn<T> A = tn_of<T>(a), Bw = tn_of<T>(b);                             \
    EwShape sh;                                                          \
    sh.n = A.n, sh.R = rows, sh.C = cols;                                \
    Tn<T> y = e.mul(A, Bw, Bcast(bcast), sh);                            \
    if (trunc) y = e.gate(graph_kinds().lrs, y);                         \
    back<T>(a, A), back<T>(b, Bw);                                       \
    put<T>(e, out, y);
    return DDG_DISPATCH_KEYGEN(d, cur, 1, BODY);
#undef BODY
}

int ddg_op_gate_keygen(ddg_dealer *d, ddg_cursor *cur, int kind, ddg_mask_wire *x, ddg_mask_wire *out)
{
    DDG_TRY(keygen_ready(d, cur, 1));
    DDG_TRY(check_wires({x, out, out ? out->d_mask : nullptr}));
    DDG_TRY(check_gate_kind(kind, d->bw, d->s));
#define BODY(T)                         \
    Tn<T> y = e.gate(kind, tn_of<T>(x)); \
    put<T>(e, out, y);
    return DDG_DISPATCH_KEYGEN(d, cur, 1, BODY);
#undef BODY
}

int ddg_maxpool_keygen(ddg_dealer *d, ddg_cursor *cur, int batch, ddg_mask_wire *masked, ddg_mask_wire *out)
{
    DDG_TRY(keygen_ready(d, cur, batch));
    DDG_TRY(check_wires({masked, out, out ? out->d_mask : nullptr}));
    DDG_CHECK(masked->n == uint64_t(batch) * NMAX * POOL, DDG_ERR_ARG, "max-pool input is not (%d, %d, %d)", batch,
              NMAX, POOL);
#define BODY(T)                                      \
    Tn<T> y = maxpool_layer<T>(e, tn_of<T>(masked)); \
    put<T>(e, out, y);
    return DDG_DISPATCH_KEYGEN(d, cur, batch, BODY);
#undef BODY
}

int ddg_op_fc_keygen(ddg_dealer *d, ddg_cursor *cur, int layer, int rows, int act, ddg_mask_wire *x,
                     ddg_mask_wire *out)
{
    DDG_TRY(keygen_ready(d, cur, 1));
    DDG_TRY(check_wires({x, out, out ? out->d_mask : nullptr}));
    DDG_CHECK(layer >= 0 && layer < NLAYERS && rows > 0 && act_ok(act), DDG_ERR_ARG, "bad FC layer, rows or act");
    DDG_CHECK(x->n == uint64_t(rows) * LAYER_IN[layer], DDG_ERR_ARG, "FC layer %d input is not %d x %d", layer, rows,
              LAYER_IN[layer]);
#define BODY(T)                                         \
    Tn<T> X = tn_of<T>(x);                              \
    Tn<T> y = fc_layer<T>(e, X, layer, rows, act);      \
    put<T>(e, out, y);
    return DDG_DISPATCH_KEYGEN(d, cur, 1, BODY);
#undef BODY
}

int ddg_op_concat_protein_keygen(ddg_dealer *d, ddg_cursor *cur, int batch, ddg_mask_wire *d2, ddg_mask_wire *out)
{
    DDG_TRY(keygen_ready(d, cur, batch));
    DDG_TRY(check_wires({d2, out, out ? out->d_mask : nullptr}));
    DDG_CHECK(d2->n == uint64_t(batch) * PROT, DDG_ERR_ARG, "concat input is not (%d, %d)", batch, PROT);
#define BODY(T)                                               \
    Tn<T> y = concat_protein_layer<T>(e, tn_of<T>(d2));       \
    put<T>(e, out, y);
    return DDG_DISPATCH_KEYGEN(d, cur, batch, BODY);
#undef BODY
}

int ddg_op_output_keygen(ddg_dealer *d, ddg_cursor *cur, ddg_mask_wire *o)
{
    DDG_TRY(keygen_ready(d, cur, 1));
    DDG_TRY(check_wires({o, o ? o->d_mask : nullptr}));
#define BODY(T) e.output(tn_of<T>(o));
    return DDG_DISPATCH_KEYGEN(d, cur, 1, BODY);
#undef BODY
}

}  // extern "C"
