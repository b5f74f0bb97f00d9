// extern "C" entry points of libddg.so (declared in include/ddg_fss.h).
#include <algorithm>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "aes_dev.cuh"
#include "channel.cuh"
#include "forward.cuh"
#include "gates.cuh"
#include "keystream.cuh"
#include "linear.cuh"
#include "ot.cuh"

using namespace ddg;

static int check_gate_args(int kind, int bw, int scale)
{
    DDG_CHECK(kind >= DDG_GATE_RELU && kind <= DDG_GATE_RELU_ARS_TTF, DDG_ERR_ARG, "gate kind %d out of range", kind);
    DDG_CHECK(bw == 32 || bw == 64, DDG_ERR_ARG, "bw must be 32 or 64 (got %d)", bw);
    DDG_CHECK(scale >= 1 && scale < bw - 1, DDG_ERR_ARG, "scale %d out of range for bw %d", scale, bw);
    DDG_CHECK(kind != DDG_GATE_LRS_SPLIT || scale >= 2, DDG_ERR_ARG, "split LRS needs scale >= 2 (got %d)", scale);
    DDG_CHECK(!gate_is_split3(kind) || scale + SPLIT3_MID < bw - 1, DDG_ERR_ARG,
              "three-part split needs scale + %d < bw - 1 (scale %d, bw %d)", SPLIT3_MID, scale, bw);
    DDG_CHECK(!gate_is_ot(kind) || ot_plan_cached(bw, scale).ok, DDG_ERR_ARG, "no OT-gate plan for bw %d, scale %d",
              bw, scale);
    DDG_CHECK(!gate_is_tt(kind) || tt_plan_of(kind, bw, scale).ok, DDG_ERR_ARG,
              "no truth-table plan for bw %d, scale %d", bw, scale);
    return DDG_OK;
}

extern "C" {

const char *ddg_last_error(void) { return ddg::last_error(); }

int ddg_version(void) { return 1; }

uint64_t ddg_gate_key_bytes(int kind, int bw, int scale, uint64_t n)
{
    if (check_gate_args(kind, bw, scale) != DDG_OK) return 0;
    return gate_layout(kind, bw, scale, n).bytes;
}

int ddg_gate_key_layout(int kind, int bw, int scale, uint64_t n, uint64_t *out)
{
    DDG_TRY(check_gate_args(kind, bw, scale));
    DDG_CHECK(out != nullptr, DDG_ERR_ARG, "null out");
    GateLayout L = gate_layout(kind, bw, scale, n);
    uint64_t v[22] = {L.H.root, L.H.cw, L.H.leaf, L.H.mu, L.Lo.root, L.Lo.cw, L.Lo.leaf, L.Lo.mu,
                      L.words, L.bytes, uint64_t(L.H.L), uint64_t(L.Lo.L), L.H.mu_eq, uint64_t(L.H.d),
                      uint64_t(L.hi_shift), uint64_t(L.Lo.d), L.Mi.root, L.Mi.cw, L.Mi.leaf, L.Mi.mu, L.Mi.mu_eq,
                      uint64_t(L.Mi.L)};
    for (int i = 0; i < 22; i++) out[i] = v[i];
    return DDG_OK;
}

int ddg_gate_keygen(int kind, int bw, int scale, uint64_t n, uint64_t seed, uint32_t op_id, const void *d_rin,
                    void *d_rout, void *d_key0, void *d_key1, void *stream)
{
    DDG_TRY(check_gate_args(kind, bw, scale));
    DDG_CHECK(n == 0 || (d_rin && d_rout && d_key0 && d_key1), DDG_ERR_ARG, "null pointer");
    return gate_keygen(gate_layout(kind, bw, scale, n), seed, op_id, d_rin, d_rout, d_key0, d_key1,
                       static_cast<cudaStream_t>(stream));
}

int ddg_gate_round1(int kind, int bw, int scale, uint64_t n, const void *d_xhat, const void *d_key,
                    uint32_t *d_bits_hi, uint32_t *d_bits_lo, void *stream)
{
    DDG_TRY(check_gate_args(kind, bw, scale));
    GateLayout L = gate_layout(kind, bw, scale, n);
    DDG_CHECK(n == 0 || (d_xhat && d_key), DDG_ERR_ARG, "null pointer");
    DDG_CHECK(n == 0 || !L.hi || d_bits_hi, DDG_ERR_ARG, "gate needs d_bits_hi");
    DDG_CHECK(n == 0 || !L.lo || d_bits_lo, DDG_ERR_ARG, "gate needs d_bits_lo");
    return gate_round1(L, d_xhat, d_key, d_bits_hi, d_bits_lo, static_cast<cudaStream_t>(stream));
}

int ddg_gate_round2(int kind, int bw, int scale, uint64_t n, int party, const void *d_xhat,
                    const uint32_t *d_hi_own, const uint32_t *d_hi_peer, const uint32_t *d_lo_own,
                    const uint32_t *d_lo_peer, const void *d_key, void *d_share, void *stream)
{
    DDG_TRY(check_gate_args(kind, bw, scale));
    DDG_CHECK(party == 0 || party == 1, DDG_ERR_ARG, "party must be 0 or 1");
    GateLayout L = gate_layout(kind, bw, scale, n);
    DDG_CHECK(n == 0 || (d_xhat && d_key && d_share), DDG_ERR_ARG, "null pointer");
    DDG_CHECK(n == 0 || !L.hi || (d_hi_own && d_hi_peer), DDG_ERR_ARG, "gate needs high-DCF bits");
    DDG_CHECK(n == 0 || !L.lo || (d_lo_own && d_lo_peer), DDG_ERR_ARG, "gate needs low-DCF bits");
    return gate_round2(L, party, d_xhat, d_hi_own, d_hi_peer, d_lo_own, d_lo_peer, d_key, d_share,
                       static_cast<cudaStream_t>(stream));
}

int ddg_ot_key_layout(int kind, int bw, int scale, uint64_t n, uint64_t *out)
{
    DDG_TRY(check_gate_args(kind, bw, scale));
    DDG_CHECK(gate_is_ot(kind) && out != nullptr, DDG_ERR_ARG, "OT gate kind and out[10] required");
    GateLayout L = gate_layout(kind, bw, scale, n);
    const OtPlan &P = ot_plan_cached(bw, scale);
    const uint64_t v[10] = {L.ot_ks, L.ot_recv, L.ot_c0, L.words, L.bytes, uint64_t(L.ot_gmax),
                            uint64_t(P.D), uint64_t(P.G0), uint64_t(P.levels), uint64_t(P.ncomb)};
    for (int i = 0; i < 10; i++) out[i] = v[i];
    return DDG_OK;
}

int ddg_gate_round1_arrays(int kind, int bw, int scale)
{
    if (check_gate_args(kind, bw, scale) != DDG_OK) return 0;
    GateLayout L = gate_layout(kind, bw, scale, 1);
    if (L.ot) return 3;
    if (L.tt) return kind == GATE_LRS_TT ? 1 : tt_mode_of(kind) == PLAN_TT_FULL ? 2 : 3;
    return (L.hi ? (L.mid ? 4 : (L.H.eq ? 2 : 1)) : 0) + (L.lo ? 1 : 0);
}

int ddg_gate_eval_pair(int kind, int bw, int scale, uint64_t n, const void *d_xhat, const void *d_key0,
                       const void *d_key1, uint32_t *d_bits0, uint32_t *d_bits1, void *d_share0, void *d_share1,
                       void *stream)
{
    DDG_TRY(check_gate_args(kind, bw, scale));
    DDG_CHECK(n == 0 || (d_xhat && d_key0 && d_key1 && d_share0 && d_share1), DDG_ERR_ARG, "null pointer");
    if (n == 0) return DDG_OK;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // the per-call openings and state come from the device's default pool:
    // keep freed blocks cached, as the forward does, so repeated calls do not
    // map and unmap memory each time
    int dev = 0;
    DDG_CUDA(cudaGetDevice(&dev));
    DDG_TRY(keep_pool_memory(dev));
    GateLayout L = gate_layout(kind, bw, scale, n);
    const uint64_t nw = (n + 31) / 32;
    const int nb = ddg_gate_round1_arrays(kind, bw, scale), nh = (L.ot || L.tt) ? 2 : nb - (L.lo ? 1 : 0);
    std::vector<void *> tmp;
    int err = DDG_OK;
    auto grab = [&](uint64_t bytes) -> void * {
        void *p = nullptr;
        if (err == DDG_OK && cudaMallocAsync(&p, bytes ? bytes : 16, st) != cudaSuccess) {
            set_last_error("cudaMallocAsync(%llu) failed", (unsigned long long)bytes);
            err = DDG_ERR_CUDA;
        }
        if (p) tmp.push_back(p);
        return p;
    };
    auto ok = [&](int s) {
        if (err == DDG_OK) err = s;
        return err == DDG_OK;
    };
    uint32_t *b[2] = {d_bits0 ? d_bits0 : static_cast<uint32_t *>(grab(4 * nw * nb)),
                      d_bits1 ? d_bits1 : static_cast<uint32_t *>(grab(4 * nw * nb))};
    const void *key[2] = {d_key0, d_key1};
    if (!L.ot && !L.tt) {
        for (int p = 0; p < 2 && err == DDG_OK; p++)
            ok(gate_round1(L, d_xhat, key[p], L.hi ? b[p] : nullptr, L.lo ? b[p] + nh * nw : nullptr, st));
    } else {
        const OtPlan &P = gate_digit_plan(L);
        const OtScratch sc = ot_scratch_bytes(L);
        const bool hi = P.nd[0] != 0;
        const int lo_arr = P.mode == PLAN_TT_FULL ? 1 : hi ? 2 : 0;  // index of the lo-compare array
        uint32_t *tab[2] = {}, *tri[2] = {};
        void *state[2];
        void *o[2][OT_MAX_LEVELS + 1] = {};
        for (int p = 0; p < 2; p++) {
            if (L.ot) tab[p] = static_cast<uint32_t *>(grab(sc.tables)), tri[p] = static_cast<uint32_t *>(grab(sc.tri));
            state[p] = grab(sc.state);
            for (int l = 1; l <= P.levels; l++) o[p][l] = grab(uint64_t(ot_open_bytes(L, l)) * n);
        }
        if (L.ot)
            for (int p = 0; p < 2 && err == DDG_OK; p++)
                ok(ot_garble(L, p, d_xhat, key[p], tab[p], state[p], tri[p], st));
        for (int l = 1; l <= P.levels + 1 && err == DDG_OK; l++)
            for (int p = 0; p < 2 && err == DDG_OK; p++) {
                const int q = 1 - p;
                const bool last = l == P.levels + 1;
                ok(ot_level(L, p, l, key[p], tab[q], o[p][l - 1], o[q][l - 1], state[p], tri[p], last ? nullptr : o[p][l],
                            last && hi ? b[p] : nullptr, last ? b[p] + lo_arr * nw : nullptr, st, d_xhat));
            }
    }
    void *sh[2] = {d_share0, d_share1};
    const bool has_hi = L.hi || L.ot || (L.tt && kind != GATE_LRS_TT);
    const bool has_lo = L.lo || L.ot || L.tt;
    const int lo_at = L.tt && kind == GATE_LRS_TT ? 0 : (L.tt && tt_mode_of(kind) == PLAN_TT_FULL) ? 1 : nh;
    for (int p = 0; p < 2 && err == DDG_OK; p++) {
        const int q = 1 - p;
        ok(gate_round2(L, p, d_xhat, has_hi ? b[p] : nullptr, has_hi ? b[q] : nullptr, has_lo ? b[p] + lo_at * nw : nullptr,
                       has_lo ? b[q] + lo_at * nw : nullptr, key[p], sh[p], st));
    }
    for (void *p : tmp) cudaFreeAsync(p, st);
    return err;
}

int ddg_tt_key_layout(int kind, int bw, int scale, uint64_t n, uint64_t *out)
{
    DDG_TRY(check_gate_args(kind, bw, scale));
    DDG_CHECK(gate_is_tt(kind) && out != nullptr, DDG_ERR_ARG, "truth-table gate kind and out[8] required");
    GateLayout L = gate_layout(kind, bw, scale, n);
    const OtPlan P = tt_plan_of(kind, bw, scale);
    const uint64_t v[8] = {L.tt_tables, uint64_t(L.tt_rows), L.tt_tri, uint64_t(L.tt_triw), L.words, L.bytes,
                           uint64_t(P.D), uint64_t(P.levels)};
    for (int i = 0; i < 8; i++) out[i] = v[i];
    return DDG_OK;
}

int ddg_relu_backend(int backend)
{
    DDG_CHECK(backend == DDG_RELU_DCF || backend == DDG_RELU_OT || backend == DDG_RELU_TT, DDG_ERR_ARG,
              "ReLU backend: %d, %d or %d (got %d)", DDG_RELU_DCF, DDG_RELU_OT, DDG_RELU_TT, backend);
    set_relu_backend(backend);
    return DDG_OK;
}

int ddg_aes_chain(uint64_t threads, int iters, uint32_t *d_out, void *stream)
{
    DDG_CHECK(threads > 0 && iters > 0 && d_out, DDG_ERR_ARG, "bad aes_chain arguments");
    return aes_chain(threads, iters, d_out, static_cast<cudaStream_t>(stream), 0);
}

int ddg_aes_chain_variant(uint64_t threads, int iters, int variant, uint32_t *d_out, void *stream)
{
    DDG_CHECK(threads > 0 && iters > 0 && d_out && (variant == 0 || variant == 2 || variant == 4), DDG_ERR_ARG,
              "bad aes_chain arguments");
    return aes_chain(threads, iters, d_out, static_cast<cudaStream_t>(stream), variant);
}

int ddg_relu_split(int parts)
{
    DDG_CHECK(parts == 2 || parts == 3, DDG_ERR_ARG, "ReLU split: 2 or 3 parts (got %d)", parts);
    set_relu_parts(parts);
    return DDG_OK;
}

int ddg_aes_tables(int tables)
{
    DDG_CHECK(tables == 2 || tables == 4, DDG_ERR_ARG, "AES engine: 2 or 4 staged tables (got %d)", tables);
    set_aes_tables(tables);
    return DDG_OK;
}

// ------------------------------------------------------------ parties

int ddg_party_create(ddg_party **out, int party, int bw, int scale, int device)
{
    DDG_CHECK(out, DDG_ERR_ARG, "null out");
    DDG_CHECK(party == 0 || party == 1, DDG_ERR_ARG, "party must be 0 or 1");
    DDG_TRY(check_gate_args(0, bw, scale));
    DDG_CUDA(cudaSetDevice(device));
    auto *h = new ddg_party();
    h->P.party = party, h->P.bw = bw, h->P.s = scale, h->P.device = device;
    cudaError_t e = cudaStreamCreateWithFlags(&h->P.stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
        delete h;
        set_last_error("cudaStreamCreate: %s", cudaGetErrorString(e));
        return DDG_ERR_CUDA;
    }
    *out = h;
    return DDG_OK;
}

int ddg_party_destroy(ddg_party *h)
{
    if (!h) return DDG_OK;
    cudaSetDevice(h->P.device);
    cudaStreamSynchronize(h->P.stream);
    h->P.w.release();
    if (h->P.copy_stream) cudaStreamSynchronize(h->P.copy_stream);
    h->P.release_inputs();
    h->P.timing.release();
    if (h->P.ref_event) cudaEventDestroy(h->P.ref_event);
    if (h->P.owns_chan) delete h->P.chan;
    cudaStreamDestroy(h->P.stream);
    delete h;
    return DDG_OK;
}

int ddg_party_set_weights(ddg_party *h, const int64_t *h_blob, uint64_t n)
{
    DDG_CHECK(h && h_blob, DDG_ERR_ARG, "null argument");
    return h->P.w.load(h_blob, n, h->P.bw, h->P.s, h->P.device);
}

int ddg_party_bind_keys(ddg_party *h, const void *d_keys, uint64_t bytes)
{
    DDG_CHECK(h && d_keys, DDG_ERR_ARG, "null argument");
    h->P.keys = static_cast<const uint8_t *>(d_keys);
    h->P.key_bytes = bytes;
    return DDG_OK;
}

int ddg_party_stream(ddg_party *h, void **stream)
{
    DDG_CHECK(h && stream, DDG_ERR_ARG, "null argument");
    *stream = h->P.stream;
    return DDG_OK;
}

int ddg_party_stats(ddg_party *h, uint64_t *out3)
{
    DDG_CHECK(h && out3, DDG_ERR_ARG, "null argument");
    out3[0] = h->P.stats.bytes_sent;
    out3[1] = h->P.stats.rounds;
    out3[2] = h->P.stats.key_bytes_used;
    return DDG_OK;
}

int ddg_party_connect_callback(ddg_party *h, const ddg_comm *comm)
{
    DDG_CHECK(h && comm && comm->exchange, DDG_ERR_ARG, "null party, transport or exchange callback");
    auto *c = new CallbackChannel();
    c->comm = *comm;
    c->timeout_ms = h->P.timeout_ms;
    if (h->P.owns_chan) delete h->P.chan;
    h->P.chan = c, h->P.owns_chan = true;
    return DDG_OK;
}

int ddg_pair_local(ddg_party *p0, ddg_party *p1)
{
    DDG_CHECK(p0 && p1 && p0 != p1, DDG_ERR_ARG, "need two distinct parties");
    DDG_CHECK(p0->P.party == 0 && p1->P.party == 1, DDG_ERR_ARG, "pair (party 0, party 1) in that order");
    DDG_CHECK(p0->P.bw == p1->P.bw && p0->P.s == p1->P.s, DDG_ERR_ARG, "parties disagree on bw/scale");
    if (p0->P.device != p1->P.device) {
        int can = 0;
        DDG_CUDA(cudaDeviceCanAccessPeer(&can, p1->P.device, p0->P.device));
        DDG_CHECK(can, DDG_ERR_ARG, "devices %d and %d have no peer access", p0->P.device, p1->P.device);
    }
    auto *c = new LocalPairChannel(p0->P.device, p1->P.device);
    p0->P.chan = c, p1->P.chan = c;
    p0->P.owns_chan = true, p1->P.owns_chan = false;
    return DDG_OK;
}

int ddg_nccl_unique_id(void *out128)
{
    DDG_CHECK(out128, DDG_ERR_ARG, "null out");
    return nccl_unique_id(out128);
}

int ddg_party_connect_nccl(ddg_party *h, const void *id128, int nranks, int rank, int peer_rank)
{
    DDG_CHECK(h && id128, DDG_ERR_ARG, "null argument");
    int st = DDG_OK;
    Channel *c = make_nccl_channel(id128, nranks, rank, peer_rank, h->P.device, &st);
    DDG_TRY(st);
    c->timeout_ms = h->P.timeout_ms;
    if (h->P.owns_chan) delete h->P.chan;
    h->P.chan = c, h->P.owns_chan = true;
    return DDG_OK;
}

int ddg_party_connect_ipc(ddg_party *h, const char *name, uint64_t slot_bytes)
{
    DDG_CHECK(h && name && *name && slot_bytes, DDG_ERR_ARG, "bad argument");
    DDG_CHECK(std::strlen(name) < 200 && !std::strchr(name, '/'), DDG_ERR_ARG, "bad shared-memory name");
    int st = DDG_OK;
    Channel *c = make_ipc_channel(name, h->P.party, h->P.device, slot_bytes, h->P.timeout_ms, &st);
    DDG_TRY(st);
    if (h->P.owns_chan) delete h->P.chan;
    h->P.chan = c, h->P.owns_chan = true;
    return DDG_OK;
}

int ddg_party_connect_ipc_push(ddg_party *h, const char *name, uint64_t slot_bytes)
{
    DDG_CHECK(h && name && *name && slot_bytes, DDG_ERR_ARG, "bad argument");
    DDG_CHECK(std::strlen(name) < 200 && !std::strchr(name, '/'), DDG_ERR_ARG, "bad shared-memory name");
    int st = DDG_OK;
    Channel *c = make_ipc_channel(name, h->P.party, h->P.device, slot_bytes, h->P.timeout_ms, &st, true);
    DDG_TRY(st);
    if (h->P.owns_chan) delete h->P.chan;
    h->P.chan = c, h->P.owns_chan = true;
    return DDG_OK;
}

uint64_t ddg_forward_max_exchange_bytes(int bw, int scale, int batch)
{
    if (check_gate_args(0, bw, scale) != DDG_OK || batch <= 0) return 0;
    // the widest opening of the graph: a (batch, 138, 376) ring tensor, or
    // with the OT backend the garbled tables of the ReLU over it
    const uint64_t n = uint64_t(batch) * NMAX * POOL;
    uint64_t per = uint64_t(bw / 8);
    if (relu_backend() == DDG_RELU_OT) {
        const uint64_t t = 4ull * uint64_t(ot_gmax(bw, scale));
        per = t > per ? t : per;
    }
    return n * per;
}

}  // extern "C"

// consumer of a probe exchange: one thread reads the peer's first word
static __global__ void k_probe_read(const uint32_t *peer, uint32_t *sink)
{
    if (threadIdx.x == 0 && blockIdx.x == 0) *sink += peer[0];
}

extern "C" {

int ddg_party_exchange_probe(ddg_party *h, uint64_t bytes, int iters, double *ms_per_exchange)
{
    DDG_CHECK(h && h->P.chan && iters > 0 && ms_per_exchange && bytes >= 4, DDG_ERR_ARG, "bad probe arguments");
    Party &P = h->P;
    DDG_CUDA(cudaSetDevice(P.device));
    cudaStream_t st = P.stream;
    void *send = nullptr, *recv = nullptr;
    uint32_t *sink = nullptr;
    DDG_CUDA(cudaMalloc(&send, bytes));
    DDG_CUDA(cudaMalloc(&recv, bytes));
    DDG_CUDA(cudaMalloc(&sink, 4));
    cudaEvent_t a = nullptr, b = nullptr;
    DDG_CUDA(cudaEventCreate(&a));
    DDG_CUDA(cudaEventCreate(&b));
    int err = DDG_OK;
    auto one = [&](int i) {
        if (err != DDG_OK) return;
        if (cudaMemsetAsync(send, i & 0xff, bytes, st) != cudaSuccess) err = DDG_ERR_CUDA;
        const void *peer = nullptr;
        if (err == DDG_OK) err = P.chan->exchange(P.party, st, send, bytes, recv, &peer);
        if (err == DDG_OK) k_probe_read<<<1, 32, 0, st>>>(static_cast<const uint32_t *>(peer), sink);
    };
    for (int i = 0; i < 3; i++) one(i);
    if (err == DDG_OK) err = P.chan->barrier(P.party, st);
    if (err == DDG_OK && cudaStreamSynchronize(st) != cudaSuccess) err = DDG_ERR_CUDA;
    if (err == DDG_OK && cudaEventRecord(a, st) != cudaSuccess) err = DDG_ERR_CUDA;
    for (int i = 0; i < iters; i++) one(i);
    if (err == DDG_OK && cudaEventRecord(b, st) != cudaSuccess) err = DDG_ERR_CUDA;
    if (err == DDG_OK) err = P.chan->barrier(P.party, st);
    if (err == DDG_OK && cudaStreamSynchronize(st) != cudaSuccess) err = DDG_ERR_CUDA;
    float ms = 0;
    if (err == DDG_OK) cudaEventElapsedTime(&ms, a, b);
    *ms_per_exchange = double(ms) / iters;
    cudaEventDestroy(a), cudaEventDestroy(b);
    cudaFree(send), cudaFree(recv), cudaFree(sink);
    if (err == DDG_ERR_CUDA) set_last_error("exchange probe: CUDA call failed");
    return err;
}

int ddg_party_set_timeout(ddg_party *h, int timeout_ms)
{
    DDG_CHECK(h && timeout_ms > 0, DDG_ERR_ARG, "bad timeout");
    h->P.timeout_ms = timeout_ms;
    if (h->P.chan) h->P.chan->timeout_ms = timeout_ms;
    return DDG_OK;
}

uint64_t ddg_forward_key_bytes(int bw, int scale, int batch)
{
    if (check_gate_args(0, bw, scale) != DDG_OK || batch <= 0) return 0;
    return forward_key_bytes(bw, scale, batch);
}

int ddg_forward_eval(ddg_party *h, int batch, const void *x_share, const void *adj_share, const void *mask_share,
                     const void *protein_share, int on_host, int64_t *h_out_raw, double *h_affinity)
{
    DDG_CHECK(h && batch > 0 && x_share && adj_share && mask_share && protein_share, DDG_ERR_ARG, "bad argument");
    DDG_CHECK(h->P.key_bytes >= forward_key_bytes(h->P.bw, h->P.s, batch), DDG_ERR_KEY,
              "bound key region (%llu B) smaller than one forward of batch %d",
              (unsigned long long)h->P.key_bytes, batch);
    return forward_eval(h->P, batch, x_share, adj_share, mask_share, protein_share, on_host != 0, h_out_raw,
                        h_affinity);
}

int ddg_forward_eval_pair(ddg_party *p0, ddg_party *p1, int batch, const void *const *in0, const void *const *in1,
                          int on_host, int64_t *h_out_raw, double *h_affinity)
{
    DDG_CHECK(p0 && p1 && in0 && in1, DDG_ERR_ARG, "null argument");
    int st1 = DDG_OK;
    std::string err1;
    std::thread t([&] {
        st1 = ddg_forward_eval(p1, batch, in1[0], in1[1], in1[2], in1[3], on_host, nullptr, nullptr);
        if (st1 != DDG_OK) err1 = ddg::last_error();
    });
    int st0 = ddg_forward_eval(p0, batch, in0[0], in0[1], in0[2], in0[3], on_host, h_out_raw, h_affinity);
    if (st0 != DDG_OK) {
        if (auto *lp = dynamic_cast<LocalPairChannel *>(p0->P.chan)) lp->fail();
    }
    t.join();
    if (st0 == DDG_OK && st1 != DDG_OK) {
        set_last_error("party 1: %s", err1.c_str());
        return st1;
    }
    return st0;
}

struct ddg_forward_graph {
    ddg_party *p0 = nullptr, *p1 = nullptr;
    int batch = 0;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    void *d_out = nullptr;          // party 0's revealed output, written by every replay
    uint64_t launches = 0;          // kernels of one replay
    uint64_t exchanges = 0;         // single-party graph: the party's channel exchanges in one replay
    // comparison-launch timing records captured into the graph, per party:
    // their events are the graph's (taken out of the party's pool), and every
    // replay re-records them
    std::vector<DcfTiming::Rec> recs[2];
};

// after a capture: the timing events the capture took from a party's pool
// belong to the graph from now on (the pool hands out pool[0..used) in order,
// and the pool was settled before the capture)
static void adopt_timing(Party &P, std::vector<DcfTiming::Rec> &dst)
{
    DcfTiming &t = P.timing;
    dst = t.recs;
    t.pool.erase(t.pool.begin(), t.pool.begin() + std::min(t.used, t.pool.size()));
    t.recs.clear(), t.used = 0;
}

int ddg_forward_graph_create(ddg_party *p0, ddg_party *p1, int batch, const void *const *in0, const void *const *in1,
                             ddg_forward_graph **out)
{
    return ddg_forward_graph_create_ex(p0, p1, batch, in0, in1, 0, out);
}

int ddg_forward_graph_create_ex(ddg_party *p0, ddg_party *p1, int batch, const void *const *in0,
                                const void *const *in1, int on_host, ddg_forward_graph **out)
{
    DDG_CHECK(p0 && p1 && in0 && in1 && out && batch > 0, DDG_ERR_ARG, "bad argument");
    *out = nullptr;
    DDG_CHECK(p0->P.device == p1->P.device && p0->P.chan && p0->P.chan == p1->P.chan &&
                  dynamic_cast<LocalPairChannel *>(p0->P.chan),
              DDG_ERR_STATE, "a forward graph needs an in-process pair on one device (ddg_pair_local)");
    for (ddg_party *p : {p0, p1})
        DDG_CHECK(p->P.keys && p->P.key_bytes >= forward_key_bytes(p->P.bw, p->P.s, batch), DDG_ERR_KEY,
                  "party %d: bound key region smaller than one forward of batch %d", p->P.party, batch);
    DDG_CUDA(cudaSetDevice(p0->P.device));
    for (ddg_party *p : {p0, p1}) {
        DDG_CHECK(!p->P.graph_recs, DDG_ERR_STATE, "party %d already has a forward graph", p->P.party);
        DDG_TRY(settle_timing(p->P));  // pending host-forward launches are read back first
        if (on_host) DDG_TRY(prepare_host_inputs(p->P, batch));  // no allocation inside the capture
    }
    auto *g = new ddg_forward_graph;
    g->p0 = p0, g->p1 = p1, g->batch = batch;
    auto fail = [&](int st) {
        if (g->d_out) cudaFree(g->d_out);
        delete g;
        return st;
    };
    if (cudaMalloc(&g->d_out, size_t(batch) * (p0->P.bw / 8)) != cudaSuccess) {
        set_last_error("cudaMalloc(forward graph output) failed");
        return fail(DDG_ERR_CUDA);
    }
    cudaEvent_t fork = nullptr, join = nullptr;
    cudaEventCreateWithFlags(&fork, cudaEventDisableTiming);
    cudaEventCreateWithFlags(&join, cudaEventDisableTiming);
    const uint64_t n0 = launch_count();
    int st = DDG_OK;
    cudaError_t ce = cudaStreamBeginCapture(p0->P.stream, cudaStreamCaptureModeRelaxed);
    if (ce != cudaSuccess) {
        set_last_error("cudaStreamBeginCapture: %s", cudaGetErrorString(ce));
        st = DDG_ERR_CUDA;
    }
    bool capturing = st == DDG_OK;
    if (st == DDG_OK) {
        // party 1's stream joins the capture through an event of party 0's stream
        if (cudaEventRecord(fork, p0->P.stream) != cudaSuccess ||
            cudaStreamWaitEvent(p1->P.stream, fork, 0) != cudaSuccess) {
            set_last_error("forward graph: fork of party 1's stream failed");
            st = DDG_ERR_CUDA;
        }
    }
    if (st == DDG_OK) {
        int st1 = DDG_OK;
        std::string err1;
        std::thread t([&] {
            st1 = forward_capture(p1->P, batch, in1[0], in1[1], in1[2], in1[3], nullptr, on_host != 0);
            if (st1 != DDG_OK) err1 = ddg::last_error();
        });
        st = forward_capture(p0->P, batch, in0[0], in0[1], in0[2], in0[3], g->d_out, on_host != 0);
        if (st != DDG_OK) {
            if (auto *lp = dynamic_cast<LocalPairChannel *>(p0->P.chan)) lp->fail();
        }
        t.join();
        if (st == DDG_OK && st1 != DDG_OK) {
            set_last_error("party 1: %s", err1.c_str());
            st = st1;
        }
        // party 1's last work joins back into party 0's stream before the capture ends
        if (cudaEventRecord(join, p1->P.stream) != cudaSuccess ||
            cudaStreamWaitEvent(p0->P.stream, join, 0) != cudaSuccess) {
            if (st == DDG_OK) set_last_error("forward graph: join of party 1's stream failed");
            if (st == DDG_OK) st = DDG_ERR_CUDA;
        }
    }
    if (capturing) {
        ce = cudaStreamEndCapture(p0->P.stream, &g->graph);
        if (st == DDG_OK && ce != cudaSuccess) {
            set_last_error("cudaStreamEndCapture: %s", cudaGetErrorString(ce));
            st = DDG_ERR_CUDA;
        }
    }
    g->launches = launch_count() - n0;
    if (st == DDG_OK) {
        ce = cudaGraphInstantiate(&g->exec, g->graph, 0);
        if (ce != cudaSuccess) {
            set_last_error("cudaGraphInstantiate: %s", cudaGetErrorString(ce));
            st = DDG_ERR_CUDA;
        }
    }
    cudaEventDestroy(fork);
    cudaEventDestroy(join);
    cudaGetLastError();  // a failed capture leaves its error here; the status carries it
    if (st != DDG_OK) {
        if (g->exec) cudaGraphExecDestroy(g->exec);
        if (g->graph) cudaGraphDestroy(g->graph);
        for (ddg_party *p : {p0, p1}) p->P.timing.recs.clear(), p->P.timing.used = 0;  // events back to the pool
        return fail(st);
    }
    ddg_party *ps[2] = {p0, p1};
    for (int i = 0; i < 2; i++) {
        Party &P = ps[i]->P;
        if (!P.timing.enabled) continue;
        adopt_timing(P, g->recs[i]);
        P.graph_recs = &g->recs[i];
        P.graph_fresh = false;
    }
    *out = g;
    return DDG_OK;
}

int ddg_party_graph_create(ddg_party *p, int batch, const void *const *in, int on_host, ddg_forward_graph **out)
{
    DDG_CHECK(p && in && out && batch > 0, DDG_ERR_ARG, "bad argument");
    *out = nullptr;
    DDG_CHECK(p->P.chan, DDG_ERR_STATE, "party %d has no channel", p->P.party);
    std::string why;
    DDG_CHECK(p->P.chan->replayable(why), DDG_ERR_STATE, "party %d: no single-party forward graph over %s",
              p->P.party, why.c_str());
    DDG_CHECK(p->P.keys && p->P.key_bytes >= forward_key_bytes(p->P.bw, p->P.s, batch), DDG_ERR_KEY,
              "party %d: bound key region smaller than one forward of batch %d", p->P.party, batch);
    DDG_CHECK(!p->P.graph_recs, DDG_ERR_STATE, "party %d already has a forward graph", p->P.party);
    DDG_CUDA(cudaSetDevice(p->P.device));
    DDG_TRY(settle_timing(p->P));
    if (on_host) DDG_TRY(prepare_host_inputs(p->P, batch));
    auto *g = new ddg_forward_graph;
    g->p0 = p, g->batch = batch;
    if (cudaMalloc(&g->d_out, size_t(batch) * (p->P.bw / 8)) != cudaSuccess) {
        delete g;
        set_last_error("cudaMalloc(forward graph output) failed");
        return DDG_ERR_CUDA;
    }
    const uint64_t n0 = launch_count(), r0 = p->P.chan->rounds[p->P.party];
    int st = DDG_OK;
    cudaError_t ce = cudaStreamBeginCapture(p->P.stream, cudaStreamCaptureModeRelaxed);
    if (ce != cudaSuccess) {
        set_last_error("cudaStreamBeginCapture: %s", cudaGetErrorString(ce));
        st = DDG_ERR_CUDA;
    }
    const bool capturing = st == DDG_OK;
    if (st == DDG_OK) st = forward_capture(p->P, batch, in[0], in[1], in[2], in[3], g->d_out, on_host != 0);
    if (capturing) {
        ce = cudaStreamEndCapture(p->P.stream, &g->graph);
        if (st == DDG_OK && ce != cudaSuccess) {
            set_last_error("cudaStreamEndCapture: %s", cudaGetErrorString(ce));
            st = DDG_ERR_CUDA;
        }
    }
    g->launches = launch_count() - n0;
    // the barrier's empty exchange is one of them (the channel does not count it as a round)
    g->exchanges = p->P.chan->rounds[p->P.party] - r0 + 1;
    if (st == DDG_OK) {
        ce = cudaGraphInstantiate(&g->exec, g->graph, 0);
        if (ce != cudaSuccess) {
            set_last_error("cudaGraphInstantiate: %s", cudaGetErrorString(ce));
            st = DDG_ERR_CUDA;
        }
    }
    cudaGetLastError();
    if (st != DDG_OK) {
        if (g->exec) cudaGraphExecDestroy(g->exec);
        if (g->graph) cudaGraphDestroy(g->graph);
        cudaFree(g->d_out);
        p->P.timing.recs.clear(), p->P.timing.used = 0;
        delete g;
        return st;
    }
    if (p->P.timing.enabled) {
        adopt_timing(p->P, g->recs[0]);
        p->P.graph_recs = &g->recs[0];
        p->P.graph_fresh = false;
    }
    *out = g;
    return DDG_OK;
}

int ddg_forward_graph_launch(ddg_forward_graph *g, int64_t *h_out_raw, double *h_affinity)
{
    DDG_CHECK(g && g->exec, DDG_ERR_ARG, "null forward graph");
    Party &P = g->p0->P;
    DDG_CUDA(cudaSetDevice(P.device));
    ddg_party *ps[2] = {g->p0, g->p1};
    const int np = g->p1 ? 2 : 1;
    for (int i = 0; i < np; i++) {
        // the timed launches of a replay are read against the party's reference
        // event: record it before the first replay of a timing session (both
        // parties share the device, so party 0's stream serves for both)
        Party &Q = ps[i]->P;
        if (!Q.timing.enabled || Q.graph_recs != &g->recs[i] || Q.ref_live) continue;
        if (!Q.ref_event) DDG_CUDA(cudaEventCreate(&Q.ref_event));
        DDG_CUDA(cudaEventRecord(Q.ref_event, P.stream));
        Q.ref_live = true;
    }
    DDG_CUDA(cudaGraphLaunch(g->exec, P.stream));
    add_launches(g->launches);
    if (!g->p1) P.chan->note_replay(P.party, g->exchanges);
    const int B = g->batch;
    std::vector<int64_t> v(B);
    std::vector<int32_t> h32(B);
    // the read-back stays on the party's stream (no legacy-stream synchronisation)
    const bool want = h_out_raw || h_affinity;
    if (want)
        DDG_CUDA(cudaMemcpyAsync(P.bw == 32 ? static_cast<void *>(h32.data()) : static_cast<void *>(v.data()),
                                 g->d_out, size_t(B) * (P.bw / 8), cudaMemcpyDeviceToHost, P.stream));
    cudaError_t ce = cudaStreamSynchronize(P.stream);
    DDG_CHECK(ce == cudaSuccess, DDG_ERR_CUDA, "forward graph: %s", cudaGetErrorString(ce));
    for (int i = 0; i < np; i++)
        if (ps[i]->P.graph_recs == &g->recs[i]) ps[i]->P.graph_fresh = true;
    DDG_TRY(ring_gemm_tc_check(P.stream));
    if (!g->p1) DDG_TRY(P.chan->status(P.party));  // the channel's device-side waits
    if (!want) return DDG_OK;
    if (P.bw == 32)
        for (int i = 0; i < B; i++) v[i] = h32[i];
    for (int i = 0; i < B; i++) {
        if (h_out_raw) h_out_raw[i] = v[i];
        // AFFINITY = int32(value) / 2^s (deepdtagen_inference.cu:594-606)
        if (h_affinity) h_affinity[i] = double(int32_t(uint32_t(uint64_t(v[i])))) / double(1ull << P.s);
    }
    return DDG_OK;
}

int ddg_forward_graph_enqueue(ddg_forward_graph *g)
{
    DDG_CHECK(g && g->exec, DDG_ERR_ARG, "null forward graph");
    Party &P = g->p0->P;
    DDG_CUDA(cudaSetDevice(P.device));
    ddg_party *ps[2] = {g->p0, g->p1};
    const int np = g->p1 ? 2 : 1;
    for (int i = 0; i < np; i++) {
        Party &Q = ps[i]->P;
        if (!Q.timing.enabled || Q.graph_recs != &g->recs[i] || Q.ref_live) continue;
        if (!Q.ref_event) DDG_CUDA(cudaEventCreate(&Q.ref_event));
        DDG_CUDA(cudaEventRecord(Q.ref_event, P.stream));
        Q.ref_live = true;
    }
    DDG_CUDA(cudaGraphLaunch(g->exec, P.stream));
    add_launches(g->launches);
    if (!g->p1) P.chan->note_replay(P.party, g->exchanges);
    // the timing read-out (after a sync) covers the last replay enqueued
    for (int i = 0; i < np; i++)
        if (ps[i]->P.graph_recs == &g->recs[i]) ps[i]->P.graph_fresh = true;
    return DDG_OK;
}

int ddg_forward_graph_sync(ddg_forward_graph *g, int64_t *h_out_raw, double *h_affinity)
{
    DDG_CHECK(g && g->exec, DDG_ERR_ARG, "null forward graph");
    Party &P = g->p0->P;
    DDG_CUDA(cudaSetDevice(P.device));
    const int B = g->batch;
    std::vector<int64_t> v(B);
    std::vector<int32_t> h32(B);
    const bool want = h_out_raw || h_affinity;
    if (want)
        DDG_CUDA(cudaMemcpyAsync(P.bw == 32 ? static_cast<void *>(h32.data()) : static_cast<void *>(v.data()),
                                 g->d_out, size_t(B) * (P.bw / 8), cudaMemcpyDeviceToHost, P.stream));
    const cudaError_t ce = cudaStreamSynchronize(P.stream);
    DDG_CHECK(ce == cudaSuccess, DDG_ERR_CUDA, "forward graph: %s", cudaGetErrorString(ce));
    DDG_TRY(ring_gemm_tc_check(P.stream));
    if (!g->p1) DDG_TRY(P.chan->status(P.party));
    if (!want) return DDG_OK;
    if (P.bw == 32)
        for (int i = 0; i < B; i++) v[i] = h32[i];
    for (int i = 0; i < B; i++) {
        if (h_out_raw) h_out_raw[i] = v[i];
        // AFFINITY = int32(value) / 2^s (deepdtagen_inference.cu:594-606)
        if (h_affinity) h_affinity[i] = double(int32_t(uint32_t(uint64_t(v[i])))) / double(1ull << P.s);
    }
    return DDG_OK;
}

int ddg_forward_graph_destroy(ddg_forward_graph *g)
{
    if (!g) return DDG_OK;
    cudaSetDevice(g->p0->P.device);
    cudaStreamSynchronize(g->p0->P.stream);
    if (g->exec) cudaGraphExecDestroy(g->exec);
    if (g->graph) cudaGraphDestroy(g->graph);
    if (g->d_out) cudaFree(g->d_out);
    ddg_party *ps[2] = {g->p0, g->p1};
    for (int i = 0; i < 2; i++) {
        if (!ps[i]) continue;
        Party &P = ps[i]->P;
        if (P.graph_recs == &g->recs[i]) P.graph_recs = nullptr, P.graph_fresh = false;
        for (const auto &r : g->recs[i]) cudaEventDestroy(r.a), cudaEventDestroy(r.b);
    }
    delete g;
    return DDG_OK;
}

// ---- pipelined forwards of an in-process pair on host inputs: two graphs of
// the forward, each reading its own device staging set; step k's host->device
// copies run on a copy stream while step k-1's graph runs

struct ddg_forward_pipeline {
    ddg_party *p0 = nullptr, *p1 = nullptr;
    int batch = 0;
    ddg_forward_graph *g[2] = {nullptr, nullptr};
    void *stage[2][2][4] = {};  // [set][party][input: x, adj, mask, protein]
    uint64_t bytes[4] = {};
    cudaStream_t copy = nullptr;
    cudaEvent_t staged[2] = {}, freed[2] = {}, done[2] = {};
    void *h_out[2] = {};        // pinned read-back of each set's revealed output
    bool pending[2] = {false, false};
    int64_t *user_raw[2] = {};
    double *user_aff[2] = {};
    uint64_t k = 0;             // steps submitted
};

static void pipeline_free(ddg_forward_pipeline *pp)
{
    cudaSetDevice(pp->p0->P.device);
    cudaStreamSynchronize(pp->p0->P.stream);
    if (pp->copy) cudaStreamSynchronize(pp->copy);
    for (int s = 0; s < 2; s++) {
        if (pp->g[s]) ddg_forward_graph_destroy(pp->g[s]);
        for (int q = 0; q < 2; q++)
            for (int i = 0; i < 4; i++)
                if (pp->stage[s][q][i]) cudaFree(pp->stage[s][q][i]);
        for (cudaEvent_t e : {pp->staged[s], pp->freed[s], pp->done[s]})
            if (e) cudaEventDestroy(e);
        if (pp->h_out[s]) cudaFreeHost(pp->h_out[s]);
    }
    if (pp->copy) cudaStreamDestroy(pp->copy);
    delete pp;
}

int ddg_forward_pipeline_create(ddg_party *p0, ddg_party *p1, int batch, ddg_forward_pipeline **out)
{
    DDG_CHECK(p0 && p1 && out && batch > 0, DDG_ERR_ARG, "bad argument");
    *out = nullptr;
    DDG_CHECK(!p0->P.timing.enabled && !p1->P.timing.enabled, DDG_ERR_STATE,
              "a forward pipeline needs DCF timing off on both parties (each of its graphs would own the events)");
    DDG_CUDA(cudaSetDevice(p0->P.device));
    auto *pp = new ddg_forward_pipeline;
    pp->p0 = p0, pp->p1 = p1, pp->batch = batch;
    const uint64_t es = p0->P.bw / 8, B = uint64_t(batch);
    const uint64_t n[4] = {B * NMAX * FEAT, B * NMAX * NMAX, B * NMAX * POOL, B * PROT};
    for (int i = 0; i < 4; i++) pp->bytes[i] = n[i] * es;
    int st = DDG_OK;
    auto cu = [&](cudaError_t e, const char *what) {
        if (e != cudaSuccess && st == DDG_OK) {
            set_last_error("forward pipeline: %s: %s", what, cudaGetErrorString(e));
            st = DDG_ERR_CUDA;
        }
    };
    for (int s = 0; s < 2 && st == DDG_OK; s++)
        for (int q = 0; q < 2; q++)
            for (int i = 0; i < 4; i++) cu(cudaMalloc(&pp->stage[s][q][i], pp->bytes[i]), "staging allocation");
    cu(cudaStreamCreateWithFlags(&pp->copy, cudaStreamNonBlocking), "copy stream");
    for (int s = 0; s < 2 && st == DDG_OK; s++) {
        cu(cudaEventCreateWithFlags(&pp->staged[s], cudaEventDisableTiming), "event");
        cu(cudaEventCreateWithFlags(&pp->freed[s], cudaEventDisableTiming), "event");
        cu(cudaEventCreateWithFlags(&pp->done[s], cudaEventDisableTiming), "event");
        cu(cudaHostAlloc(&pp->h_out[s], B * 8, cudaHostAllocDefault), "pinned read-back");
        if (st == DDG_OK) cu(cudaEventRecord(pp->freed[s], p0->P.stream), "event record");
    }
    for (int s = 0; s < 2 && st == DDG_OK; s++) {
        const void *in0[4] = {pp->stage[s][0][0], pp->stage[s][0][1], pp->stage[s][0][2], pp->stage[s][0][3]};
        const void *in1[4] = {pp->stage[s][1][0], pp->stage[s][1][1], pp->stage[s][1][2], pp->stage[s][1][3]};
        st = ddg_forward_graph_create_ex(p0, p1, batch, in0, in1, 0, &pp->g[s]);
    }
    if (st != DDG_OK) {
        const std::string err = ddg::last_error();
        pipeline_free(pp);
        set_last_error("%s", err.c_str());
        return st;
    }
    *out = pp;
    return DDG_OK;
}

// step k-2's outputs (staging set s): wait for its read-back and hand it over
static int pipeline_deliver(ddg_forward_pipeline *pp, int s)
{
    if (!pp->pending[s]) return DDG_OK;
    pp->pending[s] = false;
    const cudaError_t ce = cudaEventSynchronize(pp->done[s]);
    DDG_CHECK(ce == cudaSuccess, DDG_ERR_CUDA, "forward pipeline: %s", cudaGetErrorString(ce));
    const Party &P = pp->p0->P;
    for (int i = 0; i < pp->batch; i++) {
        const int64_t v = P.bw == 32 ? int64_t(static_cast<const int32_t *>(pp->h_out[s])[i])
                                     : static_cast<const int64_t *>(pp->h_out[s])[i];
        if (pp->user_raw[s]) pp->user_raw[s][i] = v;
        // AFFINITY = int32(value) / 2^s (deepdtagen_inference.cu:594-606)
        if (pp->user_aff[s]) pp->user_aff[s][i] = double(int32_t(uint32_t(uint64_t(v)))) / double(1ull << P.s);
    }
    return DDG_OK;
}

int ddg_forward_pipeline_submit(ddg_forward_pipeline *pp, const void *const *in0, const void *const *in1,
                                int64_t *h_out_raw, double *h_affinity)
{
    DDG_CHECK(pp && in0 && in1, DDG_ERR_ARG, "bad argument");
    const int s = int(pp->k & 1);
    Party &P = pp->p0->P;
    DDG_CUDA(cudaSetDevice(P.device));
    // keeps two steps in flight: the step that last used this staging set has read back
    DDG_TRY(pipeline_deliver(pp, s));
    // the copies into set s start once the graph that last read it is done
    DDG_CUDA(cudaStreamWaitEvent(pp->copy, pp->freed[s], 0));
    const void *const *in[2] = {in0, in1};
    for (int q = 0; q < 2; q++)
        for (int i = 0; i < 4; i++)
            DDG_CUDA(cudaMemcpyAsync(pp->stage[s][q][i], in[q][i], pp->bytes[i], cudaMemcpyHostToDevice, pp->copy));
    DDG_CUDA(cudaEventRecord(pp->staged[s], pp->copy));
    DDG_CUDA(cudaStreamWaitEvent(P.stream, pp->staged[s], 0));
    DDG_CUDA(cudaGraphLaunch(pp->g[s]->exec, P.stream));
    add_launches(pp->g[s]->launches);
    DDG_CUDA(cudaEventRecord(pp->freed[s], P.stream));
    DDG_CUDA(cudaMemcpyAsync(pp->h_out[s], pp->g[s]->d_out, size_t(pp->batch) * (P.bw / 8), cudaMemcpyDeviceToHost,
                             P.stream));
    DDG_CUDA(cudaEventRecord(pp->done[s], P.stream));
    pp->pending[s] = true, pp->user_raw[s] = h_out_raw, pp->user_aff[s] = h_affinity;
    pp->k++;
    return DDG_OK;
}

int ddg_forward_pipeline_wait(ddg_forward_pipeline *pp)
{
    DDG_CHECK(pp, DDG_ERR_ARG, "null pipeline");
    DDG_CUDA(cudaSetDevice(pp->p0->P.device));
    const int older = int(pp->k & 1);  // the slot of step k-2 (if pending) comes before step k-1's
    DDG_TRY(pipeline_deliver(pp, older));
    DDG_TRY(pipeline_deliver(pp, 1 - older));
    return ring_gemm_tc_check(pp->p0->P.stream);
}

int ddg_forward_pipeline_destroy(ddg_forward_pipeline *pp)
{
    if (!pp) return DDG_OK;
    pipeline_free(pp);
    return DDG_OK;
}

int ddg_party_enable_dcf_timing(ddg_party *h, int on)
{
    DDG_CHECK(h, DDG_ERR_ARG, "null party");
    return reset_timing(h->P, on != 0);
}

int ddg_party_dcf_timing(ddg_party *h, double *out6)
{
    DDG_CHECK(h && out6, DDG_ERR_ARG, "null argument");
    DDG_TRY(settle_timing(h->P));
    const DcfAcc &a = h->P.dcf;
    double v[6] = {a.launches, a.bytes, a.aes, a.sum_ms, a.union_ms, a.pair_union_ms};
    for (int i = 0; i < 6; i++) out6[i] = v[i];
    return DDG_OK;
}

uint64_t ddg_launch_count(void) { return launch_count(); }

int ddg_parties_dcf_union(ddg_party *const *parties, int n)
{
    DDG_CHECK(parties && n > 0, DDG_ERR_ARG, "bad argument");
    std::vector<Party *> ps(n);
    for (int i = 0; i < n; i++) {
        DDG_CHECK(parties[i], DDG_ERR_ARG, "null party");
        ps[i] = &parties[i]->P;
    }
    return parties_dcf_union(ps.data(), n);
}

// ------------------------------------------------------------ key chunks / streaming

struct ddg_keystream {
    KeyStream ks;
};

uint64_t ddg_key_chunk_bytes(int bw, int scale, int batch)
{
    if (check_gate_args(0, bw, scale) != DDG_OK || batch <= 0) return 0;
    return key_chunk_bytes(bw, scale, batch);
}

int ddg_key_checksum(const void *d_key, uint64_t bytes, uint64_t *out, void *stream)
{
    DDG_CHECK(d_key && out, DDG_ERR_ARG, "null argument");
    return key_checksum(d_key, bytes, out, static_cast<cudaStream_t>(stream));
}

int ddg_key_chunk_seal(void *d_chunk, int bw, int scale, int batch, uint64_t chunk_index, void *stream)
{
    DDG_TRY(check_gate_args(0, bw, scale));
    DDG_CHECK(d_chunk && batch > 0, DDG_ERR_ARG, "bad argument");
    return chunk_seal(d_chunk, bw, scale, batch, chunk_index, static_cast<cudaStream_t>(stream));
}

int ddg_key_chunk_verify(const void *d_chunk, int bw, int scale, int batch, uint64_t *chunk_index, void *stream)
{
    DDG_TRY(check_gate_args(0, bw, scale));
    DDG_CHECK(d_chunk && batch > 0, DDG_ERR_ARG, "bad argument");
    ChunkTrailer t;
    DDG_TRY(chunk_verify(d_chunk, bw, scale, batch, &t, static_cast<cudaStream_t>(stream)));
    if (chunk_index) *chunk_index = t.index;
    return DDG_OK;
}

int ddg_keystream_create(ddg_keystream **out, ddg_party *party, int batch)
{
    DDG_CHECK(out && party && batch > 0, DDG_ERR_ARG, "bad argument");
    auto *h = new ddg_keystream();
    int st = h->ks.init(&party->P, batch);
    if (st != DDG_OK) {
        delete h;
        return st;
    }
    *out = h;
    return DDG_OK;
}

int ddg_keystream_destroy(ddg_keystream *ks)
{
    delete ks;
    return DDG_OK;
}

int ddg_keystream_add_host_chunk(ddg_keystream *ks, const void *h_chunk)
{
    DDG_CHECK(ks && h_chunk, DDG_ERR_ARG, "null argument");
    DDG_CHECK(ks->ks.fd < 0, DDG_ERR_STATE, "key stream already reads a key file");
    ks->ks.host.push_back(h_chunk);
    return DDG_OK;
}

int ddg_keystream_open_file(ddg_keystream *ks, const char *path, int nchunks)
{
    DDG_CHECK(ks && path, DDG_ERR_ARG, "null argument");
    return ks->ks.open_file(path, nchunks);
}

int ddg_keystream_set_verify(ddg_keystream *ks, int on)
{
    DDG_CHECK(ks, DDG_ERR_ARG, "null argument");
    ks->ks.verify = on != 0;
    return DDG_OK;
}

int ddg_keystream_stats(ddg_keystream *ks, double *out5)
{
    DDG_CHECK(ks && out5, DDG_ERR_ARG, "null argument");
    double v[5] = {double(ks->ks.consumed_chunks), ks->ks.bytes_copied, ks->ks.copy_ms, ks->ks.read_ms,
                   ks->ks.wait_ms};
    for (int i = 0; i < 5; i++) out5[i] = v[i];
    return DDG_OK;
}

int ddg_forward_eval_streamed(ddg_keystream *ks, int batch, const void *x_share, const void *adj_share,
                              const void *mask_share, const void *protein_share, int on_host, int64_t *h_out_raw,
                              double *h_affinity)
{
    DDG_CHECK(ks && batch == ks->ks.B, DDG_ERR_ARG, "key stream was created for batch %d", ks ? ks->ks.B : 0);
    int st = ks->ks.begin_forward();
    if (st == DDG_OK)
        st = forward_eval(*ks->ks.P, batch, x_share, adj_share, mask_share, protein_share, on_host != 0, h_out_raw,
                          h_affinity);
    else if (auto *lp = dynamic_cast<LocalPairChannel *>(ks->ks.P->chan))
        lp->fail();
    return ks->ks.end_forward(st);
}

int ddg_forward_eval_pair_streamed(ddg_keystream *ks0, ddg_keystream *ks1, int batch, const void *const *in0,
                                   const void *const *in1, int on_host, int64_t *h_out_raw, double *h_affinity)
{
    DDG_CHECK(ks0 && ks1 && in0 && in1, DDG_ERR_ARG, "null argument");
    int st1 = DDG_OK;
    std::string err1;
    std::thread t([&] {
        st1 = ddg_forward_eval_streamed(ks1, batch, in1[0], in1[1], in1[2], in1[3], on_host, nullptr, nullptr);
        if (st1 != DDG_OK) err1 = ddg::last_error();
    });
    int st0 = ddg_forward_eval_streamed(ks0, batch, in0[0], in0[1], in0[2], in0[3], on_host, h_out_raw, h_affinity);
    if (st0 != DDG_OK) {
        if (auto *lp = dynamic_cast<LocalPairChannel *>(ks0->ks.P->chan)) lp->fail();
    }
    t.join();
    if (st0 == DDG_OK && st1 != DDG_OK) {
        set_last_error("party 1: %s", err1.c_str());
        return st1;
    }
    return st0;
}

int ddg_dealer_forward(int bw, int scale, int batch, uint64_t seed, const int64_t *h_weights, uint64_t n_weights,
                       int device, void *d_key0, void *d_key1, void *stream)
{
    DDG_TRY(check_gate_args(0, bw, scale));
    DDG_CHECK(batch > 0 && h_weights && d_key0 && d_key1, DDG_ERR_ARG, "bad argument");
    DDG_CUDA(cudaSetDevice(device));
    DevWeights w;
    DDG_TRY(w.load(h_weights, n_weights, bw, scale, device));
    int st = dealer_forward(bw, scale, batch, seed, w, static_cast<uint8_t *>(d_key0), static_cast<uint8_t *>(d_key1),
                            static_cast<cudaStream_t>(stream));
    cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
    w.release();
    return st;
}

}  // extern "C"
