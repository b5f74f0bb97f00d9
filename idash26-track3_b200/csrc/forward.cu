// Public weights, party state, the comparison-backend settings and the
// whole-forward entry points (dealer, one party's evaluation, its CUDA-graph
// capture, launch timing).  The graph itself and its executors are in
// graph.cuh.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <vector>

#include "graph.cuh"

namespace ddg {

// ------------------------------------------------------------------ weights

int DevWeights::load(const int64_t *h_blob, uint64_t n, int bw_, int s_, int device_)
{
    DDG_CHECK(n == weights_elems(), DDG_ERR_ARG, "weights blob has %llu int64 values, expected %llu",
              (unsigned long long)n, (unsigned long long)weights_elems());
    release();
    bw = bw_, s = s_, device = device_;
    DDG_CUDA(cudaSetDevice(device));
    const int es = bw / 8;
    int64_t *tmp = nullptr;
    DDG_CUDA(cudaMalloc(&tmp, n * sizeof(int64_t)));
    DDG_CUDA(cudaMemcpy(tmp, h_blob, n * sizeof(int64_t), cudaMemcpyHostToDevice));
    uint64_t off = 0;
    int st = DDG_OK;
    for (int l = 0; l < NLAYERS && st == DDG_OK; l++) {
        const uint64_t nw = uint64_t(LAYER_IN[l]) * LAYER_OUT[l], nb = LAYER_OUT[l];
        DDG_CUDA(cudaMalloc(&W[l], nw * es));
        DDG_CUDA(cudaMalloc(&b2s[l], nb * es));
        if (bw == 32) {
            st = i64_to_ring<uint32_t>(tmp + off, (uint32_t *)W[l], nw, 0, nullptr);
            if (st == DDG_OK) st = i64_to_ring<uint32_t>(tmp + off + nw, (uint32_t *)b2s[l], nb, s, nullptr);
        } else {
            st = i64_to_ring<uint64_t>(tmp + off, (uint64_t *)W[l], nw, 0, nullptr);
            if (st == DDG_OK) st = i64_to_ring<uint64_t>(tmp + off + nw, (uint64_t *)b2s[l], nb, s, nullptr);
        }
        off += nw + nb;
    }
    // public 8-bit degree table: t[0] = 0, t[d] = llround(2^s / sqrt(d)), d <= NMAX (secure_adj_norm.h:139-184)
    uint64_t tab[256] = {0};
    for (int d = 1; d <= NMAX; d++) tab[d] = uint64_t(std::llround(std::ldexp(1.0, s) / std::sqrt(double(d))));
    DDG_CUDA(cudaMalloc(&table, 256 * es));
    if (bw == 32) {
        uint32_t t32[256];
        for (int i = 0; i < 256; i++) t32[i] = uint32_t(tab[i]);
        DDG_CUDA(cudaMemcpy(table, t32, sizeof(t32), cudaMemcpyHostToDevice));
    } else {
        DDG_CUDA(cudaMemcpy(table, tab, sizeof(tab), cudaMemcpyHostToDevice));
    }
    DDG_CUDA(cudaDeviceSynchronize());
    cudaFree(tmp);
    return st;
}

void DevWeights::release()
{
    for (int l = 0; l < NLAYERS; l++) {
        if (W[l]) cudaFree(W[l]);
        if (b2s[l]) cudaFree(b2s[l]);
        W[l] = b2s[l] = nullptr;
    }
    if (table) cudaFree(table);
    table = nullptr;
}

int Party::ensure_copy_stream()
{
    if (copy_stream) return DDG_OK;
    DDG_CUDA(cudaStreamCreateWithFlags(&copy_stream, cudaStreamNonBlocking));
    for (auto &ev : in_ev) DDG_CUDA(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
    return DDG_OK;
}

void Party::release_inputs()
{
    for (int i = 0; i < 4; i++)
        if (in_buf[i]) cudaFree(in_buf[i]), in_buf[i] = nullptr, in_cap[i] = 0;
    for (auto &ev : in_ev)
        if (ev) cudaEventDestroy(ev), ev = nullptr;
    if (copy_stream) cudaStreamDestroy(copy_stream), copy_stream = nullptr;
}

int Party::ensure_input(int which, uint64_t bytes)
{
    if (in_cap[which] >= bytes) return DDG_OK;
    if (in_buf[which]) cudaFree(in_buf[which]);
    in_buf[which] = nullptr;
    DDG_CUDA(cudaMalloc(&in_buf[which], bytes ? bytes : 16));
    in_cap[which] = bytes;
    return DDG_OK;
}

int keep_pool_memory(int device)
{
    static std::atomic<bool> done[64] = {};
    if (device >= 0 && device < 64 && done[device].load()) return DDG_OK;
    cudaMemPool_t pool;
    DDG_CUDA(cudaDeviceGetDefaultMemPool(&pool, device));
    uint64_t thr = ~uint64_t(0);
    DDG_CUDA(cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &thr));
    if (device >= 0 && device < 64) done[device].store(true);
    return DDG_OK;
}

// ------------------------------------------------------------------ comparison backend settings

// comparison split of the ReLU gates: 3 parts (default; fewest AES) or 2
// (smaller keys: 94.8 vs 111.8 MB per sample and party at bw=32).  Key sizes
// differ, so dealer and evaluators must run with the same setting.
static std::atomic<int> g_relu_parts{3};
void set_relu_parts(int parts) { g_relu_parts.store(parts == 2 ? 2 : 3); }
int relu_parts() { return g_relu_parts.load(); }
// comparison backend of the ReLU (and truncation) gates: dealer truth tables
// per digit with a Beaver AND tree (GATE_RELU*_TT and GATE_LRS_TT at the
// truncation sites; default: no AES online), OT-leaf digit tables with the
// same tree (GATE_RELU*_OT: 2 AES and ~8 key bytes per element and party
// besides the words) or DCF keys (split per relu_parts)
static std::atomic<int> g_relu_backend{DDG_RELU_TT};
void set_relu_backend(int backend)
{
    g_relu_backend.store(backend == DDG_RELU_OT || backend == DDG_RELU_TT ? backend : DDG_RELU_DCF);
}
int relu_backend() { return g_relu_backend.load(); }


// ------------------------------------------------------------------ entry points

uint64_t forward_key_bytes(int bw, int s, int B)
{
    if (bw == 32) {
        SizeExec<uint32_t> e;
        e.B = B, e.bw = bw, e.s = s;
        affinity_graph<uint32_t>(e);
        return align256(e.off);
    }
    SizeExec<uint64_t> e;
    e.B = B, e.bw = bw, e.s = s;
    affinity_graph<uint64_t>(e);
    return align256(e.off);
}

template <typename T>
static int dealer_t(int bw, int s, int B, uint64_t seed, const DevWeights &w, uint8_t *k0, uint8_t *k1,
                    cudaStream_t st)
{
    DealerExec<T> e;
    e.B = B, e.bw = bw, e.s = s, e.st = st, e.seed = seed, e.dk = dealer_key(seed), e.k0 = k0, e.k1 = k1, e.w = &w;
    affinity_graph<T>(e);
    if (e.err == DDG_OK) {
        cudaError_t ce = cudaStreamSynchronize(st);
        if (ce != cudaSuccess) {
            set_last_error("dealer: %s", cudaGetErrorString(ce));
            e.err = DDG_ERR_CUDA;
        }
    }
    if (e.err == DDG_OK) e.err = ring_gemm_tc_check(st);
    e.free_all();
    return e.err;
}

int dealer_forward(int bw, int s, int B, uint64_t seed, const DevWeights &w, uint8_t *k0, uint8_t *k1,
                   cudaStream_t st)
{
    DDG_TRY(keep_pool_memory(w.device));
    DDG_TRY(aes_device_init());
    return bw == 32 ? dealer_t<uint32_t>(bw, s, B, seed, w, k0, k1, st)
                    : dealer_t<uint64_t>(bw, s, B, seed, w, k0, k1, st);
}

// capture: the stream is being captured into a CUDA graph (forward_capture):
// the output goes to the device buffer capture_out (when not null) instead of
// the host, and nothing waits for the device
template <typename T>
static int eval_t(Party &P, int B, const void *x_sh, const void *adj_sh, const void *mask_sh, const void *prot_sh,
                  bool on_host, int64_t *h_out_raw, double *h_aff, bool capture = false, void *capture_out = nullptr)
{
    EvalExec<T> e;
    e.B = B, e.bw = P.bw, e.s = P.s, e.st = P.stream, e.P = &P, e.p = P.party;
    e.lazy = P.chan->peer_stable();  // consumers add the two shares of an opening on load
    const uint64_t sizes[4] = {uint64_t(B) * NMAX * FEAT, uint64_t(B) * NMAX * NMAX, uint64_t(B) * NMAX * POOL,
                               uint64_t(B) * PROT};
    const void *src[4] = {x_sh, adj_sh, mask_sh, prot_sh};
    if (on_host) {
        // host -> device on the party's copy stream, in order of first use; the
        // graph waits on each input's event right before revealing it
        DDG_TRY(P.ensure_copy_stream());
        DDG_CUDA(cudaEventRecord(P.in_ev[4], P.stream));
        DDG_CUDA(cudaStreamWaitEvent(P.copy_stream, P.in_ev[4], 0));  // buffers free: the last forward is done
        for (int i : {int(IN_ADJ), int(IN_X), int(IN_MASK), int(IN_PROT)}) {
            DDG_TRY(P.ensure_input(i, sizes[i] * sizeof(T)));
            DDG_CUDA(cudaMemcpyAsync(P.in_buf[i], src[i], sizes[i] * sizeof(T), cudaMemcpyHostToDevice,
                                     P.copy_stream));
            DDG_CUDA(cudaEventRecord(P.in_ev[i], P.copy_stream));
            e.in[i] = static_cast<const T *>(P.in_buf[i]);
            e.in_ready[i] = P.in_ev[i];
        }
    } else {
        for (int i = 0; i < 4; i++) e.in[i] = static_cast<const T *>(src[i]);
    }
    const uint64_t sent0 = P.chan->bytes_sent[P.party], rounds0 = P.chan->rounds[P.party];
    if (P.timing.enabled) {
        // one reference event per timing session: every timed launch of every
        // forward since enabling is read against it.  A capture does not record
        // it (a replay would move it); ddg_forward_graph_launch records it
        // before the first replay of a session instead.
        if (!P.ref_event) DDG_CUDA(cudaEventCreate(&P.ref_event));
        if (!P.ref_live && !capture) {
            DDG_TRY(record_timing_event(P.ref_event, P.stream));
            P.ref_live = true;
        }
        set_dcf_timing_sink(&P.timing);
    }
    affinity_graph<T>(e);
    set_dcf_timing_sink(nullptr);
    std::vector<T> h(B);
    if (e.err == DDG_OK && !capture)
        e.ok(cudaMemcpyAsync(h.data(), e.out, B * sizeof(T), cudaMemcpyDeviceToHost, P.stream) == cudaSuccess
                 ? DDG_OK : DDG_ERR_CUDA);
    if (e.err == DDG_OK && capture && capture_out)
        e.ok(cudaMemcpyAsync(capture_out, e.out, B * sizeof(T), cudaMemcpyDeviceToDevice, P.stream) == cudaSuccess
                 ? DDG_OK : DDG_ERR_CUDA);
    // the peer may still read buffers this party allocated: join before freeing
    int bs = P.chan->barrier(P.party, P.stream);
    if (e.err == DDG_OK) e.err = bs;
    e.free_all();
    if (capture) {
        if (e.err != DDG_OK) {
            if (auto *lp = dynamic_cast<LocalPairChannel *>(P.chan)) lp->fail();
            return e.err;
        }
        P.stats.bytes_sent = P.chan->bytes_sent[P.party] - sent0;
        P.stats.rounds = P.chan->rounds[P.party] - rounds0;
        P.stats.key_bytes_used = e.off;
        return DDG_OK;
    }
    cudaError_t ce = cudaStreamSynchronize(P.stream);
    if (e.err == DDG_OK && ce != cudaSuccess) {
        set_last_error("forward: %s", cudaGetErrorString(ce));
        e.err = DDG_ERR_CUDA;
    }
    if (e.err == DDG_OK) e.err = ring_gemm_tc_check(P.stream);
    if (e.err == DDG_OK) e.err = P.chan->status(P.party);  // the channel's device-side waits
    // the caller may reuse its host buffers once this returns
    if (P.copy_stream) {
        ce = cudaStreamSynchronize(P.copy_stream);
        if (e.err == DDG_OK && ce != cudaSuccess) {
            set_last_error("forward input copy: %s", cudaGetErrorString(ce));
            e.err = DDG_ERR_CUDA;
        }
    }
    if (e.err != DDG_OK) {
        if (auto *lp = dynamic_cast<LocalPairChannel *>(P.chan)) lp->fail();
        return e.err;
    }
    P.stats.bytes_sent = P.chan->bytes_sent[P.party] - sent0;
    P.stats.rounds = P.chan->rounds[P.party] - rounds0;
    P.stats.key_bytes_used = e.off;
    for (int i = 0; i < B; i++) {
        using S = typename std::conditional<sizeof(T) == 4, int32_t, int64_t>::type;
        const int64_t v = int64_t(S(h[i]));
        if (h_out_raw) h_out_raw[i] = v;
        // AFFINITY = int32(value) / 2^s (deepdtagen_inference.cu:594-606)
        if (h_aff) h_aff[i] = double(int32_t(uint32_t(uint64_t(v)))) / double(1ull << P.s);
    }
    return DDG_OK;
}

double union_ms(std::vector<std::pair<double, double>> v)
{
    std::sort(v.begin(), v.end());
    double tot = 0, cs = -1, ce = -1;
    for (auto &iv : v) {
        if (iv.first > ce) {
            if (ce > cs) tot += ce - cs;
            cs = iv.first, ce = iv.second;
        } else if (iv.second > ce) {
            ce = iv.second;
        }
    }
    if (ce > cs) tot += ce - cs;
    return tot;
}

// read back the party's pending timed launches (their forwards have finished:
// the forward drains its stream before returning) into its intervals and
// totals, and hand their events back to the pool
static int settle_recs(Party &P, const std::vector<DcfTiming::Rec> &recs)
{
    for (const auto &r : recs) {
        if (!r.done) continue;  // a launch that failed between its two events
        float a = 0, b = 0;
        DDG_CUDA(cudaEventElapsedTime(&a, P.ref_event, r.a));
        DDG_CUDA(cudaEventElapsedTime(&b, P.ref_event, r.b));
        P.intervals.emplace_back(double(a), double(b));
        P.dcf.launches += 1, P.dcf.bytes += r.bytes, P.dcf.aes += r.aes, P.dcf.sum_ms += double(b - a);
    }
    return DDG_OK;
}

// also adds the launches of the last replay of a CUDA graph that holds this
// party's timed launches, once per replay that ran since the last read-back
int settle_timing(Party &P)
{
    DcfTiming &t = P.timing;
    const bool graph = P.timing.enabled && P.graph_recs && P.graph_fresh;
    if (t.recs.empty() && !graph) return DDG_OK;
    DDG_CHECK(P.ref_live, DDG_ERR_STATE, "timed launches without a reference event");
    DDG_CUDA(cudaSetDevice(P.device));
    DDG_TRY(settle_recs(P, t.recs));
    t.recs.clear(), t.used = 0;
    if (graph) {
        DDG_TRY(settle_recs(P, *P.graph_recs));
        P.graph_fresh = false;
    }
    // forwards of one party never overlap, so the union over the whole
    // session is the sum of the per-forward unions
    P.dcf.union_ms = union_ms(P.intervals);
    return DDG_OK;
}

int reset_timing(Party &P, bool on)
{
    P.timing.enabled = on;
    P.timing.recs.clear(), P.timing.used = 0;
    P.dcf = DcfAcc();
    P.intervals.clear();
    P.ref_live = false;
    P.graph_fresh = false;
    if (!on) return DDG_OK;
    // events for ~28 forwards' comparison launches up front; the pool grows on
    // demand beyond that, while the host is ahead of the device
    DDG_CUDA(cudaSetDevice(P.device));
    while (P.timing.pool.size() < 4096) {
        cudaEvent_t e = nullptr;
        DDG_CUDA(cudaEventCreate(&e));
        P.timing.pool.push_back(e);
    }
    return DDG_OK;
}

// union of several parties' comparison-launch intervals since timing was
// enabled, on the timeline of ps[0] (all on one device); stored on ps[0]
int parties_dcf_union(Party *const *ps, int n)
{
    for (int i = 0; i < n; i++) {
        if (!ps[i]->timing.enabled || !ps[i]->ref_live) return DDG_OK;
        DDG_TRY(settle_timing(*ps[i]));
    }
    std::vector<std::pair<double, double>> all = ps[0]->intervals;
    for (int i = 1; i < n; i++) {
        DDG_CHECK(ps[i]->device == ps[0]->device, DDG_ERR_ARG, "DCF interval union needs one device");
        float off = 0;
        DDG_CUDA(cudaEventElapsedTime(&off, ps[0]->ref_event, ps[i]->ref_event));
        for (auto &iv : ps[i]->intervals) all.emplace_back(iv.first + off, iv.second + off);
    }
    ps[0]->dcf.pair_union_ms = union_ms(all);
    return DDG_OK;
}

int prepare_host_inputs(Party &P, int B)
{
    const uint64_t es = P.bw / 8;
    const uint64_t sizes[4] = {uint64_t(B) * NMAX * FEAT, uint64_t(B) * NMAX * NMAX, uint64_t(B) * NMAX * POOL,
                               uint64_t(B) * PROT};
    DDG_CUDA(cudaSetDevice(P.device));
    DDG_TRY(P.ensure_copy_stream());
    for (int i = 0; i < 4; i++) DDG_TRY(P.ensure_input(i, sizes[i] * es));
    return DDG_OK;
}

int forward_capture(Party &P, int B, const void *x_sh, const void *adj_sh, const void *mask_sh, const void *prot_sh,
                    void *d_out, bool on_host)
{
    DDG_CHECK(P.chan, DDG_ERR_STATE, "party %d has no channel", P.party);
    DDG_CHECK(P.keys, DDG_ERR_STATE, "party %d has no keys bound", P.party);
    DDG_CHECK(P.w.table, DDG_ERR_STATE, "party %d has no weights", P.party);
    DDG_CUDA(cudaSetDevice(P.device));
    return P.bw == 32 ? eval_t<uint32_t>(P, B, x_sh, adj_sh, mask_sh, prot_sh, on_host, nullptr, nullptr, true, d_out)
                      : eval_t<uint64_t>(P, B, x_sh, adj_sh, mask_sh, prot_sh, on_host, nullptr, nullptr, true, d_out);
}

int forward_eval(Party &P, int B, const void *x_sh, const void *adj_sh, const void *mask_sh, const void *prot_sh,
                 bool on_host, int64_t *h_out_raw, double *h_aff)
{
    DDG_CHECK(P.chan, DDG_ERR_STATE, "party %d has no channel", P.party);
    DDG_CHECK(P.keys, DDG_ERR_STATE, "party %d has no keys bound", P.party);
    DDG_CHECK(P.w.table, DDG_ERR_STATE, "party %d has no weights", P.party);
    DDG_CUDA(cudaSetDevice(P.device));
    DDG_TRY(keep_pool_memory(P.device));
    DDG_TRY(aes_device_init());
    return P.bw == 32 ? eval_t<uint32_t>(P, B, x_sh, adj_sh, mask_sh, prot_sh, on_host, h_out_raw, h_aff)
                      : eval_t<uint64_t>(P, B, x_sh, adj_sh, mask_sh, prot_sh, on_host, h_out_raw, h_aff);
}

}  // namespace ddg
