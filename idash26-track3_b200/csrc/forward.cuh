// The affinity-branch graph and the party / dealer contexts that walk it.
#pragma once
#include <vector>

#include "channel.cuh"
#include "common.cuh"

namespace ddg {

constexpr int NMAX = 138, FEAT = 94, POOL = 376, PROT = 128;
constexpr int NLAYERS = 9;
// (in, out) per layer, forward order: gcn 0-2, drug fc 3-4, fusion 5-8
// (reference gpu_mpc/deepdtagen_inference.cu:113-123)
constexpr int LAYER_IN[NLAYERS] = {94, 188, 282, 376, 1024, 256, 1024, 512, 256};
constexpr int LAYER_OUT[NLAYERS] = {188, 282, 376, 1024, 128, 1024, 512, 256, 1};

inline uint64_t weights_elems()
{
    uint64_t n = 0;
    for (int l = 0; l < NLAYERS; l++) n += uint64_t(LAYER_IN[l]) * LAYER_OUT[l] + LAYER_OUT[l];
    return n;
}

// device copy of the public weights as ring elements: W (in,out) and b << s
struct DevWeights {
    int bw = 0, s = 0, device = -1;
    void *W[NLAYERS] = {};
    void *b2s[NLAYERS] = {};
    void *table = nullptr;  // 256-entry inverse-sqrt degree table
    int load(const int64_t *h_blob, uint64_t n, int bw_, int s_, int device_);
    void release();
};

// per-forward statistics of one party
struct PartyStats {
    uint64_t bytes_sent = 0, rounds = 0, key_bytes_used = 0;
    double ms_total = 0;
};

// accumulated DCF-kernel timing (see DcfTiming): launches, algorithmic bytes,
// AES blocks, summed launch durations, union of this party's launch intervals,
// union over both parties of an in-process pair (stored on party 0)
struct DcfAcc {
    double launches = 0, bytes = 0, aes = 0, sum_ms = 0, union_ms = 0, pair_union_ms = 0;
};

struct Party {
    int party = 0, bw = 32, s = 12, device = 0;
    cudaStream_t stream = nullptr;
    Channel *chan = nullptr;
    bool owns_chan = false;
    int timeout_ms = 60000;  // bound on every wait for the peer (applied to the channel)
    const uint8_t *keys = nullptr;
    uint64_t key_bytes = 0;
    DevWeights w;
    PartyStats stats;
    DcfTiming timing;
    DcfAcc dcf;
    cudaEvent_t ref_event = nullptr;                     // start of the first forward since timing was enabled
    bool ref_live = false;                               // ref_event is recorded for this timing session
    std::vector<std::pair<double, double>> intervals;    // read-back comparison launches, ms after ref_event
    // comparison launches captured into a CUDA graph (ddg_forward_graph): the
    // graph owns these records' events and every replay re-records them;
    // graph_fresh = a replay ran since they were last read back
    const std::vector<DcfTiming::Rec> *graph_recs = nullptr;
    bool graph_fresh = false;
    // device staging of host inputs (kept across forwards), copied on a side
    // stream; in_ev[0..3] mark each input's arrival, in_ev[4] the start of a forward
    void *in_buf[4] = {};
    uint64_t in_cap[4] = {};
    cudaStream_t copy_stream = nullptr;
    cudaEvent_t in_ev[5] = {};
    int ensure_input(int which, uint64_t bytes);
    int ensure_copy_stream();
    void release_inputs();
};

uint64_t forward_key_bytes(int bw, int s, int B);
void set_relu_parts(int parts);
int relu_parts();  // 3 or 2
void set_relu_backend(int backend);  // DDG_RELU_DCF or DDG_RELU_OT
int relu_backend();
double union_ms(std::vector<std::pair<double, double>> v);
int settle_timing(Party &P);
int reset_timing(Party &P, bool on);
int parties_dcf_union(Party *const *ps, int n);
int forward_eval(Party &P, int B, const void *x_sh, const void *adj_sh, const void *mask_sh, const void *prot_sh,
                 bool on_host, int64_t *h_out_raw, double *h_aff);
// enqueue one forward on P.stream while it is being captured into a CUDA
// graph: the revealed output (party 0) goes to d_out, and nothing waits for
// the device (the caller ends the capture and replays it).  on_host: the
// inputs are pinned host buffers, copied on the party's copy stream (which
// joins the capture) into its staging buffers (prepare_host_inputs first)
int forward_capture(Party &P, int B, const void *x_sh, const void *adj_sh, const void *mask_sh, const void *prot_sh,
                    void *d_out, bool on_host = false);
// the party's copy stream and device staging buffers of B samples' inputs
int prepare_host_inputs(Party &P, int B);
int dealer_forward(int bw, int s, int B, uint64_t seed, const DevWeights &w, uint8_t *k0, uint8_t *k1,
                   cudaStream_t st);

}  // namespace ddg

// the opaque handle of the C ABI (include/ddg_fss.h)
struct ddg_party {
    ddg::Party P;
};
