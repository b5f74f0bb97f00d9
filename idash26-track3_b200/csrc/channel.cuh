// Inter-party channels.  An opening sends this party's share and makes the
// peer's share readable on this party's device; the caller adds (or XORs).
// Replaces GpuPeer::reconstructInPlace (gpu_mpc/utils/gpu_comms.h:291-302;
// sigma_comms.cpp:106-150: D2H -> TCP -> H2D per opening).
//   LocalPairChannel: both parties in one process (two host threads).  Same
//     device: zero-copy, the consumer reads the peer's buffer after waiting on
//     the peer's event.  Different devices: cudaMemcpyPeerAsync over NVLink.
//   NcclChannel: one party per process, grouped ncclSend/ncclRecv with the
//     paired rank on the party's stream.
//   IpcChannel: one party per process, both on one node: CUDA-IPC send slots
//     read in place over NVLink, ordered by interprocess events and a shared-
//     memory block of generation counters.
#pragma once
#include <atomic>
#include <condition_variable>
#include <cstdint>
#include <mutex>
#include <string>

#include "common.cuh"

namespace ddg {

struct Channel {
    virtual ~Channel() {}
    // Send `bytes` at `send` (ready once work queued on `st` so far is done);
    // on return *peer points at the peer's bytes, readable by work queued on
    // `st` afterwards.  `recv` is a device buffer of `bytes` the channel may
    // use for the copy.
    virtual int exchange(int party, cudaStream_t st, const void *send, uint64_t bytes, void *recv,
                         const void **peer) = 0;
    // both parties reach this point; afterwards each party's stream has waited
    // for all work the peer queued before it
    virtual int barrier(int party, cudaStream_t st) = 0;
    virtual bool same_device() const { return false; }
    // errors the channel's own device-side waits recorded (read after the
    // party's stream has drained); DDG_OK for channels without device waits
    virtual int status(int party) { (void)party; return DDG_OK; }
    // exchange() needs the caller's `recv` buffer (it copies the peer's bytes there)
    virtual bool needs_recv_buffer() const { return !same_device(); }
    // the peer's bytes of an exchange stay valid to the end of the forward:
    // the peer's own buffer in place (an in-process pair) or the caller's recv
    // buffer; not a channel slot that later exchanges overwrite
    virtual bool peer_stable() const { return same_device() || needs_recv_buffer(); }
    // one party's forward, captured on its own stream, can be replayed from a
    // CUDA graph (every handoff of the capture happens on the device); `why`
    // says what stands in the way otherwise
    virtual bool replayable(std::string &why) const
    {
        why = "a channel whose exchanges wait on the host";
        return false;
    }
    // a graph replay holding `exchanges` exchanges of this party was enqueued
    virtual void note_replay(int party, uint64_t exchanges) { (void)party, (void)exchanges; }
    uint64_t bytes_sent[2] = {0, 0};
    uint64_t rounds[2] = {0, 0};
    int timeout_ms = 60000;
};

// Handoff between the two party threads: each exchange publishes the party's
// buffer for generation g with a release store of pub[party] = g, then spins
// (bounded) for the peer's g before sleeping on the condition variable; a
// sleeping waiter is counted in `sleepers` so that a publisher only takes the
// mutex to notify when someone sleeps.  The spin keeps the handoff of the
// ~100 openings of a forward at the latency of a cache line, where a futex
// wake-up costs tens of microseconds of host time that small gates cannot hide.
struct LocalPairChannel : Channel {
    struct Slot {
        const void *ptr = nullptr;
        uint64_t bytes = 0;
    };
    std::mutex mu;
    std::condition_variable cv;
    Slot slot[2][2];        // [party][gen & 1]
    uint64_t gen[2] = {0, 0};
    std::atomic<uint64_t> pub[2] = {{0}, {0}};
    std::atomic<int> sleepers{0};
    std::atomic<bool> broken{false};
    cudaEvent_t ev[2][2] = {{nullptr, nullptr}, {nullptr, nullptr}};
    int dev[2] = {0, 0};
    LocalPairChannel(int dev0, int dev1);
    ~LocalPairChannel() override;
    int exchange(int party, cudaStream_t st, const void *send, uint64_t bytes, void *recv, const void **peer) override;
    int barrier(int party, cudaStream_t st) override;
    bool same_device() const override { return dev[0] == dev[1]; }
    void fail();  // wake a waiting peer with an error (the other party gave up)
};

// The caller's own transport (ddg_comm, include/ddg_fss.h): every opening
// hands the caller this party's device send buffer, a device receive buffer
// and the party's stream; the callback returns once the peer's bytes of the
// same opening are (or, in stream order, will be) in the receive buffer.
// This is the reference's GpuPeer::reconstructInPlace (gpu_comms.h:291-302)
// seam: a caller can run the openings over its own sockets or fabric.
struct CallbackChannel : Channel {
    ddg_comm comm{};
    int exchange(int party, cudaStream_t st, const void *send, uint64_t bytes, void *recv, const void **peer) override;
    int barrier(int, cudaStream_t) override { return DDG_OK; }  // the peer never reads this party's buffers
    bool needs_recv_buffer() const override { return true; }
};

Channel *make_nccl_channel(const void *unique_id, int nranks, int rank, int peer_rank, int device, int *status);
// CUDA-IPC channel between two party processes on one node (channel.cu); both
// call it with the same `name` (a POSIX shared-memory name, no slash)
// push = true: each party's kernels write its share into the peer's receive
// slot (peer stores over NVLink) and raise a flag in the peer's memory; the
// consumer waits for the flag on the device and reads its own HBM (no host
// wait per opening).  Needs the two parties on different GPUs.
Channel *make_ipc_channel(const char *name, int party, int device, uint64_t slot_bytes, int timeout_ms, int *status,
                          bool push = false);
int nccl_unique_id(void *out128);

}  // namespace ddg
