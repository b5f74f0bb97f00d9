#include <chrono>
#include <cstring>

#include "channel.cuh"

#ifdef DDG_HAVE_NCCL
#include <nccl.h>
#endif

namespace ddg {

LocalPairChannel::LocalPairChannel(int dev0, int dev1)
{
    dev[0] = dev0, dev[1] = dev1;
    for (int p = 0; p < 2; p++) {
        int prev = 0;
        cudaGetDevice(&prev);
        cudaSetDevice(dev[p]);
        for (int g = 0; g < 2; g++) cudaEventCreateWithFlags(&ev[p][g], cudaEventDisableTiming);
        cudaSetDevice(prev);
    }
}

LocalPairChannel::~LocalPairChannel()
{
    for (int p = 0; p < 2; p++)
        for (int g = 0; g < 2; g++)
            if (ev[p][g]) cudaEventDestroy(ev[p][g]);
}

void LocalPairChannel::fail()
{
    std::lock_guard<std::mutex> g(mu);
    broken = true;
    cv.notify_all();
}

int LocalPairChannel::exchange(int party, cudaStream_t st, const void *send, uint64_t bytes, void *recv,
                               const void **peer)
{
    const int q = 1 - party;
    std::unique_lock<std::mutex> lk(mu);
    const uint64_t g = ++gen[party];
    cudaEvent_t e = ev[party][g & 1];
    DDG_CUDA(cudaEventRecord(e, st));
    slot[party][g & 1] = Slot{send, bytes, g};
    cv.notify_all();
    const bool ok = cv.wait_for(lk, std::chrono::milliseconds(timeout_ms),
                                [&] { return broken || slot[q][g & 1].gen == g; });
    DDG_CHECK(!broken, DDG_ERR_PEER, "peer party failed during exchange %llu", (unsigned long long)g);
    if (!ok) {
        broken = true;
        cv.notify_all();
        set_last_error("peer party did not reach exchange %llu within %d ms", (unsigned long long)g, timeout_ms);
        return DDG_ERR_PEER;
    }
    const Slot s = slot[q][g & 1];
    cudaEvent_t pe = ev[q][g & 1];
    lk.unlock();
    DDG_CHECK(s.bytes == bytes, DDG_ERR_PEER, "exchange %llu size mismatch: %llu vs peer %llu",
              (unsigned long long)g, (unsigned long long)bytes, (unsigned long long)s.bytes);
    DDG_CUDA(cudaStreamWaitEvent(st, pe, 0));
    if (dev[0] == dev[1]) {
        *peer = s.ptr;
    } else {
        DDG_CUDA(cudaMemcpyPeerAsync(recv, dev[party], s.ptr, dev[q], bytes, st));
        *peer = recv;
    }
    bytes_sent[party] += bytes;
    rounds[party] += 1;
    return DDG_OK;
}

int LocalPairChannel::barrier(int party, cudaStream_t st)
{
    // an empty exchange orders both streams against each other; it is not an opening
    const void *dummy = nullptr;
    DDG_TRY(exchange(party, st, nullptr, 0, nullptr, &dummy));
    rounds[party] -= 1;
    return DDG_OK;
}

#ifdef DDG_HAVE_NCCL
struct NcclChannel : Channel {
    ncclComm_t comm = nullptr;
    int peer_rank = -1;
    ~NcclChannel() override
    {
        if (comm) ncclCommDestroy(comm);
    }
    int exchange(int party, cudaStream_t st, const void *send, uint64_t bytes, void *recv, const void **peer) override
    {
        if (bytes) {
            ncclResult_t r = ncclGroupStart();
            if (r == ncclSuccess) r = ncclSend(send, bytes, ncclUint8, peer_rank, comm, st);
            if (r == ncclSuccess) r = ncclRecv(recv, bytes, ncclUint8, peer_rank, comm, st);
            ncclResult_t r2 = ncclGroupEnd();
            DDG_CHECK(r == ncclSuccess && r2 == ncclSuccess, DDG_ERR_PEER, "nccl exchange failed: %s",
                      ncclGetErrorString(r != ncclSuccess ? r : r2));
        }
        *peer = recv;
        bytes_sent[party] += bytes;
        rounds[party] += 1;
        return DDG_OK;
    }
    int barrier(int party, cudaStream_t st) override
    {
        // a one-word exchange orders the two ranks' streams
        (void)party;
        return DDG_OK;
    }
};

Channel *make_nccl_channel(const void *unique_id, int nranks, int rank, int peer_rank, int device, int *status)
{
    ncclUniqueId id;
    memcpy(&id, unique_id, sizeof(id));
    if (cudaSetDevice(device) != cudaSuccess) {
        set_last_error("cudaSetDevice(%d) failed", device);
        *status = DDG_ERR_CUDA;
        return nullptr;
    }
    auto *c = new NcclChannel();
    c->peer_rank = peer_rank;
    ncclResult_t r = ncclCommInitRank(&c->comm, nranks, id, rank);
    if (r != ncclSuccess) {
        set_last_error("ncclCommInitRank failed: %s", ncclGetErrorString(r));
        c->comm = nullptr;
        delete c;
        *status = DDG_ERR_PEER;
        return nullptr;
    }
    *status = DDG_OK;
    return c;
}

int nccl_unique_id(void *out128)
{
    ncclUniqueId id;
    ncclResult_t r = ncclGetUniqueId(&id);
    DDG_CHECK(r == ncclSuccess, DDG_ERR_PEER, "ncclGetUniqueId failed: %s", ncclGetErrorString(r));
    static_assert(sizeof(ncclUniqueId) == 128, "nccl unique id size");
    memcpy(out128, &id, sizeof(id));
    return DDG_OK;
}
#else
Channel *make_nccl_channel(const void *, int, int, int, int, int *status)
{
    set_last_error("libddg.so was built without NCCL");
    *status = DDG_ERR_STATE;
    return nullptr;
}
int nccl_unique_id(void *)
{
    set_last_error("libddg.so was built without NCCL");
    return DDG_ERR_STATE;
}
#endif

}  // namespace ddg
