#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstring>
#include <string>
#include <thread>

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
    broken.store(true);
    std::lock_guard<std::mutex> g(mu);
    cv.notify_all();
}

int LocalPairChannel::exchange(int party, cudaStream_t st, const void *send, uint64_t bytes, void *recv,
                               const void **peer)
{
    const int q = 1 - party;
    const uint64_t g = ++gen[party];
    cudaEvent_t e = ev[party][g & 1];
    DDG_CUDA(cudaEventRecord(e, st));
    slot[party][g & 1] = Slot{send, bytes};
    pub[party].store(g);  // sequentially consistent: ordered against the sleepers check below
    if (sleepers.load() > 0) {
        std::lock_guard<std::mutex> lk(mu);
        cv.notify_all();
    }
    // the peer's generation g: spin first, then sleep with the deadline
    bool ready = false;
    for (int it = 0; it < 200000 && !(ready = pub[q].load() >= g) && !broken.load(); it++) {
        if (it > 2000) std::this_thread::yield();
    }
    if (!ready && !broken.load()) {
        std::unique_lock<std::mutex> lk(mu);
        sleepers.fetch_add(1);
        ready = cv.wait_for(lk, std::chrono::milliseconds(timeout_ms),
                            [&] { return broken.load() || pub[q].load() >= g; });
        sleepers.fetch_sub(1);
        ready = ready && pub[q].load() >= g;
    }
    DDG_CHECK(!broken.load(), DDG_ERR_PEER, "peer party failed during exchange %llu", (unsigned long long)g);
    if (!ready) {
        fail();
        set_last_error("peer party did not reach exchange %llu within %d ms", (unsigned long long)g, timeout_ms);
        return DDG_ERR_PEER;
    }
    const Slot s = slot[q][g & 1];
    cudaEvent_t pe = ev[q][g & 1];
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

int CallbackChannel::exchange(int party, cudaStream_t st, const void *send, uint64_t bytes, void *recv,
                              const void **peer)
{
    if (bytes) {
        const int r = comm.exchange(comm.user, party, send, recv, bytes, st);
        DDG_CHECK(r == 0, DDG_ERR_PEER, "the caller's exchange callback failed (%d) on an opening of %llu bytes", r,
                  (unsigned long long)bytes);
    }
    *peer = recv;
    bytes_sent[party] += bytes;
    rounds[party] += 1;
    return DDG_OK;
}

// ------------------------------------------------------------------ IPC channel
//
// Two party processes on one node, one GPU each.  Every party owns S = 4
// send slots of `slot_bytes` in one cudaMalloc'd arena, exported with
// cudaIpcGetMemHandle, and two interprocess events per slot: "posted" (its
// share of generation g sits in slot g % S) and "read" (it has finished
// reading the peer's slot g % S).  A POSIX shared-memory block carries the
// handles and, per party, the last generation posted and the last one read.
// Exchange g of party p:
//   1. the read of generation g - 1 is complete on p's stream: record read[(g-1)%S], publish read = g - 1;
//   2. slot g % S is free once the peer has read generation g - S: wait (host,
//      bounded) for its read >= g - S, then make the stream wait on its read[g%S];
//   3. copy the share into the slot, record posted[g%S], publish posted = g;
//   4. wait (host, bounded) for the peer's posted >= g, make the stream wait on
//      its posted[g%S]; the peer's share is then read in place over NVLink.
// An event is re-recorded only after the host has seen the generation it
// guards consumed, so every stream wait binds to the right record.  Host
// waits give up after timeout_ms with DDG_ERR_PEER and mark the block failed,
// which the peer then also reports.  Teardown: each party's stream is idle
// before its channel is destroyed; the arena is freed only once the peer has
// said (or timed out saying) that it is closing too, so no kernel of the peer
// can still be reading it.

struct IpcShared {
    std::atomic<uint32_t> ready[2], closing[2];
    std::atomic<uint32_t> failed;
    std::atomic<uint64_t> posted[2], read[2];
    uint64_t slot_bytes;
    uint32_t push;                    // push mode (both parties must agree)
    cudaIpcMemHandle_t arena[2];
    cudaIpcEventHandle_t ev_posted[2][4], ev_read[2][4];
    cudaIpcMemHandle_t flags[2];      // push mode: each party's PushFlags block
    char bus_id[2][32];               // PCI bus id of each party's GPU
};

// ------------------------------------------------------------------ push mode (device-side handoff)
//
// Every party owns, in its own device memory, S receive slots (the arena) and
// a PushFlags block; both are mapped into the peer's process.  Generations
// are numbered on the device: exchange i (1-based) since the last barrier has
// generation g = base + i, where `base` (this party's own flags) is advanced
// by the barrier to the next multiple of S above the last generation, so slot
// s = (g-1) % S = (i-1) % S is known to the host at enqueue time and the same
// launches replay unchanged from a CUDA graph (both parties advance their
// bases identically: their exchange sequences are the same).  Exchange g of
// party p, enqueued on p's stream:
//   1. k_push_send: every block's first thread publishes "p consumed the
//      peer's generation g-1" into the peer's flags (every kernel that read
//      it came before this one on the stream) and waits until the peer has
//      consumed p's generation g-S, the last one that used slot s on the
//      peer's side; the blocks then copy the share into the peer's slot s
//      with peer stores (16- or 4-byte words), each fences at system scope,
//      and the last block to finish raises the peer's `posted` to g;
//   2. k_push_wait (one thread), or the last block of k_push_send itself when
//      the forward is being captured into a graph: wait until the peer's
//      generation g has been posted into p's own slot s; the consumers then
//      read local HBM.
// The waits are bounded by the party's timeout: one that gives up sets `err`,
// which the host reads after the forward (status()).  Both parties must be on
// different GPUs: kernels that wait on one another are never launched on one
// GPU.  A host-launched step 2 is enqueued only once the peer's host has
// enqueued its step 1 of the same exchange (the shared `posted` counters,
// published at enqueue time; the slot wait of step 1 is covered by the
// previous exchange's).  Every device-side wait therefore depends on work
// that is already queued on the peer's GPU, never on a launch still to come
// from the peer's host: a context-wide synchronisation on either GPU (a
// cudaMalloc or cudaFree, a kernel's first launch under lazy module loading)
// taken by another thread of the process, e.g. a second party of the same
// GPU, always drains instead of closing a cycle through the peer's host.  A
// graph replay enqueues the whole forward at once; it is allowed only for a
// party that is the one push-mode party of its device in the process (no
// other thread of the process can then wait on its device mid-forward).
struct PushFlags {
    unsigned long long posted;     // the peer's last generation in this party's receive slots
    unsigned long long consumed;   // this party's last generation that the peer has consumed
    unsigned int done_blocks;      // k_push_send's block counter (this party's own)
    unsigned int err;              // a wait of this party gave up
    unsigned long long base;       // generation base of the exchanges since the last barrier (this party's own)
    unsigned long long pad[28];
};
static_assert(sizeof(PushFlags) == 256, "flags block");

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long *p)
{
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(unsigned long long *p, unsigned long long v)
{
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long globaltimer_ns()
{
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void st_release_sys_u32(unsigned int *p, unsigned int v)
{
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// bounded spin of one thread until *p >= target.  After limit_ns it gives up:
// it sets this party's err and the peer's (the peer's waits then give up at
// once instead of each running out its own limit), and returns false; a wait
// that finds err already set gives up at once.  A channel whose wait gave up
// is failed: its forward reports DDG_ERR_PEER (status()).
__device__ bool spin_until(const unsigned long long *p, unsigned long long target, unsigned long long limit_ns,
                           PushFlags *me, PushFlags *peer)
{
    if (ld_acquire_sys(p) >= target) return true;
    const unsigned long long t0 = globaltimer_ns();
    for (unsigned int it = 0;; it++) {
        if (ld_acquire_sys(p) >= target) return true;
        if ((it & 63u) == 0 &&
            (*reinterpret_cast<volatile unsigned int *>(&me->err) != 0 || globaltimer_ns() - t0 > limit_ns)) {
            atomicOr(&me->err, 1u);
            st_release_sys_u32(&peer->err, 1u);
            return false;
        }
        __nanosleep(200);
    }
}

template <bool kWait>
__global__ void k_push_send(const uint32_t *src, uint32_t *dst, uint64_t words, PushFlags *me, PushFlags *peer,
                            unsigned long long rel, unsigned int S, unsigned long long limit_ns)
{
    const unsigned long long g = me->base + rel;
    __shared__ bool go;
    if (threadIdx.x == 0) {
        // every block publishes (the same value), so whichever block runs first unblocks the peer
        st_release_sys(&peer->consumed, g - 1);
        go = g <= S || spin_until(&me->consumed, g - S, limit_ns, me, peer);
    }
    __syncthreads();
    if (go) {
        const uint64_t tid = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x, nth = uint64_t(gridDim.x) * blockDim.x;
        if ((reinterpret_cast<uintptr_t>(src) & 15) == 0 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
            const uint64_t n16 = words / 4;
            const uint4 *s4 = reinterpret_cast<const uint4 *>(src);
            uint4 *d4 = reinterpret_cast<uint4 *>(dst);
            for (uint64_t i = tid; i < n16; i += nth) d4[i] = s4[i];
            for (uint64_t i = 4 * n16 + tid; i < words; i += nth) dst[i] = src[i];
        } else {
            for (uint64_t i = tid; i < words; i += nth) dst[i] = src[i];
        }
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
        if (atomicAdd(&me->done_blocks, 1u) == gridDim.x - 1) {
            me->done_blocks = 0;
            __threadfence_system();
            st_release_sys(&peer->posted, g);
            if (kWait) spin_until(&me->posted, g, limit_ns, me, peer);
        }
    }
}

__global__ void k_push_wait(PushFlags *me, PushFlags *peer, unsigned long long rel, unsigned long long limit_ns)
{
    if (threadIdx.x == 0) spin_until(&me->posted, me->base + rel, limit_ns, me, peer);
}

// barrier: the next exchange starts a new run of S-aligned generations
__global__ void k_push_advance(PushFlags *me, unsigned long long rel, unsigned int S)
{
    if (threadIdx.x == 0) me->base += (rel + S - 1) / S * S;
}

// live push-mode parties per device in this process (a graph replay needs to be the only one)
static std::atomic<int> g_push_parties[64];

struct IpcChannel : Channel {
    static constexpr int S = 4;
    int party = 0, device = 0;
    bool push = false;
    uint64_t slot_bytes = 0, gen = 0;
    uint64_t rel = 0;   // push mode: exchanges since the last barrier (the device adds its base)
    uint64_t hgen = 0;  // push mode: exchanges enqueued by this party's host, published for the peer's host
    std::string shm_name;
    IpcShared *sh = nullptr;
    uint8_t *arena = nullptr, *peer_arena = nullptr;
    PushFlags *flags = nullptr, *peer_flags = nullptr;  // push mode
    unsigned int *h_err = nullptr;                      // pinned mirror of flags->err
    int push_blocks = 148;
    bool counted = false;  // push mode: counted in g_push_parties[device]
    cudaEvent_t posted[S] = {}, read[S] = {}, peer_posted[S] = {}, peer_read[S] = {};

    ~IpcChannel() override
    {
        cudaSetDevice(device);
        if (sh && sh->ready[party].load()) {
            sh->closing[party].store(1, std::memory_order_release);
            const auto t0 = std::chrono::steady_clock::now();
            while (sh->ready[1 - party].load() && !sh->closing[1 - party].load(std::memory_order_acquire) &&
                   !sh->failed.load() &&
                   std::chrono::steady_clock::now() - t0 < std::chrono::milliseconds(timeout_ms))
                std::this_thread::sleep_for(std::chrono::milliseconds(1));
        }
        if (peer_arena) cudaIpcCloseMemHandle(peer_arena);
        if (peer_flags) cudaIpcCloseMemHandle(peer_flags);
        if (flags) cudaFree(flags);
        if (counted) g_push_parties[device].fetch_sub(1);
        if (h_err) cudaFreeHost(h_err);
        for (int i = 0; i < S; i++) {
            for (cudaEvent_t e : {posted[i], read[i], peer_posted[i], peer_read[i]})
                if (e) cudaEventDestroy(e);
        }
        if (arena) cudaFree(arena);
        if (sh) munmap(sh, sizeof(IpcShared));
        if (party == 0 && !shm_name.empty()) shm_unlink(shm_name.c_str());
    }

    int wait_for(std::atomic<uint64_t> &v, uint64_t target, const char *what)
    {
        const auto t0 = std::chrono::steady_clock::now();
        for (uint64_t it = 0; v.load(std::memory_order_acquire) < target; it++) {
            if (sh->failed.load()) {
                set_last_error("peer party failed (IPC channel)");
                return DDG_ERR_PEER;
            }
            if ((it & 1023) == 0 && std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(timeout_ms)) {
                sh->failed.store(1);
                set_last_error("peer party did not reach %s %llu within %d ms", what, (unsigned long long)target,
                               timeout_ms);
                return DDG_ERR_PEER;
            }
            if (it > 4096) std::this_thread::yield();
        }
        return DDG_OK;
    }

    int finish_read(cudaStream_t st)
    {
        if (gen == 0) return DDG_OK;
        DDG_CUDA(cudaEventRecord(read[(gen - 1) % S], st));
        sh->read[party].store(gen, std::memory_order_release);
        return DDG_OK;
    }

    static bool capturing(cudaStream_t st)
    {
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        return cudaStreamIsCapturing(st, &cs) == cudaSuccess && cs == cudaStreamCaptureStatusActive;
    }

    int exchange_push(int p, cudaStream_t st, const void *send, uint64_t bytes, const void **peer)
    {
        DDG_CHECK(bytes % 4 == 0, DDG_ERR_ARG, "IPC push exchange of %llu bytes (not whole 32-bit words)",
                  (unsigned long long)bytes);
        const uint64_t i = ++rel;
        const uint64_t s = (i - 1) % S;
        const unsigned long long limit = 1000000ull * unsigned(timeout_ms);
        const uint64_t words = bytes / 4;
        const int blocks = words ? int(std::min<uint64_t>(push_blocks, (words + 1023) / 1024)) : 1;
        const uint32_t *src = static_cast<const uint32_t *>(send);
        uint32_t *dst = reinterpret_cast<uint32_t *>(peer_arena + s * slot_bytes);
        if (capturing(st)) {
            // a graph replay enqueues the whole forward at once: post and wait in one launch
            k_push_send<true><<<blocks, 256, 0, st>>>(src, dst, words, flags, peer_flags, i, S, limit);
            note_launch();
        } else {
            k_push_send<false><<<blocks, 256, 0, st>>>(src, dst, words, flags, peer_flags, i, S, limit);
            note_launch();
            sh->posted[p].store(++hgen, std::memory_order_release);
            DDG_TRY(wait_for(sh->posted[1 - p], hgen, "enqueue of exchange"));
            k_push_wait<<<1, 32, 0, st>>>(flags, peer_flags, i, limit);
            note_launch();
        }
        DDG_CUDA(cudaGetLastError());
        *peer = arena + s * slot_bytes;
        bytes_sent[p] += bytes;
        rounds[p] += 1;
        return DDG_OK;
    }

    // a graph replay of `exchanges` exchanges was enqueued: publish them for the
    // peer's host, as the host-launched exchanges do one by one
    void note_replay(int p, uint64_t exchanges) override
    {
        if (!push) return;
        hgen += exchanges;
        sh->posted[p].store(hgen, std::memory_order_release);
    }

    bool replayable(std::string &why) const override
    {
        if (!push) {
            why = "IPC channel with host handoffs (its exchanges wait on the host)";
            return false;
        }
        if (device < 0 || device >= 64 || g_push_parties[device].load() != 1) {
            why = "more than one push-mode party on this device in the process";
            return false;
        }
        return true;
    }

    int status(int p) override
    {
        (void)p;
        if (!push) return DDG_OK;
        DDG_CHECK(*reinterpret_cast<volatile unsigned int *>(h_err) == 0, DDG_ERR_PEER,
                  "IPC push channel: a device-side wait for the peer gave up after %d ms", timeout_ms);
        return DDG_OK;
    }

    int exchange(int p, cudaStream_t st, const void *send, uint64_t bytes, void *recv, const void **peer) override
    {
        (void)recv;
        const int q = 1 - p;
        DDG_CHECK(bytes <= slot_bytes, DDG_ERR_ARG, "IPC exchange of %llu bytes exceeds the %llu-byte slots",
                  (unsigned long long)bytes, (unsigned long long)slot_bytes);
        if (push) return exchange_push(p, st, send, bytes, peer);
        DDG_TRY(finish_read(st));  // generation gen (the previous exchange) has been read by work queued on st
        const uint64_t g = ++gen;
        const int s = int((g - 1) % S);
        if (g > uint64_t(S)) {
            DDG_TRY(wait_for(sh->read[q], g - S, "read of generation"));
            DDG_CUDA(cudaStreamWaitEvent(st, peer_read[s], 0));
        }
        uint8_t *slot = arena + uint64_t(s) * slot_bytes;
        if (bytes) DDG_CUDA(cudaMemcpyAsync(slot, send, bytes, cudaMemcpyDeviceToDevice, st));
        DDG_CUDA(cudaEventRecord(posted[s], st));
        sh->posted[p].store(g, std::memory_order_release);
        DDG_TRY(wait_for(sh->posted[q], g, "posting of generation"));
        DDG_CUDA(cudaStreamWaitEvent(st, peer_posted[s], 0));
        *peer = peer_arena + uint64_t(s) * slot_bytes;
        bytes_sent[p] += bytes;
        rounds[p] += 1;
        return DDG_OK;
    }

    bool needs_recv_buffer() const override { return false; }  // the peer's slot (or this party's) is read in place

    int barrier(int p, cudaStream_t st) override
    {
        // an empty exchange: both parties posted everything before it, and the
        // reads of the last real exchange are published
        const void *dummy = nullptr;
        DDG_TRY(exchange(p, st, nullptr, 0, nullptr, &dummy));
        rounds[p] -= 1;
        if (push) {
            // the next exchange starts on a slot-aligned generation; the device-side
            // waits' verdict is read by status() once the stream has drained
            k_push_advance<<<1, 32, 0, st>>>(flags, rel, S);
            note_launch();
            rel = 0;
            DDG_CUDA(cudaMemcpyAsync(h_err, &flags->err, sizeof(unsigned int), cudaMemcpyDeviceToHost, st));
        }
        return DDG_OK;
    }
};

Channel *make_ipc_channel(const char *name, int party, int device, uint64_t slot_bytes, int timeout_ms, int *status,
                          bool push)
{
    *status = DDG_ERR_PEER;
    auto fail = [&](int code, const char *fmt, const char *a) {
        set_last_error(fmt, a);
        *status = code;
        return static_cast<Channel *>(nullptr);
    };
    if (cudaSetDevice(device) != cudaSuccess) return fail(DDG_ERR_CUDA, "cudaSetDevice failed%s", "");
    auto *c = new IpcChannel();
    c->push = push;
    c->party = party, c->device = device, c->slot_bytes = (slot_bytes + 255) & ~uint64_t(255);
    c->timeout_ms = timeout_ms;
    c->shm_name = std::string("/") + name;
    // party 0 creates and sizes the block, party 1 opens it once it exists
    int fd = -1;
    const auto t0 = std::chrono::steady_clock::now();
    while (true) {
        fd = party == 0 ? shm_open(c->shm_name.c_str(), O_CREAT | O_EXCL | O_RDWR, 0600)
                        : shm_open(c->shm_name.c_str(), O_RDWR, 0600);
        if (fd >= 0) {
            struct stat stt;
            if (party == 0) {
                if (ftruncate(fd, sizeof(IpcShared)) != 0) {
                    close(fd);
                    delete c;
                    return fail(DDG_ERR_PEER, "cannot size the shared block %s", name);
                }
                break;
            }
            if (fstat(fd, &stt) == 0 && uint64_t(stt.st_size) >= sizeof(IpcShared)) break;
            close(fd);
            fd = -1;
        } else if (party == 0) {
            delete c;
            return fail(DDG_ERR_PEER, "cannot create the shared block %s (name in use?)", name);
        }
        if (std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(timeout_ms)) {
            delete c;
            return fail(DDG_ERR_PEER, "party 0 never created the shared block %s", name);
        }
        std::this_thread::sleep_for(std::chrono::milliseconds(2));
    }
    void *m = mmap(nullptr, sizeof(IpcShared), PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
    close(fd);
    if (m == MAP_FAILED) {
        delete c;
        return fail(DDG_ERR_PEER, "cannot map the shared block %s", name);
    }
    c->sh = static_cast<IpcShared *>(m);
    IpcShared *sh = c->sh;
    // own arena and events, published in the block
    const int S = IpcChannel::S;
    if (cudaMalloc(&c->arena, uint64_t(S) * c->slot_bytes) != cudaSuccess ||
        cudaIpcGetMemHandle(&sh->arena[party], c->arena) != cudaSuccess) {
        c->sh->failed.store(1);  // the peer stops waiting on us
        delete c;
        return fail(DDG_ERR_CUDA, "IPC arena allocation / export failed%s", "");
    }
    for (int i = 0; i < S; i++) {
        if (cudaEventCreateWithFlags(&c->posted[i], cudaEventDisableTiming | cudaEventInterprocess) != cudaSuccess ||
            cudaEventCreateWithFlags(&c->read[i], cudaEventDisableTiming | cudaEventInterprocess) != cudaSuccess ||
            cudaIpcGetEventHandle(&sh->ev_posted[party][i], c->posted[i]) != cudaSuccess ||
            cudaIpcGetEventHandle(&sh->ev_read[party][i], c->read[i]) != cudaSuccess) {
            c->sh->failed.store(1);  // the peer stops waiting on us
            delete c;
            return fail(DDG_ERR_CUDA, "IPC event creation / export failed%s", "");
        }
    }
    if (push) {
        // the flags block (zeroed before the peer can see it) and a pinned word for its error flag
        if (cudaMalloc(&c->flags, sizeof(PushFlags)) != cudaSuccess ||
            cudaMemset(c->flags, 0, sizeof(PushFlags)) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess ||
            cudaIpcGetMemHandle(&sh->flags[party], c->flags) != cudaSuccess ||
            cudaHostAlloc(reinterpret_cast<void **>(&c->h_err), sizeof(unsigned int), cudaHostAllocDefault) !=
                cudaSuccess) {
            c->sh->failed.store(1);  // the peer stops waiting on us
            delete c;
            return fail(DDG_ERR_CUDA, "IPC push flags allocation / export failed%s", "");
        }
        *c->h_err = 0;
        cudaDeviceGetAttribute(&c->push_blocks, cudaDevAttrMultiProcessorCount, device);
        if (device >= 0 && device < 64) {
            g_push_parties[device].fetch_add(1);
            c->counted = true;
        }
    }
    if (cudaDeviceGetPCIBusId(sh->bus_id[party], sizeof(sh->bus_id[party]), device) != cudaSuccess)
        sh->bus_id[party][0] = 0;
    if (party == 0) sh->slot_bytes = c->slot_bytes, sh->push = push ? 1u : 0u;
    sh->ready[party].store(1, std::memory_order_release);
    const auto t1 = std::chrono::steady_clock::now();
    while (!sh->ready[1 - party].load(std::memory_order_acquire)) {
        if (sh->failed.load() || std::chrono::steady_clock::now() - t1 > std::chrono::milliseconds(timeout_ms)) {
            c->sh->failed.store(1);  // the peer stops waiting on us
            delete c;
            return fail(DDG_ERR_PEER, "the peer party never joined the shared block %s", name);
        }
        std::this_thread::sleep_for(std::chrono::milliseconds(1));
    }
    if (sh->slot_bytes != c->slot_bytes || sh->push != (push ? 1u : 0u)) {
        c->sh->failed.store(1);  // the peer stops waiting on us
        delete c;
        return fail(DDG_ERR_ARG, "the two parties asked for different IPC slot sizes or modes%s", "");
    }
    if (push && std::strncmp(sh->bus_id[0], sh->bus_id[1], sizeof(sh->bus_id[0])) == 0) {
        c->sh->failed.store(1);
        delete c;
        return fail(DDG_ERR_ARG, "IPC push mode needs the two parties on different GPUs (both on %s)",
                    sh->bus_id[party]);
    }
    const int q = 1 - party;
    void *pa = nullptr;
    if (cudaIpcOpenMemHandle(&pa, sh->arena[q], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
        c->sh->failed.store(1);  // the peer stops waiting on us
        delete c;
        return fail(DDG_ERR_CUDA, "cannot map the peer's IPC arena (are both GPUs on this node?)%s", "");
    }
    c->peer_arena = static_cast<uint8_t *>(pa);
    if (push) {
        void *pf = nullptr;
        if (cudaIpcOpenMemHandle(&pf, sh->flags[q], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            c->sh->failed.store(1);
            delete c;
            return fail(DDG_ERR_CUDA, "cannot map the peer's IPC push flags%s", "");
        }
        c->peer_flags = static_cast<PushFlags *>(pf);
    }
    for (int i = 0; i < S; i++) {
        if (cudaIpcOpenEventHandle(&c->peer_posted[i], sh->ev_posted[q][i]) != cudaSuccess ||
            cudaIpcOpenEventHandle(&c->peer_read[i], sh->ev_read[q][i]) != cudaSuccess) {
            c->sh->failed.store(1);  // the peer stops waiting on us
            delete c;
            return fail(DDG_ERR_CUDA, "cannot open the peer's IPC events%s", "");
        }
    }
    *status = DDG_OK;
    return c;
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
