// Key chunks and the double-buffered key stream.
//
// Replaces the reference's chunked key file and streaming evaluation
// (gpu_mpc/deepdtagen_inference.cu:344-416 dealer pwrite of 4 KiB-padded
// chunks at ck*chunkKeySize; :608-826 I/O thread + 2 pinned + 2 VRAM slots +
// copy stream + evH2D/evFree events; patch setGPUKeyArenaSlot).
//
// Chunk = one forward's key region, then zero padding, then a 64-byte
// trailer, the whole rounded up to 4 KiB:
//   trailer: magic "DDGKEY01" | bw | scale | batch | chunk index | key bytes | checksum
// The checksum is a position-keyed 64-bit sum computed on the GPU
// (sum_i mix(word_i, i) mod 2^64, an order-free reduction); it detects
// truncated, shifted or corrupted chunks (storage and transfer errors).
//
// KeyStream: two device slots of one chunk each and a copy stream.  Before
// forward k the stream issues the H2D copy of chunk k+1 into the other slot
// (after the forward that last used that slot has finished: event wait on the
// copy stream), and the party's stream waits on chunk k's copy event; so the
// copy of the next chunk runs under the current forward.  Sources: a ring of
// pinned host chunks used cyclically (the timing discipline of the
// reference's benchmark, which rewinds its keys), or a key file read by an
// I/O thread with pread into two pinned staging buffers.
#include <fcntl.h>
#include <unistd.h>

#include <chrono>
#include <condition_variable>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "forward.cuh"
#include "gates.cuh"
#include "keystream.cuh"

namespace ddg {

static const char kMagic[8] = {'D', 'D', 'G', 'K', 'E', 'Y', '0', '1'};

uint64_t key_chunk_bytes(int bw, int s, int B)
{
    const uint64_t kb = forward_key_bytes(bw, s, B);
    return (kb + sizeof(ChunkTrailer) + 4095) & ~uint64_t(4095);
}

__global__ void k_checksum(const uint64_t *p, uint64_t nwords, unsigned long long *acc)
{
    uint64_t h = 0;
    for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < nwords; i += uint64_t(gridDim.x) * blockDim.x) {
        uint64_t w = __ldcs(p + i) ^ (i * 0x9E3779B97F4A7C15ull);
        w *= 0xBF58476D1CE4E5B9ull;
        w ^= w >> 31;
        h += w;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) h += __shfl_xor_sync(0xFFFFFFFFu, h, o);
    if ((threadIdx.x & 31) == 0) atomicAdd(acc, (unsigned long long)h);
}

int key_checksum(const void *d, uint64_t bytes, uint64_t *out, cudaStream_t st)
{
    DDG_CHECK(bytes % 8 == 0, DDG_ERR_ARG, "checksum length %llu not a multiple of 8", (unsigned long long)bytes);
    unsigned long long *acc = nullptr;
    DDG_CUDA(cudaMallocAsync(&acc, sizeof(*acc), st));
    DDG_CUDA(cudaMemsetAsync(acc, 0, sizeof(*acc), st));
    int sms = device_sms();
    k_checksum<<<sms * 8, 256, 0, st>>>(static_cast<const uint64_t *>(d), bytes / 8, acc);
    note_launch();
    DDG_CUDA(cudaGetLastError());
    unsigned long long h = 0;
    DDG_CUDA(cudaMemcpyAsync(&h, acc, sizeof(h), cudaMemcpyDeviceToHost, st));
    DDG_CUDA(cudaFreeAsync(acc, st));
    DDG_CUDA(cudaStreamSynchronize(st));
    *out = h;
    return DDG_OK;
}

int chunk_seal(void *d_chunk, int bw, int s, int B, uint64_t index, cudaStream_t st)
{
    const uint64_t kb = forward_key_bytes(bw, s, B), cb = key_chunk_bytes(bw, s, B);
    DDG_CUDA(cudaMemsetAsync(static_cast<uint8_t *>(d_chunk) + kb, 0, cb - kb, st));
    ChunkTrailer t;
    memcpy(t.magic, kMagic, 8);
    t.bw = uint32_t(bw), t.scale = uint32_t(s), t.batch = uint32_t(B), t.pad = 0;
    t.index = index, t.key_bytes = kb;
    DDG_TRY(key_checksum(d_chunk, kb, &t.checksum, st));
    DDG_CUDA(cudaMemcpyAsync(static_cast<uint8_t *>(d_chunk) + cb - sizeof(t), &t, sizeof(t), cudaMemcpyHostToDevice,
                             st));
    DDG_CUDA(cudaStreamSynchronize(st));
    return DDG_OK;
}

int check_trailer(const ChunkTrailer &t, int bw, int s, int B)
{
    DDG_CHECK(memcmp(t.magic, kMagic, 8) == 0, DDG_ERR_KEY, "key chunk has no DDGKEY01 trailer (truncated or not a key file)");
    DDG_CHECK(t.bw == uint32_t(bw) && t.scale == uint32_t(s) && t.batch == uint32_t(B), DDG_ERR_KEY,
              "key chunk is for bw=%u scale=%u batch=%u, expected %d/%d/%d", t.bw, t.scale, t.batch, bw, s, B);
    DDG_CHECK(t.key_bytes == forward_key_bytes(bw, s, B), DDG_ERR_KEY, "key chunk layout size mismatch");
    return DDG_OK;
}

int chunk_verify(const void *d_chunk, int bw, int s, int B, ChunkTrailer *out, cudaStream_t st)
{
    const uint64_t cb = key_chunk_bytes(bw, s, B);
    ChunkTrailer t;
    DDG_CUDA(cudaMemcpyAsync(&t, static_cast<const uint8_t *>(d_chunk) + cb - sizeof(t), sizeof(t),
                             cudaMemcpyDeviceToHost, st));
    DDG_CUDA(cudaStreamSynchronize(st));
    DDG_TRY(check_trailer(t, bw, s, B));
    uint64_t h = 0;
    DDG_TRY(key_checksum(d_chunk, t.key_bytes, &h, st));
    DDG_CHECK(h == t.checksum, DDG_ERR_KEY, "key chunk %llu checksum mismatch (corrupted keys)",
              (unsigned long long)t.index);
    if (out) *out = t;
    return DDG_OK;
}

// ---------------------------------------------------------------- KeyStream

KeyStream::~KeyStream()
{
    stop_io();
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(device);
    if (copy) cudaStreamSynchronize(copy);
    for (int s = 0; s < 2; s++) {
        if (d_slot[s]) cudaFree(d_slot[s]);
        if (staging[s]) cudaFreeHost(staging[s]);
        for (cudaEvent_t e : {ev_h2d[s], ev_free[s], ev_c0[s]})
            if (e) cudaEventDestroy(e);
    }
    if (copy) cudaStreamDestroy(copy);
    cudaSetDevice(prev);
}

int KeyStream::init(Party *p, int B_)
{
    P = p, B = B_, device = p->device;
    chunk = key_chunk_bytes(p->bw, p->s, B);
    DDG_CUDA(cudaSetDevice(device));
    DDG_CUDA(cudaStreamCreateWithFlags(&copy, cudaStreamNonBlocking));
    for (int s = 0; s < 2; s++) {
        DDG_CUDA(cudaMalloc(&d_slot[s], chunk));
        DDG_CUDA(cudaEventCreateWithFlags(&ev_free[s], cudaEventDisableTiming));
        DDG_CUDA(cudaEventCreate(&ev_h2d[s]));
        DDG_CUDA(cudaEventCreate(&ev_c0[s]));
        // both slots start free
        DDG_CUDA(cudaEventRecord(ev_free[s], copy));
    }
    return DDG_OK;
}

int KeyStream::open_file(const char *p, int nchunks)
{
    DDG_CHECK(nchunks > 0 && host.empty() && fd < 0, DDG_ERR_STATE, "key stream already has a source");
    fd = open(p, O_RDONLY);
    DDG_CHECK(fd >= 0, DDG_ERR_ARG, "cannot open key file %s", p);
    const off_t size = lseek(fd, 0, SEEK_END);
    DDG_CHECK(size >= off_t(chunk) * nchunks, DDG_ERR_KEY,
              "key file %s holds %lld bytes, %d chunks of %llu need %llu", p, (long long)size, nchunks,
              (unsigned long long)chunk, (unsigned long long)(chunk * uint64_t(nchunks)));
    file_chunks = nchunks;
    path = p;
    for (int s = 0; s < 2; s++) DDG_CUDA(cudaHostAlloc(&staging[s], chunk, cudaHostAllocDefault));
    io = std::thread([this] { io_loop(); });
    return DDG_OK;
}

void KeyStream::stop_io()
{
    {
        std::lock_guard<std::mutex> g(mu);
        quit = true;
    }
    cv.notify_all();
    if (io.joinable()) io.join();
    if (fd >= 0) close(fd);
    fd = -1;
}

// I/O thread: read chunk j (file order j mod nchunks) into staging[j % 2] once
// the copy that last read that staging buffer has completed
void KeyStream::io_loop()
{
    cudaSetDevice(device);
    for (uint64_t j = 0;; j++) {
        const int s = int(j & 1);
        {
            std::unique_lock<std::mutex> lk(mu);
            cv.wait(lk, [&] { return quit || j < 2 || consumed[s] >= int64_t(j) - 2; });
            if (quit) return;
        }
        // the H2D copy that read staging[s] (chunk j-2) must be complete
        if (j >= 2) cudaEventSynchronize(ev_h2d[s]);
        const off_t off = off_t(j % uint64_t(file_chunks)) * off_t(chunk);
        uint64_t done = 0;
        bool ok = true;
        auto t0 = std::chrono::steady_clock::now();
        while (done < chunk) {
            ssize_t r = pread(fd, static_cast<uint8_t *>(staging[s]) + done, chunk - done, off + off_t(done));
            if (r <= 0) {
                ok = false;
                break;
            }
            done += uint64_t(r);
        }
        const double ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
        {
            std::lock_guard<std::mutex> g(mu);
            read_ms += ms;
            if (!ok) io_error = true;
            staged_upto = int64_t(j);
        }
        cv.notify_all();
        if (!ok) return;
    }
}

// make chunk j's source available in host memory; returns its address
int KeyStream::source_of(uint64_t j, const void **src)
{
    if (!host.empty()) {
        *src = host[j % host.size()];
        return DDG_OK;
    }
    DDG_CHECK(fd >= 0, DDG_ERR_STATE, "key stream has no source (add host chunks or open a key file)");
    std::unique_lock<std::mutex> lk(mu);
    auto t0 = std::chrono::steady_clock::now();
    const bool ok = cv.wait_for(lk, std::chrono::milliseconds(timeout_ms),
                                [&] { return io_error || staged_upto >= int64_t(j); });
    wait_ms += std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    DDG_CHECK(!io_error, DDG_ERR_KEY, "reading key file %s failed (short read)", path.c_str());
    DDG_CHECK(ok, DDG_ERR_KEY, "key file reader did not deliver chunk %llu within %d ms", (unsigned long long)j,
              timeout_ms);
    *src = staging[j & 1];
    return DDG_OK;
}

int KeyStream::issue(uint64_t j)
{
    const int s = int(j & 1);
    const void *src = nullptr;
    DDG_TRY(source_of(j, &src));
    // the forward that used slot s (chunk j-2) must have finished
    DDG_CUDA(cudaStreamWaitEvent(copy, ev_free[s], 0));
    DDG_CUDA(cudaEventRecord(ev_c0[s], copy));
    DDG_CUDA(cudaMemcpyAsync(d_slot[s], src, chunk, cudaMemcpyHostToDevice, copy));
    DDG_CUDA(cudaEventRecord(ev_h2d[s], copy));
    if (fd >= 0) {
        std::lock_guard<std::mutex> g(mu);
        consumed[s] = int64_t(j);  // the I/O thread may refill staging[s] once this copy completes
    }
    cv.notify_all();
    issued = int64_t(j);
    bytes_copied += chunk;
    return DDG_OK;
}

// bind chunk k for the next forward: issue its copy (first call) and the next one
int KeyStream::begin_forward()
{
    DDG_CUDA(cudaSetDevice(device));
    const uint64_t k = next;
    if (issued < int64_t(k)) DDG_TRY(issue(k));
    DDG_TRY(issue(k + 1));
    const int s = int(k & 1);
    DDG_CUDA(cudaStreamWaitEvent(P->stream, ev_h2d[s], 0));
    if (verify) {
        DDG_CUDA(cudaStreamSynchronize(P->stream));
        ChunkTrailer t;
        DDG_TRY(chunk_verify(d_slot[s], P->bw, P->s, B, &t, P->stream));
    }
    P->keys = static_cast<const uint8_t *>(d_slot[s]);
    P->key_bytes = forward_key_bytes(P->bw, P->s, B);
    return DDG_OK;
}

int KeyStream::end_forward(int status)
{
    const int s = int(next & 1);
    cudaEventRecord(ev_free[s], P->stream);
    // copy duration of chunk k (its events completed before the forward used the slot)
    float ms = 0;
    if (cudaEventElapsedTime(&ms, ev_c0[s], ev_h2d[s]) == cudaSuccess) copy_ms += ms;
    next++;
    consumed_chunks++;
    P->keys = nullptr;
    P->key_bytes = 0;
    return status;
}

}  // namespace ddg
