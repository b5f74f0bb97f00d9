// Gate evaluation of both parties on one device without any device allocation.
//
// ddg_gate_eval_pair_noalloc runs the same kernels as two ddg_gate_round1 +
// ddg_gate_round2 calls per party followed by the opening, but the round-1
// bits and round-2 shares that those calls keep in caller-allocated buffers
// live here in one file-scope device array instead.  It serves callers that
// cannot call cudaMalloc: code embedded in a host framework that owns all
// device memory through its own allocator, code that must avoid the implicit
// device synchronisation cudaMalloc/cudaFree can trigger in the middle of a
// pipeline, and deployments whose device memory budget is fixed up front.
//
// Limits and sharing: at most DDG_NOALLOC_MAX_N elements per call.  Every
// GPU that loads the library holds the array (4,325,376 bytes = 4.125 MiB:
// 4 x 8,192 bit words, then two shares of 262,144 64-bit words) until the process
// exits.  All calls share it and it keeps the last call's contents; each call
// overwrites every word it reads, so nothing needs clearing, but calls that
// overlap on the GPU (different streams, or different host threads on one
// device) race on it.  The first call on a device looks up the array's device
// address (cudaGetSymbolAddress) and uploads the AES tables; make that first
// call before any stream capture.
#include <mutex>

#include "aes_dev.cuh"
#include "gates.cuh"
#include "linear.cuh"

using namespace ddg;

namespace {

constexpr uint64_t kMaxN = DDG_NOALLOC_MAX_N;
constexpr uint64_t kWords = (kMaxN + 31) / 32;
constexpr uint64_t kBitBytes = 4 * kWords * sizeof(uint32_t);  // own/peer bits of both DCFs, both parties
constexpr uint64_t kShareBytes = kMaxN * sizeof(uint64_t);      // one party's share, widest ring
constexpr uint64_t kScratchBytes = kBitBytes + 2 * kShareBytes;

static __device__ __align__(256) uint8_t g_noalloc_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void *g_scratch_addr[kMaxDevices] = {};

// device address of the scratch array on the current device (looked up once per device)
int scratch_address(void **out)
{
    int dev = 0;
    DDG_CUDA(cudaGetDevice(&dev));
    DDG_CHECK(dev >= 0 && dev < kMaxDevices, DDG_ERR_ARG, "device ordinal %d out of range", dev);
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_scratch_addr[dev]) {
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        DDG_CHECK(e == cudaSuccess && p, DDG_ERR_CUDA, "cudaGetSymbolAddress(no-allocation scratch): %s",
                  cudaGetErrorString(e));
        g_scratch_addr[dev] = p;
    }
    *out = g_scratch_addr[dev];
    return DDG_OK;
}

}  // namespace

extern "C" int ddg_gate_eval_pair_noalloc(int kind, int bw, int scale, uint64_t n, const void *d_xhat,
                                          const void *d_key0, const void *d_key1, void *d_yhat, void *stream)
{
    DDG_CHECK(kind >= DDG_GATE_RELU && kind <= DDG_GATE_LRS, DDG_ERR_ARG,
              "gate kind %d out of range for the no-allocation entry point (0..3)", kind);
    DDG_CHECK(bw == 32 || bw == 64, DDG_ERR_ARG, "bw must be 32 or 64 (got %d)", bw);
    DDG_CHECK(scale >= 1 && scale < bw - 1, DDG_ERR_ARG, "scale %d out of range for bw %d", scale, bw);
    DDG_CHECK(n <= kMaxN, DDG_ERR_ARG,
              "n = %llu exceeds the no-allocation limit of %llu elements per call (DDG_NOALLOC_MAX_N)",
              (unsigned long long)n, (unsigned long long)kMaxN);
    if (n == 0) return DDG_OK;
    DDG_CHECK(d_xhat && d_key0 && d_key1 && d_yhat, DDG_ERR_ARG, "null pointer");
    void *base = nullptr;
    DDG_TRY(scratch_address(&base));
    auto *bits = static_cast<uint32_t *>(base);
    uint32_t *hi0 = bits, *lo0 = bits + kWords, *hi1 = bits + 2 * kWords, *lo1 = bits + 3 * kWords;
    uint8_t *sh0 = static_cast<uint8_t *>(base) + kBitBytes;
    uint8_t *sh1 = sh0 + kShareBytes;
    auto st = static_cast<cudaStream_t>(stream);
    const GateLayout L = gate_layout(kind, bw, scale, n);
    DDG_TRY(gate_round1(L, d_xhat, d_key0, hi0, lo0, st));
    DDG_TRY(gate_round1(L, d_xhat, d_key1, hi1, lo1, st));
    DDG_TRY(gate_round2(L, 0, d_xhat, hi0, hi1, lo0, lo1, d_key0, sh0, st));
    DDG_TRY(gate_round2(L, 1, d_xhat, hi1, hi0, lo1, lo0, d_key1, sh1, st));
    if (bw == 32)
        return ew_add<uint32_t>(static_cast<uint32_t *>(d_yhat), reinterpret_cast<const uint32_t *>(sh0),
                                reinterpret_cast<const uint32_t *>(sh1), n, st);
    return ew_add<uint64_t>(static_cast<uint64_t *>(d_yhat), reinterpret_cast<const uint64_t *>(sh0),
                            reinterpret_cast<const uint64_t *>(sh1), n, st);
}
