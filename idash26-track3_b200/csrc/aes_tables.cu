// Host-side AES-128 material (S-box from the GF(2^8) inverse and affine map,
// the T0 table, FIPS-197 key expansion) and its per-device upload.
#include <atomic>
#include <cstdarg>
#include <cstring>
#include <mutex>
#include <vector>

#include "aes_dev.cuh"
#include "common.cuh"

namespace ddg {

__constant__ FixedKeys c_fixed;
__device__ uint32_t g_T0[256];

static std::atomic<int> g_aes_tables{4};
int aes_tables() { return g_aes_tables.load(); }
void set_aes_tables(int nt) { g_aes_tables.store(nt == 2 ? 2 : 4); }

static uint8_t h_sbox[256];
static uint32_t h_T0[256];
static FixedKeys h_fixed;
static std::once_flag h_once;

static uint8_t xt(uint8_t a) { return uint8_t((a << 1) ^ ((a & 0x80) ? 0x1b : 0)); }
static uint8_t gf_mul(uint8_t a, uint8_t b)
{
    uint8_t p = 0;
    for (; b; b >>= 1, a = xt(a))
        if (b & 1) p ^= a;
    return p;
}

static void host_tables()
{
    for (int x = 0; x < 256; x++) {
        uint8_t inv = 0;
        if (x) {  // x^254 = x^-1
            uint8_t r = 1, base = uint8_t(x);
            for (int e = 254; e; e >>= 1, base = gf_mul(base, base))
                if (e & 1) r = gf_mul(r, base);
            inv = r;
        }
        uint8_t s = inv;
        for (int k = 1; k <= 4; k++) s ^= uint8_t((inv << k) | (inv >> (8 - k)));
        h_sbox[x] = uint8_t(s ^ 0x63);
    }
    for (int x = 0; x < 256; x++) {
        uint8_t s = h_sbox[x];
        h_T0[x] = uint32_t(gf_mul(s, 2)) | (uint32_t(s) << 8) | (uint32_t(s) << 16) | (uint32_t(gf_mul(s, 3)) << 24);
    }
    aes_expand_host(reinterpret_cast<const uint8_t *>("ddg-halftree-H:0"), h_fixed.h);
    aes_expand_host(reinterpret_cast<const uint8_t *>("ddg-halftree-C:1"), h_fixed.c);
}

void aes_expand_host(const uint8_t key[16], AesKey &out)
{
    uint8_t w[176];
    memcpy(w, key, 16);
    uint8_t rcon = 1;
    for (int i = 4; i < 44; i++) {
        uint8_t t[4];
        memcpy(t, w + 4 * (i - 1), 4);
        if (i % 4 == 0) {
            uint8_t t0 = t[0];
            t[0] = uint8_t(h_sbox[t[1]] ^ rcon);
            t[1] = h_sbox[t[2]];
            t[2] = h_sbox[t[3]];
            t[3] = h_sbox[t0];
            rcon = xt(rcon);
        }
        for (int k = 0; k < 4; k++) w[4 * i + k] = uint8_t(w[4 * (i - 4) + k] ^ t[k]);
    }
    for (int i = 0; i < 44; i++)
        out.rk[i] = uint32_t(w[4 * i]) | (uint32_t(w[4 * i + 1]) << 8) | (uint32_t(w[4 * i + 2]) << 16) |
                    (uint32_t(w[4 * i + 3]) << 24);
}

void aes_host_init() { std::call_once(h_once, host_tables); }

// FIPS-197 encryption of one block (column words, little-endian bytes)
void aes_encrypt_host(const AesKey &k, const uint32_t in[4], uint32_t out[4])
{
    aes_host_init();
    uint8_t st[16], t[16];
    auto add_key = [&](int r) {
        for (int i = 0; i < 16; i++) st[i] ^= uint8_t(k.rk[4 * r + i / 4] >> (8 * (i % 4)));
    };
    for (int i = 0; i < 16; i++) st[i] = uint8_t(in[i / 4] >> (8 * (i % 4)));
    add_key(0);
    for (int r = 1; r <= 10; r++) {
        for (int c = 0; c < 4; c++)  // SubBytes + ShiftRows: row j of column c comes from column c + j
            for (int j = 0; j < 4; j++) t[4 * c + j] = h_sbox[st[4 * ((c + j) % 4) + j]];
        if (r < 10) {
            for (int c = 0; c < 4; c++) {  // MixColumns
                const uint8_t a0 = t[4 * c], a1 = t[4 * c + 1], a2 = t[4 * c + 2], a3 = t[4 * c + 3];
                st[4 * c] = uint8_t(xt(a0) ^ xt(a1) ^ a1 ^ a2 ^ a3);
                st[4 * c + 1] = uint8_t(a0 ^ xt(a1) ^ xt(a2) ^ a2 ^ a3);
                st[4 * c + 2] = uint8_t(a0 ^ a1 ^ xt(a2) ^ xt(a3) ^ a3);
                st[4 * c + 3] = uint8_t(xt(a0) ^ a0 ^ a1 ^ a2 ^ xt(a3));
            }
        } else {
            memcpy(st, t, 16);
        }
        add_key(r);
    }
    for (int c = 0; c < 4; c++)
        out[c] = uint32_t(st[4 * c]) | (uint32_t(st[4 * c + 1]) << 8) | (uint32_t(st[4 * c + 2]) << 16) |
                 (uint32_t(st[4 * c + 3]) << 24);
}

// dealer key: seed (8 bytes LE) || "dealerK1"
AesKey dealer_key(uint64_t seed)
{
    aes_host_init();
    uint8_t k[16];
    for (int i = 0; i < 8; i++) k[i] = uint8_t(seed >> (8 * i));
    memcpy(k + 8, "dealerK1", 8);
    AesKey out;
    aes_expand_host(k, out);
    return out;
}

// Upload the tables to the current device once per device.
int aes_device_init()
{
    aes_host_init();
    static std::mutex mu;
    static std::vector<int> done;
    int dev = 0;
    DDG_CUDA(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> g(mu);
    if (dev >= int(done.size())) done.resize(dev + 1, 0);
    if (done[dev]) return DDG_OK;
    DDG_CUDA(cudaMemcpyToSymbol(c_fixed, &h_fixed, sizeof(h_fixed)));
    DDG_CUDA(cudaMemcpyToSymbol(g_T0, h_T0, sizeof(h_T0)));
    done[dev] = 1;
    return DDG_OK;
}

// ----------------------------------------------------------------- counters

static std::atomic<uint64_t> g_launches{0};
void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
uint64_t launch_count() { return g_launches.load(); }
void add_launches(uint64_t n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

int record_timing_event(cudaEvent_t e, cudaStream_t st)
{
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    DDG_CUDA(cudaStreamIsCapturing(st, &cs));
    if (cs == cudaStreamCaptureStatusActive) {
        DDG_CUDA(cudaEventRecordWithFlags(e, st, cudaEventRecordExternal));
    } else {
        DDG_CUDA(cudaEventRecord(e, st));
    }
    return DDG_OK;
}

static thread_local DcfTiming *t_dcf_sink = nullptr;
DcfTiming *dcf_timing_sink() { return t_dcf_sink; }
void set_dcf_timing_sink(DcfTiming *t) { t_dcf_sink = t; }

int DcfTiming::take(cudaEvent_t *e)
{
    if (used == pool.size()) {
        cudaEvent_t n = nullptr;
        DDG_CUDA(cudaEventCreate(&n));
        pool.push_back(n);
    }
    *e = pool[used++];
    return DDG_OK;
}

void DcfTiming::release()
{
    for (cudaEvent_t e : pool) cudaEventDestroy(e);
    pool.clear(), recs.clear(), used = 0;
}

int TimedLaunch::begin(cudaStream_t st)
{
    DcfTiming *tm = t_dcf_sink;
    if (!tm || !tm->enabled) return DDG_OK;
    DcfTiming::Rec r{};
    DDG_TRY(tm->take(&r.a));
    DDG_TRY(tm->take(&r.b));
    DDG_TRY(record_timing_event(r.a, st));
    tm->recs.push_back(r);
    sink = tm, idx = tm->recs.size() - 1;
    return DDG_OK;
}

int TimedLaunch::end(cudaStream_t st, double bytes, double aes, double evals)
{
    if (!sink) return DDG_OK;
    DcfTiming::Rec &r = sink->recs[idx];
    DDG_TRY(record_timing_event(r.b, st));
    r.bytes = bytes, r.aes = aes, r.evals = evals, r.done = true;
    return DDG_OK;
}

// ----------------------------------------------------------------- errors

static thread_local char t_err[512] = "";

void set_last_error(const char *fmt, ...)
{
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(t_err, sizeof(t_err), fmt, ap);
    va_end(ap);
}

const char *last_error() { return t_err; }

}  // namespace ddg
