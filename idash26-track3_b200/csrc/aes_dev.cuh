// AES-128 for sm_100a: bank-conflict-free T-table rounds in shared memory.
//
// One thread encrypts one 16-byte block held as four little-endian 32-bit
// column words (word c = bytes 4c..4c+3).  A full round of column c is
//   T0[b0(w_c)] ^ T1[b1(w_c+1)] ^ T2[b2(w_c+2)] ^ T3[b3(w_c+3)] ^ rk
// with T0[x] = (2S, S, S, 3S) bytes and Tk = rotl(T0, 8k).  Every table is
// replicated 32 times, lane l reading copy l, so a warp-wide lookup hits 32
// distinct banks; the row/lane byte address is formed by one PRMT.
//
// Two engines share that scheme:
// * AesLaneT<2> stages T0 and T2 (64 KiB: 256 rows of 32 x T0 | 32 x T2)
//   and forms T1 ^ T3 as one 8-bit rotation of T0 ^ T2: 8 integer-pipe
//   instructions per column, three 256-thread CTAs per SM.
// * AesLaneT<4> stages all four tables (128 KiB: rows of 32 x T0 | 32 x T1,
//   then rows of 32 x T2 | 32 x T3 at +64 KiB, the region bit carried in byte 2
//   of the lane offset so one PRMT still forms the address): 6 integer-pipe
//   instructions per column, one 768-thread CTA per SM.
// The last round takes S(x) out of T0/T2 bytes (T2 byte 0 = T0 byte 1 = S).
// An earlier measured variant that moved the rotations onto integer
// multiply-adds ran slower on B200 (38.8 vs 46.4 G blocks/s) and was dropped.
#pragma once
#include <cstdint>

namespace ddg {

struct AesKey {
    uint32_t rk[44];
};

// fixed public keys of the tree hash and the leaf conversion
struct FixedKeys {
    AesKey h;
    AesKey c;
};

extern __constant__ FixedKeys c_fixed;   // defined in aes_tables.cu
extern __device__ uint32_t g_T0[256];    // global copy, staged into shared memory per CTA

struct Blk {
    uint32_t w[4];
};

template <int NT>
struct AesLaneT {
    static_assert(NT == 2 || NT == 4, "2 or 4 staged tables");
    static constexpr int SMEM = NT * 32 * 1024;   // dynamic shared memory per CTA
    static constexpr int THREADS = NT == 4 ? 768 : 256;
    static constexpr int CTAS = NT == 4 ? 1 : 3;  // resident CTAs per SM the launch bounds target

    const char *tab;  // shared table base (generic pointer to shared memory)
    uint32_t o0, o1, o2, o3;  // per-table lane offsets (o1, o3 unused with two tables)

    __device__ __forceinline__ AesLaneT(const void *smem)
    {
        tab = reinterpret_cast<const char *>(smem);
        const uint32_t lane4 = (threadIdx.x & 31) * 4u;
        o0 = lane4;
        if (NT == 4) {
            o1 = 128u + lane4, o2 = 0x10000u | lane4, o3 = 0x10000u | (128u + lane4);
        } else {
            o1 = 0, o2 = 128u + lane4, o3 = 0;
        }
    }

    // fill the shared tables (every thread of the CTA, then a barrier)
    static __device__ __forceinline__ void stage(uint32_t *smem_words)
    {
        for (int i = threadIdx.x; i < NT * 8192; i += blockDim.x) {
            const int region = i >> 14, j = i & 16383, x = j >> 6, slot = j & 63;
            const uint32_t t0 = g_T0[x];
            const int rot = NT == 4 ? 16 * region + (slot < 32 ? 0 : 8) : (slot < 32 ? 0 : 16);
            smem_words[i] = __funnelshift_l(t0, t0, rot);
        }
    }

    // table word for byte k of w: byte address = byte0 of o | (w.byte k) << 8 | byte2 of o << 16
    __device__ __forceinline__ uint32_t look(uint32_t w, int k, uint32_t o) const
    {
        return *reinterpret_cast<const uint32_t *>(tab + __byte_perm(w, o, 0x7604u | (uint32_t(k) << 4)));
    }

    __device__ __forceinline__ void encrypt(Blk &b, const uint32_t *__restrict__ rk) const
    {
        uint32_t s0 = b.w[0] ^ rk[0], s1 = b.w[1] ^ rk[1], s2 = b.w[2] ^ rk[2], s3 = b.w[3] ^ rk[3];
#pragma unroll
        for (int r = 1; r < 10; r++) {
            uint32_t u0, u1, u2, u3;
            if (NT == 4) {
                u0 = look(s0, 0, o0) ^ look(s1, 1, o1) ^ look(s2, 2, o2) ^ look(s3, 3, o3) ^ rk[4 * r + 0];
                u1 = look(s1, 0, o0) ^ look(s2, 1, o1) ^ look(s3, 2, o2) ^ look(s0, 3, o3) ^ rk[4 * r + 1];
                u2 = look(s2, 0, o0) ^ look(s3, 1, o1) ^ look(s0, 2, o2) ^ look(s1, 3, o3) ^ rk[4 * r + 2];
                u3 = look(s3, 0, o0) ^ look(s0, 1, o1) ^ look(s1, 2, o2) ^ look(s2, 3, o3) ^ rk[4 * r + 3];
            } else {
                uint32_t v0 = look(s1, 1, o0) ^ look(s3, 3, o2);
                u0 = look(s0, 0, o0) ^ look(s2, 2, o2) ^ rk[4 * r + 0] ^ __funnelshift_l(v0, v0, 8);
                uint32_t v1 = look(s2, 1, o0) ^ look(s0, 3, o2);
                u1 = look(s1, 0, o0) ^ look(s3, 2, o2) ^ rk[4 * r + 1] ^ __funnelshift_l(v1, v1, 8);
                uint32_t v2 = look(s3, 1, o0) ^ look(s1, 3, o2);
                u2 = look(s2, 0, o0) ^ look(s0, 2, o2) ^ rk[4 * r + 2] ^ __funnelshift_l(v2, v2, 8);
                uint32_t v3 = look(s0, 1, o0) ^ look(s2, 3, o2);
                u3 = look(s3, 0, o0) ^ look(s1, 2, o2) ^ rk[4 * r + 3] ^ __funnelshift_l(v3, v3, 8);
            }
            s0 = u0, s1 = u1, s2 = u2, s3 = u3;
        }
        // last round: SubBytes + ShiftRows + AddRoundKey
        // column c bytes: S(b0(s_c)), S(b1(s_c+1)), S(b2(s_c+2)), S(b3(s_c+3))
        auto last = [&](uint32_t a, uint32_t bb, uint32_t c, uint32_t d) {
            uint32_t lo = __byte_perm(look(a, 0, o2), look(bb, 1, o0), 0x3250u);  // byte0 = T2 b0, byte1 = T0 b1
            uint32_t hi = __byte_perm(look(c, 2, o0), look(d, 3, o2), 0x7210u);   // byte2 = T0 b2, byte3 = T2 b3
            return __byte_perm(lo, hi, 0x7610u);
        };
        b.w[0] = last(s0, s1, s2, s3) ^ rk[40];
        b.w[1] = last(s1, s2, s3, s0) ^ rk[41];
        b.w[2] = last(s2, s3, s0, s1) ^ rk[42];
        b.w[3] = last(s3, s0, s1, s2) ^ rk[43];
    }

    // correlation-robust hash pi(sigma(x)) ^ sigma(x), sigma(lo,hi) = (hi, lo^hi)
    __device__ __forceinline__ Blk ccr(const Blk &x, const uint32_t *__restrict__ rk) const
    {
        Blk s;
        s.w[0] = x.w[2];
        s.w[1] = x.w[3];
        s.w[2] = x.w[0] ^ x.w[2];
        s.w[3] = x.w[1] ^ x.w[3];
        Blk e = s;
        encrypt(e, rk);
        e.w[0] ^= s.w[0], e.w[1] ^= s.w[1], e.w[2] ^= s.w[2], e.w[3] ^= s.w[3];
        return e;
    }
    __device__ __forceinline__ Blk hash_h(const Blk &x) const { return ccr(x, c_fixed.h.rk); }
    __device__ __forceinline__ Blk hash_c(const Blk &x) const { return ccr(x, c_fixed.c.rk); }

    // dealer PRG block AES_K(idx || op || purpose)
    __device__ __forceinline__ Blk prg(const uint32_t *__restrict__ rk, uint32_t op, uint32_t purpose, uint64_t idx) const
    {
        Blk b;
        b.w[0] = uint32_t(idx);
        b.w[1] = uint32_t(idx >> 32);
        b.w[2] = op;
        b.w[3] = purpose;
        encrypt(b, rk);
        return b;
    }
};

using AesLane2 = AesLaneT<2>;
using AesLane4 = AesLaneT<4>;

// the engine the library's AES kernels launch with (process-wide; 2 or 4
// staged tables).  aes_tables.cu holds the setting.
int aes_tables();
void set_aes_tables(int nt);

int device_sms();  // gates.cu

// CTAs of an AES kernel over engine E with `threads` threads of work:
// min(ceil(threads / E::THREADS), SMs x E::CTAS), at least 1
template <class E>
inline int aes_blocks(uint64_t threads)
{
    int sms = device_sms();
    if (sms <= 0) sms = 148;
    const uint64_t need = (threads + E::THREADS - 1) / E::THREADS, full = uint64_t(sms) * E::CTAS;
    return int(need < full ? (need ? need : 1) : full);
}

__device__ __forceinline__ Blk blk_xor(const Blk &a, const Blk &b)
{
    Blk r;
    r.w[0] = a.w[0] ^ b.w[0], r.w[1] = a.w[1] ^ b.w[1], r.w[2] = a.w[2] ^ b.w[2], r.w[3] = a.w[3] ^ b.w[3];
    return r;
}

__device__ __forceinline__ Blk blk_and_mask(const Blk &a, uint32_t m)
{
    Blk r;
    r.w[0] = a.w[0] & m, r.w[1] = a.w[1] & m, r.w[2] = a.w[2] & m, r.w[3] = a.w[3] & m;
    return r;
}

__device__ __forceinline__ Blk ld_blk_stream(const void *p)
{
    uint4 v = __ldcs(reinterpret_cast<const uint4 *>(p));
    Blk b;
    b.w[0] = v.x, b.w[1] = v.y, b.w[2] = v.z, b.w[3] = v.w;
    return b;
}

__device__ __forceinline__ void st_blk(void *p, const Blk &b)
{
    *reinterpret_cast<uint4 *>(p) = make_uint4(b.w[0], b.w[1], b.w[2], b.w[3]);
}

__device__ __forceinline__ int blk_bit(const Blk &b, uint32_t y)
{
    // select the word without dynamic register indexing (which would spill to local memory)
    const uint32_t q = y >> 5;
    const uint32_t lo = q & 1u ? b.w[1] : b.w[0];
    const uint32_t hi = q & 1u ? b.w[3] : b.w[2];
    return ((q & 2u ? hi : lo) >> (y & 31)) & 1;
}

// host side (aes_tables.cu)
void aes_expand_host(const uint8_t key[16], AesKey &out);
void aes_encrypt_host(const AesKey &k, const uint32_t in[4], uint32_t out[4]);
void aes_host_init();
AesKey dealer_key(uint64_t seed);
int aes_device_init();
const char *last_error();

}  // namespace ddg
