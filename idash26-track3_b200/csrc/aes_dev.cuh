// AES-128 for sm_100a: bank-conflict-free T-table rounds in shared memory.
//
// One thread encrypts one 16-byte block held as four little-endian 32-bit
// column words (word c = bytes 4c..4c+3).  A full round of column c is
//   T0[b0(w_c)] ^ T2[b2(w_c+2)] ^ rotl8(T0[b1(w_c+1)] ^ T2[b3(w_c+3)]) ^ rk
// with T0[x] = (2S, S, S, 3S) bytes and T2 = rotl16(T0).  The shared table
// holds 256 rows of 256 bytes: 32 copies of T0[x] then 32 copies of T2[x],
// lane l reading copy l, so every warp-wide lookup hits 32 distinct banks.
// The row/lane byte address (x << 8) | laneoff is formed by one PRMT.
// The last round takes S(x) out of T0/T2 bytes (T2 byte 0 = T0 byte 1 = S).
#pragma once
#include <cstdint>

// DDG_AES_IMAD = 1 moves the byte-3 table addresses and the 8-bit rotations
// from the integer ALU pipe to integer multiply-adds.  Measured on B200 with the
// ddg_aes_chain_variant probe it is slower (38.8 vs 46.4 G blocks/s), so the
// ALU form (PRMT / funnel shift) is the default.
#ifndef DDG_AES_IMAD
#define DDG_AES_IMAD 0
#endif

namespace ddg {

constexpr int AES_SMEM_BYTES = 256 * 256;

struct AesKey {
    uint32_t rk[44];
};

// fixed public keys of the tree hash and the leaf conversion; `m256` holds
// the constant 256, read from constant memory so that multiplies by it stay
// integer multiply-adds (FMA pipe) instead of being folded into shifts (ALU pipe)
struct FixedKeys {
    AesKey h;
    AesKey c;
    uint32_t m256;
};

extern __constant__ FixedKeys c_fixed;   // defined in aes_tables.cu
extern __device__ uint32_t g_T0[256];    // global copy, staged into shared memory per CTA

struct Blk {
    uint32_t w[4];
};

// Fill the 64 KiB shared table: row x = 32 x T0[x] then 32 x T2[x].
__device__ __forceinline__ void aes_stage_tables(uint32_t *smem_words)
{
    for (int i = threadIdx.x; i < 256 * 64; i += blockDim.x) {
        int x = i >> 6, slot = i & 63;
        uint32_t t0 = g_T0[x];
        smem_words[i] = slot < 32 ? t0 : __funnelshift_l(t0, t0, 16);
    }
}

struct AesLane {
    const char *tab;   // shared table base (generic pointer to shared memory)
    uint32_t off0;     // 4*lane        : T0 copy of this lane
    uint32_t off2;     // 128 + 4*lane  : T2 copy of this lane
    __device__ __forceinline__ AesLane(const void *smem)
    {
        tab = reinterpret_cast<const char *>(smem);
        uint32_t lane = threadIdx.x & 31;
        off0 = lane * 4u;
        off2 = 128u + lane * 4u;
    }
    // table word at byte k of w: byte address ((w >> 8k) & 0xff) << 8 | off
    __device__ __forceinline__ uint32_t t0(uint32_t w, int k) const
    {
        return *reinterpret_cast<const uint32_t *>(tab + __byte_perm(w, off0, 0x5504u | (uint32_t(k) << 4)));
    }
    __device__ __forceinline__ uint32_t t2(uint32_t w, int k) const
    {
        return *reinterpret_cast<const uint32_t *>(tab + __byte_perm(w, off2, 0x5504u | (uint32_t(k) << 4)));
    }

    // T2 lookup of byte 3 with the address formed on the FMA pipe:
    // ((w * 2^-24) >> 0) * 256 + off = umulhi(w, 256) * 256 + off
    __device__ __forceinline__ uint32_t t2_b3_fma(uint32_t w) const
    {
        const uint32_t m = c_fixed.m256;
        return *reinterpret_cast<const uint32_t *>(tab + (__umulhi(w, m) * m + off2));
    }
    // rotl8 on the FMA pipe: v * 256 + (v >> 24)
    __device__ __forceinline__ uint32_t rot8_fma(uint32_t v) const
    {
        const uint32_t m = c_fixed.m256;
        return v * m + __umulhi(v, m);
    }

    // IMAD = true: the byte-3 lookups and the rotations use integer multiply-adds
    template <bool IMAD = DDG_AES_IMAD>
    __device__ __forceinline__ void encrypt(Blk &b, const uint32_t *__restrict__ rk) const
    {
        uint32_t s0 = b.w[0] ^ rk[0], s1 = b.w[1] ^ rk[1], s2 = b.w[2] ^ rk[2], s3 = b.w[3] ^ rk[3];
#pragma unroll
        for (int r = 1; r < 10; r++) {
            uint32_t u0, u1, u2, u3;
            if (IMAD) {
                uint32_t v0 = t0(s1, 1) ^ t2_b3_fma(s3);
                u0 = t0(s0, 0) ^ t2(s2, 2) ^ rk[4 * r + 0] ^ rot8_fma(v0);
                uint32_t v1 = t0(s2, 1) ^ t2_b3_fma(s0);
                u1 = t0(s1, 0) ^ t2(s3, 2) ^ rk[4 * r + 1] ^ rot8_fma(v1);
                uint32_t v2 = t0(s3, 1) ^ t2_b3_fma(s1);
                u2 = t0(s2, 0) ^ t2(s0, 2) ^ rk[4 * r + 2] ^ rot8_fma(v2);
                uint32_t v3 = t0(s0, 1) ^ t2_b3_fma(s2);
                u3 = t0(s3, 0) ^ t2(s1, 2) ^ rk[4 * r + 3] ^ rot8_fma(v3);
            } else {
                uint32_t v0 = t0(s1, 1) ^ t2(s3, 3);
                u0 = t0(s0, 0) ^ t2(s2, 2) ^ rk[4 * r + 0] ^ __funnelshift_l(v0, v0, 8);
                uint32_t v1 = t0(s2, 1) ^ t2(s0, 3);
                u1 = t0(s1, 0) ^ t2(s3, 2) ^ rk[4 * r + 1] ^ __funnelshift_l(v1, v1, 8);
                uint32_t v2 = t0(s3, 1) ^ t2(s1, 3);
                u2 = t0(s2, 0) ^ t2(s0, 2) ^ rk[4 * r + 2] ^ __funnelshift_l(v2, v2, 8);
                uint32_t v3 = t0(s0, 1) ^ t2(s2, 3);
                u3 = t0(s3, 0) ^ t2(s1, 2) ^ rk[4 * r + 3] ^ __funnelshift_l(v3, v3, 8);
            }
            s0 = u0, s1 = u1, s2 = u2, s3 = u3;
        }
        // last round: SubBytes + ShiftRows + AddRoundKey
        // column c bytes: S(b0(s_c)), S(b1(s_c+1)), S(b2(s_c+2)), S(b3(s_c+3))
        auto last = [&](uint32_t a, uint32_t bb, uint32_t c, uint32_t d) {
            uint32_t lo = __byte_perm(t2(a, 0), t0(bb, 1), 0x3250u);  // byte0 = T2 b0, byte1 = T0 b1
            uint32_t hi = __byte_perm(t0(c, 2), IMAD ? t2_b3_fma(d) : t2(d, 3), 0x7210u);  // byte2 = T0 b2, byte3 = T2 b3
            return __byte_perm(lo, hi, 0x7610u);
        };
        b.w[0] = last(s0, s1, s2, s3) ^ rk[40];
        b.w[1] = last(s1, s2, s3, s0) ^ rk[41];
        b.w[2] = last(s2, s3, s0, s1) ^ rk[42];
        b.w[3] = last(s3, s0, s1, s2) ^ rk[43];
    }

    // correlation-robust hash pi(sigma(x)) ^ sigma(x), sigma(lo,hi) = (hi, lo^hi)
    template <bool IMAD = DDG_AES_IMAD>
    __device__ __forceinline__ Blk ccr(const Blk &x, const uint32_t *__restrict__ rk) const
    {
        Blk s;
        s.w[0] = x.w[2];
        s.w[1] = x.w[3];
        s.w[2] = x.w[0] ^ x.w[2];
        s.w[3] = x.w[1] ^ x.w[3];
        Blk e = s;
        encrypt<IMAD>(e, rk);
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
void aes_host_init();
AesKey dealer_key(uint64_t seed);
int aes_device_init();
const char *last_error();

}  // namespace ddg
