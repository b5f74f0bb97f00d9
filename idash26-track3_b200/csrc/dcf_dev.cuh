// Half-tree DCF on the device: evaluation (one party, one element per
// thread) and dealer key generation (both parties).
//
// Scheme: on-path seeds of the two parties differ by Delta (lsb 1), the control
// bit is lsb(seed), children are cL = H(s) ^ t*CW_j and cR = cL ^ s.  The
// comparison 1{x < alpha} is the XOR of lsb(cR) at every level where x goes
// left, plus bit (x mod 2^lb) of the leaf Conv(s) ^ t*CW_leaf, lb = min(d, 7).
#pragma once
#include "aes_dev.cuh"
#include "common.cuh"

namespace ddg {

// Party's XOR share of 1{x < alpha} for d-bit x.  Key arrays are read once
// with streaming loads; the next level's correction word is fetched one level
// ahead so its latency hides under the current level's AES.
template <class E>
__device__ __forceinline__ uint32_t dcf_eval(const E &A, uint64_t x, int d, const DcfView &k, uint64_t e,
                                             uint64_t N)
{
    const int L = d > 7 ? d - 7 : 0;
    Blk s = ld_blk_stream(k.root + 16 * e);
    uint32_t c = 0;
    const uint8_t *cwp = k.cw + 16 * e;
    const uint64_t stride = 16 * N;
    Blk nxt;
    if (L > 0) nxt = ld_blk_stream(cwp);
#pragma unroll 1
    for (int j = 0; j < L; j++) {
        Blk cw = nxt;
        if (j + 1 < L) nxt = ld_blk_stream(cwp + stride * uint64_t(j + 1));
        uint32_t xj = uint32_t(x >> (d - 1 - j)) & 1u;
        uint32_t tm = 0u - (s.w[0] & 1u);
        Blk cl = blk_xor(A.hash_h(s), blk_and_mask(cw, tm));
        c ^= (xj ^ 1u) & ((cl.w[0] ^ s.w[0]) & 1u);
        s = blk_xor(cl, blk_and_mask(s, 0u - xj));
    }
    uint32_t tm = 0u - (s.w[0] & 1u);
    Blk lf = ld_blk_stream(k.leaf + 16 * e);
    Blk g = blk_xor(A.hash_c(s), blk_and_mask(lf, tm));
    const int lb = d - L;
    c ^= uint32_t(blk_bit(g, uint32_t(x) & ((1u << lb) - 1u)));
    return c;
}

// DCF with equality output: returns the party's XOR shares of 1{x < alpha}
// (bit 0) and 1{x == alpha} (bit 1) for d-bit x; the leaf holds, for the low
// min(d, 6) bits y of x, 1{y < alpha_low} at bit 2y and 1{y == alpha_low} at 2y+1.
template <class E>
__device__ __forceinline__ uint32_t dcfeq_eval(const E &A, uint64_t x, int d, const DcfView &k, uint64_t e,
                                               uint64_t N)
{
    const int L = d > 6 ? d - 6 : 0;
    Blk s = ld_blk_stream(k.root + 16 * e);
    uint32_t c = 0;
    const uint8_t *cwp = k.cw + 16 * e;
    const uint64_t stride = 16 * N;
    Blk nxt;
    if (L > 0) nxt = ld_blk_stream(cwp);
#pragma unroll 1
    for (int j = 0; j < L; j++) {
        Blk cw = nxt;
        if (j + 1 < L) nxt = ld_blk_stream(cwp + stride * uint64_t(j + 1));
        uint32_t xj = uint32_t(x >> (d - 1 - j)) & 1u;
        uint32_t tm = 0u - (s.w[0] & 1u);
        Blk cl = blk_xor(A.hash_h(s), blk_and_mask(cw, tm));
        c ^= (xj ^ 1u) & ((cl.w[0] ^ s.w[0]) & 1u);
        s = blk_xor(cl, blk_and_mask(s, 0u - xj));
    }
    uint32_t tm = 0u - (s.w[0] & 1u);
    Blk lf = ld_blk_stream(k.leaf + 16 * e);
    Blk g = blk_xor(A.hash_c(s), blk_and_mask(lf, tm));
    const uint32_t y = uint32_t(x) & 63u;
    return (c ^ uint32_t(blk_bit(g, 2 * y))) | (uint32_t(blk_bit(g, 2 * y + 1)) << 1);
}

// 128-bit vector with bit y set for every y < v (v <= 128)
__device__ __forceinline__ Blk lower_mask(uint32_t v)
{
    Blk m;
#pragma unroll
    for (int q = 0; q < 4; q++) {
        uint32_t lo = 32u * q;
        m.w[q] = v >= lo + 32 ? 0xFFFFFFFFu : (v <= lo ? 0u : ((1u << (v - lo)) - 1u));
    }
    return m;
}

// Dealer: both parties' keys for 1{x < alpha}, written at element e.
template <class E>
__device__ __forceinline__ void dcf_keygen(const E &A, uint64_t alpha, int d, Blk s0, Blk delta,
                                           const DcfOut &o, uint64_t e, uint64_t N)
{
    const int L = d > 7 ? d - 7 : 0;
    delta.w[0] |= 1u;
    Blk cur0 = s0, cur1 = blk_xor(s0, delta);
    st_blk(o.root0 + 16 * e, cur0);
    st_blk(o.root1 + 16 * e, cur1);
#pragma unroll 1
    for (int j = 0; j < L; j++) {
        uint32_t a = uint32_t(alpha >> (d - 1 - j)) & 1u;
        Blk h0 = A.hash_h(cur0), h1 = A.hash_h(cur1);
        Blk cw = blk_xor(blk_xor(h0, h1), blk_and_mask(delta, a - 1u));  // Delta when a == 0
        st_blk(o.cw0 + 16 * (uint64_t(j) * N + e), cw);
        st_blk(o.cw1 + 16 * (uint64_t(j) * N + e), cw);
        Blk c0 = blk_xor(h0, blk_and_mask(cw, 0u - (cur0.w[0] & 1u)));
        Blk c1 = blk_xor(h1, blk_and_mask(cw, 0u - (cur1.w[0] & 1u)));
        cur0 = blk_xor(c0, blk_and_mask(cur0, 0u - a));
        cur1 = blk_xor(c1, blk_and_mask(cur1, 0u - a));
    }
    const int lb = d - L;
    Blk m = lower_mask(uint32_t(alpha & ((1ull << lb) - 1)));
    Blk leaf = blk_xor(blk_xor(A.hash_c(cur0), A.hash_c(cur1)), m);
    st_blk(o.leaf0 + 16 * e, leaf);
    st_blk(o.leaf1 + 16 * e, leaf);
}

// Dealer: both parties' keys of the DCF with equality output.
template <class E>
__device__ __forceinline__ void dcfeq_keygen(const E &A, uint64_t alpha, int d, Blk s0, Blk delta,
                                             const DcfOut &o, uint64_t e, uint64_t N)
{
    const int L = d > 6 ? d - 6 : 0;
    delta.w[0] |= 1u;
    Blk cur0 = s0, cur1 = blk_xor(s0, delta);
    st_blk(o.root0 + 16 * e, cur0);
    st_blk(o.root1 + 16 * e, cur1);
#pragma unroll 1
    for (int j = 0; j < L; j++) {
        uint32_t a = uint32_t(alpha >> (d - 1 - j)) & 1u;
        Blk h0 = A.hash_h(cur0), h1 = A.hash_h(cur1);
        Blk cw = blk_xor(blk_xor(h0, h1), blk_and_mask(delta, a - 1u));
        st_blk(o.cw0 + 16 * (uint64_t(j) * N + e), cw);
        st_blk(o.cw1 + 16 * (uint64_t(j) * N + e), cw);
        Blk c0 = blk_xor(h0, blk_and_mask(cw, 0u - (cur0.w[0] & 1u)));
        Blk c1 = blk_xor(h1, blk_and_mask(cw, 0u - (cur1.w[0] & 1u)));
        cur0 = blk_xor(c0, blk_and_mask(cur0, 0u - a));
        cur1 = blk_xor(c1, blk_and_mask(cur1, 0u - a));
    }
    // leaf mask: interleaved (lt, eq) pairs for the 64 slots
    const uint32_t al = uint32_t(alpha & 63u);
    Blk m;
#pragma unroll
    for (int q = 0; q < 4; q++) {
        uint32_t w = 0;
        for (int b = 0; b < 16; b++) {
            const uint32_t y = 16u * q + b;
            if (y < al) w |= 1u << (2 * b);
            if (y == al) w |= 2u << (2 * b);
        }
        m.w[q] = w;
    }
    Blk leaf = blk_xor(blk_xor(A.hash_c(cur0), A.hash_c(cur1)), m);
    st_blk(o.leaf0 + 16 * e, leaf);
    st_blk(o.leaf1 + 16 * e, leaf);
}

template <typename T>
__device__ __forceinline__ T ring_of(const Blk &b)
{
    if constexpr (sizeof(T) == 4) return b.w[0];
    else return uint64_t(b.w[0]) | (uint64_t(b.w[1]) << 32);
}

}  // namespace ddg
