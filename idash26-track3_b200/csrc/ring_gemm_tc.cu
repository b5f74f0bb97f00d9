// Ring GEMMs over Z_2^32 / Z_2^64 on the 5th-generation tensor cores.
//
// Same contract as the CUDA-core kernel in ring_gemm.cu (GemmArgs):
//
//   C[b] = sign * ( A1[b] . (s1*B1[b] - B1m[b])  -  A2[b] . B2[b] ) + bias + Add[b]
//
// Exactness by 8-bit limb splitting.  Every ring element a = sum_i a_i 2^(8i)
// with unsigned bytes a_i (P = sizeof(T) limbs).  Modulo 2^(8P)
//
//   (A.B)[m,n] = sum_{s<P} 2^(8s) * S_s[m,n],   S_s = sum_{i+j=s} A_i . B_j ,
//
// so only the P(P+1)/2 limb products with i+j < P are needed (10 for Z_2^32,
// 36 for Z_2^64).  Each A_i . B_j is a u8 x u8 GEMM with exact int32
// accumulation (tcgen05.mma kind::i8); the P partial sums S_s live side by
// side in tensor memory and the epilogue recombines them with shifts, so the
// result is exact modulo 2^(8P) as long as no S_s exceeds 2^31 before its
// shift, i.e. (s+1) * K * 255^2 < 2^31 for every s (K <= 4096 at P = 8,
// K <= 8192 at P = 4; the host sends larger K to the CUDA-core kernel).
//
// The two products of the Beaver form are one GEMM over the concatenated
// reduction dimension: C = [A1 | A2] . [sign*(s1*B1 - B1m) ; -sign*B2], so
// the B operand is formed (and negated) in the loader, modulo 2^(8P).
//
// Per CTA: a 128 x BN output tile, 256 threads.  The K loop moves 32 ring
// elements of K per stage (one MMA K-step for 8-bit operands).  All threads
// load the stage's A (128 x 32) and B (32 x BN) ring elements from global
// memory, split them into P byte planes with byte permutes and store the
// planes in shared memory in the canonical no-swizzle UMMA layouts (A K-major,
// B either MN-major or K-major).  After fence.proxy.async + a CTA barrier one
// thread issues the limb MMAs for the stage and commits them to the stage's
// mbarrier; the stage is rewritten only after that mbarrier completes.  Two
// stages: the loads of stage k+1 are in flight while the MMAs of stage k run.
// Every mbarrier wait is bounded (about two seconds of %globaltimer); a wait
// that gives up sets the error word and the CTA skips to freeing its tensor
// memory, so a fault in this logic shows up as a status code, not a hang.
#include <vector>

#include "common.cuh"
#include "linear.cuh"

namespace ddg {

namespace {

constexpr int TC_BM = 128;       // tile rows (TMEM lanes)
constexpr int TC_BK = 32;        // K elements per stage = one kind::i8 MMA K-step
constexpr int TC_THREADS = 256;  // 8 warps
constexpr uint64_t TC_WAIT_NS = 2000000000ull;

__device__ __forceinline__ uint32_t smem_addr(const void *p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_ns()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// shared-memory matrix descriptor, no swizzle (layout type 0), version 1
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo)
{
    return uint64_t((addr >> 4) & 0x3FFFu) | (uint64_t((lbo >> 4) & 0x3FFFu) << 16) |
           (uint64_t((sbo >> 4) & 0x3FFFu) << 32) | (uint64_t(1) << 46);
}

// instruction descriptor of kind::i8: u8 x u8 -> s32, A K-major, M = 128
__host__ __device__ constexpr uint32_t i8_idesc(int bn, bool b_mn_major)
{
    return (2u << 4)                          // D format s32
           | (0u << 7) | (0u << 10)           // A, B unsigned 8-bit
           | ((b_mn_major ? 1u : 0u) << 16)   // B major
           | (uint32_t(bn >> 3) << 17)        // N >> 3
           | (uint32_t(TC_BM >> 4) << 24);    // M >> 4
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ bool mbar_test(uint64_t *bar, uint32_t parity)
{
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// wait until the phase with the given parity of `bar` has completed; false
// after TC_WAIT_NS (or 2^26 polls) without completion
__device__ bool mbar_wait(uint64_t *bar, uint32_t parity)
{
    const uint64_t t0 = global_ns();
    for (uint32_t it = 1; it < (1u << 26); ++it) {
        if (mbar_test(bar, parity)) return true;
        if ((it & 255u) == 0 && global_ns() - t0 > TC_WAIT_NS) return false;
    }
    return false;
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t da, uint64_t db, uint32_t idesc, uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(da), "l"(db), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t *bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&v)[8])
{
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(taddr)
                 : "memory");
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// the four byte planes of four consecutive 32-bit words: plane q holds byte q of e0..e3
__device__ __forceinline__ void byte_planes(uint32_t e0, uint32_t e1, uint32_t e2, uint32_t e3, uint32_t (&p)[4])
{
    const uint32_t lo01 = __byte_perm(e0, e1, 0x5140), lo23 = __byte_perm(e2, e3, 0x5140);
    const uint32_t hi01 = __byte_perm(e0, e1, 0x7362), hi23 = __byte_perm(e2, e3, 0x7362);
    p[0] = __byte_perm(lo01, lo23, 0x5410);
    p[1] = __byte_perm(lo01, lo23, 0x7632);
    p[2] = __byte_perm(hi01, hi23, 0x5410);
    p[3] = __byte_perm(hi01, hi23, 0x7632);
}

template <typename T>
__device__ __forceinline__ void store_planes(uint8_t *base, uint32_t plane_bytes, uint32_t off, const T (&e)[4])
{
    uint32_t p[4];
    byte_planes(uint32_t(e[0]), uint32_t(e[1]), uint32_t(e[2]), uint32_t(e[3]), p);
#pragma unroll
    for (int q = 0; q < 4; q++) *reinterpret_cast<uint32_t *>(base + q * plane_bytes + off) = p[q];
    if constexpr (sizeof(T) == 8) {
        byte_planes(uint32_t(uint64_t(e[0]) >> 32), uint32_t(uint64_t(e[1]) >> 32), uint32_t(uint64_t(e[2]) >> 32),
                    uint32_t(uint64_t(e[3]) >> 32), p);
#pragma unroll
        for (int q = 0; q < 4; q++) *reinterpret_cast<uint32_t *>(base + (4 + q) * plane_bytes + off) = p[q];
    }
}

constexpr int tmem_cols(int n)
{
    int c = 32;
    while (c < n) c <<= 1;
    return c;
}

// Epilogue of a 128 x BN tile: warp w reads TMEM lanes 32*(w%4).. (rows) and
// half w/4 of the columns, 8 columns per tcgen05.ld, and writes
// C = sign * sum_s S_s << 8s + bias + Add.  The Add and bias words of four
// 8-column chunks are loaded before their accumulators are read, so that
// their global-memory latencies overlap instead of adding up chunk by chunk.
template <typename T, int P, int BN>
__device__ __forceinline__ void tc_epilogue(uint32_t tmem, int warp, int lane, int m0, int n0, int M, int N, T sign,
                                            const T *bias, const T *Add, int64_t ldAdd, T *C, int64_t ldc)
{
    constexpr int NCH = BN / 2 / 8;      // 8-column chunks per warp half
    constexpr int G = NCH < 4 ? NCH : 4; // chunks per group
    static_assert(NCH % G == 0, "chunk groups");
    const int q = warp & 3, h = warp >> 2;
    const int m = m0 + 32 * q + lane;
    const bool row_ok = m < M;
#pragma unroll 1
    for (int g0 = 0; g0 < NCH; g0 += G) {
        T extra[G][8];
#pragma unroll
        for (int g = 0; g < G; g++)
#pragma unroll
            for (int e = 0; e < 8; e++) {
                const int n = n0 + h * (BN / 2) + (g0 + g) * 8 + e;
                T v = 0;
                if (row_ok && n < N) {
                    if (bias) v += __ldg(bias + n);
                    if (Add) v += __ldg(Add + int64_t(m) * ldAdd + n);
                }
                extra[g][e] = v;
            }
#pragma unroll
        for (int g = 0; g < G; g++) {
            const int c = h * (BN / 2) + (g0 + g) * 8;
            T r[8];
#pragma unroll
            for (int e = 0; e < 8; e++) r[e] = 0;
#pragma unroll
            for (int sft = 0; sft < P; sft++) {
                uint32_t v[8];
                tmem_ld8(tmem + (uint32_t(32 * q) << 16) + uint32_t(sft * BN + c), v);
                tmem_ld_wait();
#pragma unroll
                for (int e = 0; e < 8; e++) r[e] += T(v[e]) << (8 * sft);
            }
            if (row_ok) {
#pragma unroll
                for (int e = 0; e < 8; e++) {
                    const int n = n0 + c + e;
                    if (n < N) C[int64_t(m) * ldc + n] = sign * r[e] + extra[g][e];
                }
            }
        }
    }
}

// Per-stage shared-memory and tensor-memory budget of one CTA.
template <typename T, int BN, bool B_MN>
struct TcShape {
    static constexpr int P = int(sizeof(T));
    static constexpr int A_PLANE = TC_BM * TC_BK;  // bytes of one A byte plane per stage
    static constexpr int B_PLANE = BN * TC_BK;     // bytes of one B byte plane per stage
    static constexpr int STAGE = P * (A_PLANE + B_PLANE);
    // The operand tiles start on a 1024-byte boundary of the shared window
    // (after the barriers and up to 1 KiB of alignment padding), and 8 KiB of
    // slack follow the two stages so that a descriptor read differently from
    // this layout still stays inside the CTA's shared memory.
    static constexpr int SMEM = 32 + 1024 + 2 * STAGE + 8192;
    static constexpr int NCOL = tmem_cols(P * BN);
    static constexpr int A_ITEMS = TC_BM * TC_BK / 4 / TC_THREADS;  // 4-element items per thread
    static constexpr int B_ITEMS = BN * TC_BK / 4 / TC_THREADS;
    static_assert(P * BN <= 512, "accumulators exceed tensor memory");
    static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "BN");
    static_assert(B_ITEMS >= 1, "B tile too small for the loader mapping");
};

template <typename T, int BN, bool B_MN>
__global__ void __launch_bounds__(TC_THREADS, 1)
    ring_gemm_tc_kernel(const __grid_constant__ GemmArgs<T> a, int nk0, int nk1, uint32_t *err)
{
    using S = TcShape<T, BN, B_MN>;
    constexpr int P = S::P;
    // Dynamic shared memory only: [2 mbarriers | TMEM address | pad to 1024 | stage 0 | stage 1 | slack].
    // With the barriers as static __shared__ variables beside the dynamic
    // array, the MMAs read every operand tile 32 bytes below the address in
    // its descriptor (measured on B200: the products matched a model shifted
    // by exactly -32 B for A and B), so this kernel declares no static shared
    // memory.
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint64_t *const bars = reinterpret_cast<uint64_t *>(smem_raw);
    uint32_t &s_tmem = *reinterpret_cast<uint32_t *>(smem_raw + 16);
    uint8_t *const smem = smem_raw + 32 + ((1024u - ((smem_addr(smem_raw) + 32u) & 1023u)) & 1023u);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int b = blockIdx.z;
    const int m0 = blockIdx.y * TC_BM, n0 = blockIdx.x * BN;
    const int nk = nk0 + nk1;

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&s_tmem)),
                     "r"(S::NCOL)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 0) {
        mbar_init(bars + 0, 1);
        mbar_init(bars + 1, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;

    // per-batch operand bases
    const T *A1 = a.A1 + int64_t(b) * a.sA1;
    const T *A2 = a.A2 ? a.A2 + int64_t(b) * a.sA2 : nullptr;
    const T *B1 = a.B1 ? a.B1 + int64_t(b) * a.sB1 : nullptr;
    const T *B1m = a.B1m ? a.B1m + int64_t(b) * a.sB1m : nullptr;
    const T *B2 = a.B2 ? a.B2 + int64_t(b) * a.sB2 : nullptr;
    const T sgn = a.sign, s1 = a.s1;

    // loader item coordinates (fixed per thread): A item j covers row ar[j],
    // K elements 4*akq .. 4*akq+3 of the stage; see the layout notes above.
    const int akq = 4 * (warp & 1) + (lane & 3);
    T ra[S::A_ITEMS][4], rb[S::B_ITEMS][4];

    auto load_stage = [&](int kb) {
        const bool ph1 = kb >= nk0;
        const int kbase = (ph1 ? kb - nk0 : kb) * TC_BK;
        const T *A = ph1 ? A2 : A1;
        const int64_t lda = ph1 ? a.lda2 : a.lda1;
#pragma unroll
        for (int j = 0; j < S::A_ITEMS; j++) {
            const int row = 8 * (warp >> 1) + 32 * j + (lane >> 2);
            const int m = m0 + row, k = kbase + 4 * akq;
#pragma unroll
            for (int e = 0; e < 4; e++)
                ra[j][e] = (m < a.M && k + e < a.K) ? __ldg(A + int64_t(m) * lda + k + e) : T(0);
        }
        const int64_t ldb = ph1 ? a.ldb2 : a.ldb1;
#pragma unroll
        for (int j = 0; j < S::B_ITEMS; j++) {
            const int w = warp + 8 * j;  // warp-slot index of this item
            int k, n, dk, dn;            // element e sits at (k + e*dk, n + e*dn)
            if constexpr (B_MN) {
                constexpr int NG = BN / 16;
                k = kbase + 8 * (w / NG) + (lane >> 2), n = n0 + 16 * (w % NG) + 4 * (lane & 3), dk = 0, dn = 1;
            } else {
                k = kbase + 16 * (w & 1) + 4 * (lane & 3), n = n0 + 8 * (w >> 1) + (lane >> 2), dk = 1, dn = 0;
            }
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int ke = k + e * dk, ne = n + e * dn;
                T v = 0;
                if (ke < a.K && ne < a.N) {
                    const int64_t o = int64_t(ke) * ldb + ne;
                    if (ph1) {
                        v = T(0) - sgn * __ldg(B2 + o);
                    } else {
                        if (B1) v = s1 * __ldg(B1 + o);
                        if (B1m) v -= __ldg(B1m + o);
                        v *= sgn;
                    }
                }
                rb[j][e] = v;
            }
        }
    };

    auto store_stage = [&](int st) {
        uint8_t *base = smem + st * S::STAGE;
#pragma unroll
        for (int j = 0; j < S::A_ITEMS; j++) {
            const int row = 8 * (warp >> 1) + 32 * j + (lane >> 2);
            const uint32_t off = (row >> 3) * 256 + (akq >> 2) * 128 + (row & 7) * 16 + (akq & 3) * 4;
            store_planes<T>(base, S::A_PLANE, off, ra[j]);
        }
        uint8_t *bbase = base + P * S::A_PLANE;
#pragma unroll
        for (int j = 0; j < S::B_ITEMS; j++) {
            const int w = warp + 8 * j;
            uint32_t off;
            if constexpr (B_MN) {
                constexpr int NG = BN / 16;
                off = (w % NG) * 128 + (w / NG) * (8 * BN) + 4 * lane;
            } else {
                off = (w >> 1) * 256 + (w & 1) * 128 + 4 * lane;
            }
            store_planes<T>(bbase, S::B_PLANE, off, rb[j]);
        }
    };

    constexpr uint32_t IDESC = i8_idesc(BN, B_MN);
    constexpr uint32_t B_LBO = B_MN ? 8 * BN : 128, B_SBO = B_MN ? 128 : 256;
    bool ok = true;

    if (nk > 0) load_stage(0);
    for (int kb = 0; kb < nk; kb++) {
        const int st = kb & 1;
        // stage st is free once the MMAs committed two K-steps ago have completed
        bool mine = true;
        if (kb >= 2) mine = mbar_wait(&bars[st], uint32_t(((kb >> 1) - 1) & 1));
        if (mine) store_stage(st);
        if (kb + 1 < nk) load_stage(kb + 1);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        // CTA-uniform: every thread leaves the loop together if any wait gave up
        if (!__syncthreads_and(mine ? 1 : 0)) {
            ok = false;
            break;
        }
        if (tid == 0) {
            tc_fence_after();
            const uint32_t sa = smem_addr(smem + st * S::STAGE);
            const uint32_t sb = sa + P * S::A_PLANE;
#pragma unroll
            for (int i = 0; i < P; i++) {
                const uint64_t da = smem_desc(sa + i * S::A_PLANE, 128, 256);
#pragma unroll
                for (int j = 0; j + i < P; j++) {
                    const uint64_t db = smem_desc(sb + j * S::B_PLANE, B_LBO, B_SBO);
                    mma_i8(tmem + uint32_t((i + j) * BN), da, db, IDESC, (kb > 0 || i > 0) ? 1u : 0u);
                }
            }
            mma_commit(&bars[st]);
        }
    }
    // the last commit covers every MMA issued before it
    if (ok && nk > 0) ok = mbar_wait(&bars[(nk - 1) & 1], uint32_t(((nk - 1) >> 1) & 1));
    // a CTA-uniform verdict: every thread saw the same barrier phases unless one timed out
    const int all_ok = __syncthreads_and(ok ? 1 : 0);
    tc_fence_after();

    if (all_ok) {
        tc_epilogue<T, P, BN>(tmem, warp, lane, m0, n0, a.M, a.N, T(1), a.bias,
                              a.Add ? a.Add + int64_t(b) * a.sAdd : nullptr, a.ldAdd, a.C + int64_t(b) * a.sC, a.ldc);
    } else if (tid == 0) {
        atomicOr(err, 1u);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(S::NCOL) : "memory");
    }
}

// ---------------------------------------------------------------------------
// Z_2^32 variant with asynchronous operand staging.
//
// Same limb algebra and MMAs as ring_gemm_tc_kernel, but the ring elements of
// each K-step reach shared memory through cp.async (8-byte copies, zero-fill
// past the matrix edges) into one of three raw stages, so that the global
// loads of the next two K-steps are in flight while the current one is split
// into byte planes and multiplied.  Computes C = sign * (A1 . B1 + A2 . B2) +
// bias + Add: the host folds s1, B1m and the Beaver minus sign into B1 / B2
// beforehand.  128 x 128 output tiles (four 128-column s32 accumulators = all
// 512 TMEM columns), B MN-major.  Needs even row strides and 8-byte aligned
// operands (the host checks, and otherwise uses ring_gemm_tc_kernel).  The
// kernel itself also takes a second product (A2 . B2) for callers that
// prepare its B operand.
// Raw tiles are stored row-major with the 16-byte chunk index XOR-ed by
// 4 * (row & 1), which keeps the 16-byte shared loads of the split step free
// of bank conflicts.

constexpr int TC2_BN = 128;
constexpr int TC2_RS = 3;                               // raw stages
constexpr int TC2_A_PLANE = TC_BM * TC_BK;              // 4096
constexpr int TC2_B_PLANE = TC2_BN * TC_BK;             // 4096
constexpr int TC2_PSTAGE = 4 * (TC2_A_PLANE + TC2_B_PLANE);  // plane stage, 32 KiB
constexpr int TC2_RAW_A = TC_BM * TC_BK * 4;            // 16 KiB
constexpr int TC2_RAW_B = TC_BK * TC2_BN * 4;           // 16 KiB
constexpr int TC2_RSTAGE = TC2_RAW_A + TC2_RAW_B;
constexpr int TC2_SMEM = 32 + 1024 + 2 * TC2_PSTAGE + TC2_RS * TC2_RSTAGE + 8192;

struct Gemm2Args {
    int M, N, K, nk0, nk1;
    const uint32_t *A1, *A2, *B1, *B2;
    int64_t lda1, lda2, ldb1, ldb2, sA1, sA2, sB1, sB2;
    uint32_t sign;
    const uint32_t *bias, *Add;
    int64_t ldAdd, sAdd;
    uint32_t *C;
    int64_t ldc, sC;
};

__device__ __forceinline__ void cp_async8(uint32_t dst, const void *src, uint32_t src_bytes)
{
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__global__ void __launch_bounds__(TC_THREADS, 1) ring_gemm_tc2_kernel(const __grid_constant__ Gemm2Args a, uint32_t *err)
{
    constexpr int P = 4, BN = TC2_BN;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint64_t *const bars = reinterpret_cast<uint64_t *>(smem_raw);
    uint32_t &s_tmem = *reinterpret_cast<uint32_t *>(smem_raw + 16);
    uint8_t *const planes = smem_raw + 32 + ((1024u - ((smem_addr(smem_raw) + 32u) & 1023u)) & 1023u);
    uint8_t *const raws = planes + 2 * TC2_PSTAGE;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int b = blockIdx.z;
    const int m0 = blockIdx.y * TC_BM, n0 = blockIdx.x * BN;
    const int nk = a.nk0 + a.nk1;

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&s_tmem)),
                     "r"(512)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 0) {
        mbar_init(bars + 0, 1);
        mbar_init(bars + 1, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;

    const uint32_t *A1 = a.A1 + int64_t(b) * a.sA1;
    const uint32_t *A2 = a.A2 ? a.A2 + int64_t(b) * a.sA2 : nullptr;
    const uint32_t *B1 = a.B1 + int64_t(b) * a.sB1;
    const uint32_t *B2 = a.B2 ? a.B2 + int64_t(b) * a.sB2 : nullptr;
    const uint32_t raw_base = smem_addr(raws);

    // issue the cp.async copies of K-step kb into raw stage kb % RS (every thread: 8 + 8 copies)
    auto issue = [&](int kb) {
        const bool ph1 = kb >= a.nk0;
        const int kbase = (ph1 ? kb - a.nk0 : kb) * TC_BK;
        const uint32_t *A = ph1 ? A2 : A1, *B = ph1 ? B2 : B1;
        const int64_t lda = ph1 ? a.lda2 : a.lda1, ldb = ph1 ? a.ldb2 : a.ldb1;
        const uint32_t ra = raw_base + uint32_t((kb % TC2_RS) * TC2_RSTAGE), rb = ra + TC2_RAW_A;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int j = tid + TC_THREADS * i;  // A chunk: 16 per row
            const int row = j >> 4, c8 = j & 15;
            const int m = m0 + row, k = kbase + 2 * c8;
            const int nv = m < a.M ? min(max(a.K - k, 0), 2) : 0;
            const uint32_t *src = nv ? A + int64_t(m) * lda + k : A;
            cp_async8(ra + row * 128 + (((c8 >> 1) ^ ((row & 1) << 2)) << 4) + ((c8 & 1) << 3), src, 4u * nv);
        }
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int j = tid + TC_THREADS * i;  // B chunk: 64 per row
            const int kr = j >> 6, c8 = j & 63;
            const int k = kbase + kr, n = n0 + 2 * c8;
            const int nv = k < a.K ? min(max(a.N - n, 0), 2) : 0;
            const uint32_t *src = nv ? B + int64_t(k) * ldb + n : B;
            cp_async8(rb + kr * 512 + (((c8 >> 1) ^ ((kr & 1) << 2)) << 4) + ((c8 & 1) << 3), src, 4u * nv);
        }
    };

    // split raw stage rs into plane stage ps (byte planes in the canonical layouts)
    const int akq = 4 * (warp & 1) + (lane & 3);
    auto split = [&](int rs, int ps) {
        const uint8_t *ra = raws + rs * TC2_RSTAGE, *rb = ra + TC2_RAW_A;
        uint8_t *pa = planes + ps * TC2_PSTAGE, *pb = pa + P * TC2_A_PLANE;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int row = 8 * (warp >> 1) + 32 * j + (lane >> 2);
            const uint4 v = *reinterpret_cast<const uint4 *>(ra + row * 128 + ((akq ^ ((row & 1) << 2)) << 4));
            const uint32_t e[4] = {v.x, v.y, v.z, v.w};
            store_planes<uint32_t>(pa, TC2_A_PLANE, (row >> 3) * 256 + (akq >> 2) * 128 + (row & 7) * 16 + (akq & 3) * 4,
                                   e);
        }
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int w = warp + 8 * j, kg = w >> 3, ng = w & 7;
            const int kr = 8 * kg + (lane >> 2), cq = 4 * ng + (lane & 3);
            const uint4 v = *reinterpret_cast<const uint4 *>(rb + kr * 512 + ((cq ^ ((kr & 1) << 2)) << 4));
            const uint32_t e[4] = {v.x, v.y, v.z, v.w};
            store_planes<uint32_t>(pb, TC2_B_PLANE, ng * 128 + kg * (8 * BN) + 4 * lane, e);
        }
    };

    constexpr uint32_t IDESC = i8_idesc(BN, true);
    bool ok = true;
    for (int kb = 0; kb < TC2_RS - 1; kb++) {
        if (kb < nk) issue(kb);
        cp_async_commit();
    }
    for (int kb = 0; kb < nk; kb++) {
        if (kb + TC2_RS - 1 < nk) issue(kb + TC2_RS - 1);
        cp_async_commit();
        cp_async_wait<TC2_RS - 1>();  // this thread's copies of K-step kb have landed
        const int ps = kb & 1;
        bool mine = true;
        if (kb >= 2) mine = mbar_wait(&bars[ps], uint32_t(((kb >> 1) - 1) & 1));
        if (!__syncthreads_and(mine ? 1 : 0)) {  // every thread's copies landed, plane stage ps is free
            ok = false;
            break;
        }
        split(kb % TC2_RS, ps);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
            const uint32_t sa = smem_addr(planes + ps * TC2_PSTAGE);
            const uint32_t sb = sa + P * TC2_A_PLANE;
#pragma unroll
            for (int i = 0; i < P; i++) {
                const uint64_t da = smem_desc(sa + i * TC2_A_PLANE, 128, 256);
#pragma unroll
                for (int j = 0; j + i < P; j++) {
                    const uint64_t db = smem_desc(sb + j * TC2_B_PLANE, 8 * BN, 128);
                    mma_i8(tmem + uint32_t((i + j) * BN), da, db, IDESC, (kb > 0 || i > 0) ? 1u : 0u);
                }
            }
            mma_commit(&bars[ps]);
        }
    }
    cp_async_wait<0>();
    if (ok && nk > 0) ok = mbar_wait(&bars[(nk - 1) & 1], uint32_t(((nk - 1) >> 1) & 1));
    const int all_ok = __syncthreads_and(ok ? 1 : 0);
    tc_fence_after();

    if (all_ok) {
        tc_epilogue<uint32_t, P, BN>(tmem, warp, lane, m0, n0, a.M, a.N, a.sign, a.bias,
                                     a.Add ? a.Add + int64_t(b) * a.sAdd : nullptr, a.ldAdd, a.C + int64_t(b) * a.sC,
                                     a.ldc);
    } else if (tid == 0) {
        atomicOr(err, 2u);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512) : "memory");
    }
}

__device__ uint32_t g_tc_err;

// 0: tensor cores (default): for Z_2^32 the packed-operand kernel
// (ring_gemm_pk.cu); for Z_2^64 B MN-major with 32-column tiles; 1: CUDA cores
// only; 2: tensor cores, B K-major; 3: tensor cores, 128-column tiles
// (Z_2^32) or 32-column tiles (Z_2^64); 4: tensor cores, B MN-major,
// 64-column tiles (the synchronous kernel); 5: for Z_2^32 the in-kernel
// operand split (the asynchronous-staging kernel where the operands allow it,
// else 64-column tiles) with the CUDA cores on ragged last rows.  2-5 exist for
// the layout/tile comparison tests.
int g_gemm_path = 0;

template <typename T, int BN, bool B_MN>
int launch_tc(const GemmArgs<T> &a, cudaStream_t st)
{
    using S = TcShape<T, BN, B_MN>;
    auto kern = ring_gemm_tc_kernel<T, BN, B_MN>;
    static thread_local int configured_dev = -1;
    int dev = 0;
    DDG_CUDA(cudaGetDevice(&dev));
    if (configured_dev != dev) {
        DDG_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::SMEM));
        configured_dev = dev;
    }
    uint32_t *err = nullptr;
    DDG_CUDA(cudaGetSymbolAddress(reinterpret_cast<void **>(&err), g_tc_err));
    DDG_CHECK(a.A1 && a.C && (!a.A2 || a.B2), DDG_ERR_ARG, "gemm: missing operand");
    const int nk0 = (a.K + TC_BK - 1) / TC_BK;
    const int nk1 = a.A2 ? nk0 : 0;
    dim3 grid((a.N + BN - 1) / BN, (a.M + TC_BM - 1) / TC_BM, a.batch);
    DDG_CHECK(grid.y <= 65535 && grid.z <= 65535, DDG_ERR_ARG, "gemm grid too large (M=%d batch=%d)", a.M, a.batch);
    kern<<<grid, TC_THREADS, S::SMEM, st>>>(a, nk0, nk1, err);
    note_launch();
    DDG_CUDA(cudaGetLastError());
    return DDG_OK;
}

// the asynchronous-staging kernel for Z_2^32 when the operands allow it
// (*launched = 1), else nothing (*launched = 0).  The Beaver form (B1m, s1,
// a second product) is left to ring_gemm_tc_kernel, whose loader folds those
// terms: rewriting the B operands first for this kernel measured slower.
int launch_tc2(const GemmArgs<uint32_t> &a, cudaStream_t st, int *launched)
{
    *launched = 0;
    auto even = [](int64_t v) { return (v & 1) == 0; };
    auto al8 = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 7) == 0; };
    if (a.A2 || a.B1m || a.s1 != 1u || !a.B1) return DDG_OK;
    if (!even(a.lda1) || !even(a.sA1) || !al8(a.A1) || !even(a.ldb1) || !even(a.sB1) || !al8(a.B1)) return DDG_OK;
    DDG_CHECK(a.A1 && a.C, DDG_ERR_ARG, "gemm: missing operand");
    static thread_local int configured_dev = -1;
    int dev = 0;
    DDG_CUDA(cudaGetDevice(&dev));
    if (configured_dev != dev) {
        DDG_CUDA(cudaFuncSetAttribute(ring_gemm_tc2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, TC2_SMEM));
        configured_dev = dev;
    }
    uint32_t *err = nullptr;
    DDG_CUDA(cudaGetSymbolAddress(reinterpret_cast<void **>(&err), g_tc_err));
    Gemm2Args g;
    g.M = a.M, g.N = a.N, g.K = a.K;
    g.nk0 = (a.K + TC_BK - 1) / TC_BK, g.nk1 = 0;
    g.A1 = a.A1, g.A2 = nullptr, g.lda1 = a.lda1, g.lda2 = 0, g.sA1 = a.sA1, g.sA2 = 0;
    g.B1 = a.B1, g.B2 = nullptr, g.ldb1 = a.ldb1, g.ldb2 = 0, g.sB1 = a.sB1, g.sB2 = 0;
    g.sign = a.sign, g.bias = a.bias, g.Add = a.Add, g.ldAdd = a.ldAdd, g.sAdd = a.sAdd;
    g.C = a.C, g.ldc = a.ldc, g.sC = a.sC;
    dim3 grid((a.N + TC2_BN - 1) / TC2_BN, (a.M + TC_BM - 1) / TC_BM, a.batch);
    DDG_CHECK(grid.y <= 65535 && grid.z <= 65535, DDG_ERR_ARG, "gemm grid too large (M=%d batch=%d)", a.M, a.batch);
    ring_gemm_tc2_kernel<<<grid, TC_THREADS, TC2_SMEM, st>>>(g, err);
    note_launch();
    DDG_CUDA(cudaGetLastError());
    *launched = 1;
    return DDG_OK;
}

}  // namespace

// the error word every tensor-core GEMM kernel sets when a bounded wait gives up
int ring_gemm_err_word(uint32_t **out)
{
    DDG_CUDA(cudaGetSymbolAddress(reinterpret_cast<void **>(out), g_tc_err));
    return DDG_OK;
}

int ring_gemm_packed(const GemmArgs<uint32_t> &a, cudaStream_t st);  // ring_gemm_pk.cu
uint64_t ring_gemm_packed_a_bytes(const GemmArgs<uint32_t> &a);      // ring_gemm_pk.cu

int ring_gemm_tc_error(bool clear)
{
    uint32_t v = 0;
    DDG_CUDA(cudaMemcpyFromSymbol(&v, g_tc_err, sizeof(v)));
    if (clear && v) {
        const uint32_t z = 0;
        DDG_CUDA(cudaMemcpyToSymbol(g_tc_err, &z, sizeof(z)));
    }
    DDG_CHECK(v == 0, DDG_ERR_CUDA, "tensor-core ring GEMM: an mbarrier wait gave up (error word %u)", v);
    return DDG_OK;
}

int ring_gemm_tc_check(cudaStream_t st)
{
    uint32_t v = 0;
    DDG_CUDA(cudaMemcpyFromSymbolAsync(&v, g_tc_err, sizeof(v), 0, cudaMemcpyDeviceToHost, st));
    DDG_CUDA(cudaStreamSynchronize(st));
    DDG_CHECK(v == 0, DDG_ERR_CUDA, "tensor-core ring GEMM: an mbarrier wait gave up (error word %u)", v);
    return DDG_OK;
}

void set_gemm_path(int path) { g_gemm_path = path; }
int gemm_path() { return g_gemm_path; }

// largest reduction length (per phase) whose limb sums stay below 2^31
template <typename T>
constexpr int tc_max_k()
{
    return sizeof(T) == 4 ? 8192 : 4096;
}

// rows beyond the last whole 128-row tile that go to the CUDA cores instead
// of a mostly empty tensor-core tile (default path)
constexpr int TC_THIN_TAIL = 32;

// the packed-operand engine takes this GEMM (the default at bw=32)
template <typename T>
static bool takes_packed(const GemmArgs<T> &a)
{
    const int ktot = a.A2 ? 2 * a.K : a.K;
    if (sizeof(T) != 4 || g_gemm_path != 0 || a.K == 0 || ktot > tc_max_k<T>()) return false;
    const int ng = (a.M + TC_BM - 1) / TC_BM, nks = (ktot + TC_BK - 1) / TC_BK;
    return a.batch <= 65535 && int64_t(ng) * nks <= 65535;
}

// x + y over `extent` words into a stream-ordered temporary
template <typename T>
static int sum_operand(const T *x, const T *y, uint64_t extent, cudaStream_t st, const T **out,
                       std::vector<void *> &tmp)
{
    T *p = nullptr;
    DDG_CUDA(cudaMallocAsync(&p, (extent ? extent : 1) * sizeof(T), st));
    tmp.push_back(p);
    DDG_TRY(ew_add<T>(p, x, y, extent, st));
    *out = p;
    return DDG_OK;
}

template <typename T>
int ring_gemm(const GemmArgs<T> &a, cudaStream_t st)
{
    if (a.M == 0 || a.N == 0 || a.batch == 0) return DDG_OK;
    const int ktot = a.A2 ? 2 * a.K : a.K;
    if ((a.A1b || a.B1b || a.B2b) && !takes_packed(a)) {
        // operands held as two addends: the other engines read one operand, so add them first
        GemmArgs<T> m = a;
        m.A1b = m.B1b = m.B2b = nullptr;
        std::vector<void *> tmp;
        const uint64_t nb = uint64_t(a.batch - 1);
        int err = DDG_OK;
        if (a.A1b)
            err = sum_operand<T>(a.A1, a.A1b, nb * a.sA1 + uint64_t(a.M - 1) * a.lda1 + a.K, st, &m.A1, tmp);
        if (err == DDG_OK && a.B1b && a.B1)
            err = sum_operand<T>(a.B1, a.B1b, nb * a.sB1 + uint64_t(a.K - 1) * a.ldb1 + a.N, st, &m.B1, tmp);
        if (err == DDG_OK && a.B2b && a.B2) {
            if (a.B2 == a.B1 && a.B2b == a.B1b && a.sB2 == a.sB1 && a.ldb2 == a.ldb1)
                m.B2 = m.B1;
            else
                err = sum_operand<T>(a.B2, a.B2b, nb * a.sB2 + uint64_t(a.K - 1) * a.ldb2 + a.N, st, &m.B2, tmp);
        }
        if (err == DDG_OK) err = ring_gemm<T>(m, st);
        for (void *p : tmp) cudaFreeAsync(p, st);
        return err;
    }
    if (g_gemm_path == 1 || a.K == 0 || ktot > tc_max_k<T>()) return ring_gemm_simt<T>(a, st);
    if constexpr (sizeof(T) == 4) {
        if (takes_packed(a)) return ring_gemm_packed(a, st);
    }
    const int tail = a.M % TC_BM;
    if ((g_gemm_path == 0 || g_gemm_path == 5) && a.M > TC_BM && tail != 0 && tail <= TC_THIN_TAIL) {
        GemmArgs<T> whole = a;
        whole.M = a.M - tail;
        DDG_TRY(ring_gemm<T>(whole, st));
        return ring_gemm_rows<T>(a, whole.M, st);
    }
    if (g_gemm_path == 2) return launch_tc<T, 64, false>(a, st);
    if (g_gemm_path == 3) return launch_tc<T, sizeof(T) == 4 ? 128 : 32, true>(a, st);
    if constexpr (sizeof(T) == 4) {
        if (g_gemm_path == 0 || g_gemm_path == 5) {
            int launched = 0;
            DDG_TRY(launch_tc2(a, st, &launched));
            if (launched) return DDG_OK;
        }
        return launch_tc<T, 64, true>(a, st);
    } else {
        // Z_2^64: 32-column tiles (8 accumulators x 32 = 256 TMEM columns, two
        // CTAs per SM) measured 1.2-1.5x faster than 64-column tiles
        if (g_gemm_path == 0) return launch_tc<T, 32, true>(a, st);
        return launch_tc<T, 64, true>(a, st);
    }
}

template int ring_gemm<uint32_t>(const GemmArgs<uint32_t> &, cudaStream_t);
template int ring_gemm<uint64_t>(const GemmArgs<uint64_t> &, cudaStream_t);

template <typename T>
uint64_t ring_gemm_a_pack_bytes(const GemmArgs<T> &a)
{
    if constexpr (sizeof(T) == 4) {
        if (a.M > 0 && a.N > 0 && a.batch > 0 && takes_packed(a)) return ring_gemm_packed_a_bytes(a);
    }
    return 0;
}
template uint64_t ring_gemm_a_pack_bytes<uint32_t>(const GemmArgs<uint32_t> &);
template uint64_t ring_gemm_a_pack_bytes<uint64_t>(const GemmArgs<uint64_t> &);

}  // namespace ddg
