// Ring GEMM over Z_2^32 on the tensor cores with packed operands.
//
// Same contract and limb algebra as ring_gemm_tc.cu (GemmArgs):
//   C[b] = sign * ( A1[b] . (s1*B1[b] - B1m[b])  -  A2[b] . B2[b] ) + bias + Add[b]
// computed as P(P+1)/2 = 10 byte-plane products u8 x u8 -> s32
// (tcgen05.mma kind::i8) accumulated in tensor memory and recombined with
// shifts, exact modulo 2^32 while (s+1) * K * 255^2 < 2^31.
//
// What differs is how the operands reach shared memory.  The ring operands
// have row strides of 138 / 282 / 376 elements (not a multiple of 16 bytes),
// so they cannot be described by a TMA tensor map, and splitting them into
// byte planes inside the GEMM kept its loads, splits and MMAs in lock step.
// Here two streaming kernels first write the operands, split into byte
// planes and already in the canonical no-swizzle K-major UMMA layout, as
// contiguous blocks (one block = one row group or column tile for one
// 32-element K-step: exactly the bytes of one pipeline stage), and the GEMM
// moves each stage with two bulk copies (cp.async.bulk, mbarrier transaction
// counts) into a ring of 4 stages (3 with 64-column tiles):
//
//   warp 0       producer: one thread issues the bulk copies of stage ks
//                once the MMAs of the stage's previous use have released it;
//   warp 1       owns the tensor memory; one thread issues the limb MMAs of
//                a stage once its bytes have landed and commits them to the
//                stage's "empty" barrier, then commits the tile to "acc";
//   warps 2..5   epilogue: while the mainloop runs, the Add words of the
//                output tile into shared memory (asynchronous 4-byte copies,
//                one row per warp step) and its bias words; then per row
//                (TMEM lane) tcgen05.ld of the P partial sums, shift-add
//                into the tile with the bias; then coalesced stores of C.
//
// A block of A covers a row group of 128 rows; when the last rows of a
// matrix are a short tail (M % 128 <= 16, e.g. the 10 rows 128..137 of each
// 138-row sample of the Beaver products), the group also carries a 16-row
// tile of those rows and the CTA keeps a second set of accumulators for it,
// so the tail shares the B stages of the group instead of a second pass.
// Its MMAs still run at M = 128: the descriptor walks 128 rows from the tail
// tile's base, and the 112 rows past its 16 read other bytes of the same
// stage (their products land in accumulator rows that are never stored).
//
// Two CTAs per SM (about 108 KiB of shared memory, 256 tensor-memory columns
// each), so one CTA's epilogue overlaps the other's copies and MMAs.  Every
// mbarrier wait is bounded (about two seconds of %globaltimer); a wait that
// gives up sets the error word of ring_gemm_tc_check.  Before a CTA leaves,
// the producer waits (bounded) for the copies it has issued and for the MMA
// warp's releases of the last stages, warp 1 for the MMAs it has issued, and
// the CTA frees its tensor memory: no asynchronous arrive or copy may land in
// shared memory that the next CTA on the SM already uses.
#include "common.cuh"
#include "linear.cuh"

namespace ddg {

int ring_gemm_err_word(uint32_t **out);  // ring_gemm_tc.cu

namespace {

constexpr int PK_BM = 128;        // rows of a full tile (TMEM lanes)
constexpr int PK_BK = 32;         // K elements (bytes per plane row) per stage
constexpr int PK_THIN = 16;       // rows of a tail tile
constexpr int PK_THREADS = 192;   // 6 warps
constexpr uint32_t PK_NCOL = 256; // tensor-memory columns per CTA
constexpr uint64_t PK_WAIT_NS = 2000000000ull;
constexpr uint32_t PK_FULL_PLANE = PK_BM * PK_BK;  // 4096 bytes
constexpr uint32_t PK_THIN_PLANE = PK_THIN * PK_BK;  // 512 bytes
constexpr int PK_BAR_SLOTS = 4;   // barrier slots per kind (the most stages of either tile width)

// geometry of one packed GEMM (host and device)
struct PkGeom {
    int nks = 0;          // K-steps of 32 over the concatenated reduction [A1 | A2]
    int ng = 0;           // row groups per batch entry
    int thin = 0;         // the last group carries a 16-row tail tile
    int nnt = 0;          // column tiles
    int bn = 0;           // columns per tile
    uint32_t sa = 0;      // bytes of an A block: P * 4096 (+ P * 512 with a tail tile)
    uint32_t sb = 0;      // bytes of a B block: P * bn * 32
    int batches_b = 1;    // B blocks per batch entry (1 when B is shared by the batch)
};

template <typename T>
struct PkArgs {
    const uint8_t *apk, *bpk;
    int64_t b_batch_bytes;  // bytes between the B blocks of consecutive batch entries (0: shared)
    PkGeom g;
    int M, N;
    const T *bias, *Add;
    int64_t ldAdd, sAdd;
    T *C;
    int64_t ldc, sC;
};

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ uint64_t now_ns()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void bar_init(uint64_t *bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ bool bar_test(uint64_t *bar, uint32_t parity)
{
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// bounded wait for the completion of the phase with this parity
__device__ bool bar_wait(uint64_t *bar, uint32_t parity)
{
    const uint64_t t0 = now_ns();
    for (uint32_t it = 1; it < (1u << 26); ++it) {
        if (bar_test(bar, parity)) return true;
        if ((it & 255u) == 0 && now_ns() - t0 > PK_WAIT_NS) return false;
    }
    return false;
}

__device__ __forceinline__ void bar_expect_tx(uint64_t *bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

// global -> shared bulk copy (no tensor map, no multicast); completes `bytes` on bar
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes, uint64_t *bar)
{
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// shared-memory matrix descriptor, no swizzle, version 1 (the layout of ring_gemm_tc.cu)
__device__ __forceinline__ uint64_t desc(uint32_t addr, uint32_t lbo, uint32_t sbo)
{
    return uint64_t((addr >> 4) & 0x3FFFu) | (uint64_t((lbo >> 4) & 0x3FFFu) << 16) |
           (uint64_t((sbo >> 4) & 0x3FFFu) << 32) | (uint64_t(1) << 46);
}

// kind::i8, u8 x u8 -> s32, A and B K-major, M = 128
__host__ __device__ constexpr uint32_t idesc_i8(int bn)
{
    return (2u << 4) | (uint32_t(bn >> 3) << 17) | (uint32_t(PK_BM >> 4) << 24);
}

__device__ __forceinline__ void mma(uint32_t d_tmem, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(da), "l"(db), "r"(idesc), "r"(acc)
        : "memory");
}

__device__ __forceinline__ void commit(uint64_t *bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tld8(uint32_t taddr, uint32_t (&v)[8])
{
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(taddr)
                 : "memory");
}

__device__ __forceinline__ void tld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// byte offset of element (row r, K byte k) inside one plane of a K-major,
// no-swizzle tile: 8 x 16-byte core matrices, K-adjacent ones 128 bytes
// apart (LBO), row-adjacent ones 256 bytes apart (SBO)
__host__ __device__ constexpr uint32_t kmajor_off(int r, int k)
{
    return uint32_t((r >> 3) * 256 + (k >> 4) * 128 + (r & 7) * 16 + (k & 15));
}

// four consecutive 32-bit ring words -> their four byte planes (plane q = byte q of each)
__device__ __forceinline__ void planes4(const uint32_t (&e)[4], uint32_t (&p)[4])
{
    const uint32_t lo01 = __byte_perm(e[0], e[1], 0x5140), lo23 = __byte_perm(e[2], e[3], 0x5140);
    const uint32_t hi01 = __byte_perm(e[0], e[1], 0x7362), hi23 = __byte_perm(e[2], e[3], 0x7362);
    p[0] = __byte_perm(lo01, lo23, 0x5410);
    p[1] = __byte_perm(lo01, lo23, 0x7632);
    p[2] = __byte_perm(hi01, hi23, 0x5410);
    p[3] = __byte_perm(hi01, hi23, 0x7632);
}

// ---------------------------------------------------------------- packing

// A blocks: [batch][group][K-step] of sa bytes; inside, the full tile's P
// planes (4096 bytes each) then, for the last group with a tail, the tail
// tile's P planes (512 bytes each).  One thread = one row, four K elements.
__global__ void pk_pack_a(const __grid_constant__ GemmArgs<uint32_t> a, PkGeom g, uint8_t *apk)
{
    const int grp = blockIdx.y / g.nks, ks = blockIdx.y % g.nks, b = blockIdx.z;
    const int rows = PK_BM + ((g.thin && grp == g.ng - 1) ? PK_THIN : 0);
    const int r = blockIdx.x * 32 + (threadIdx.x >> 3), kq = threadIdx.x & 7;
    if (r >= rows) return;
    const int m = grp * PK_BM + r;
    const int ktot = a.A2 ? 2 * a.K : a.K;
    uint32_t e[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int k = ks * PK_BK + 4 * kq + i;
        uint32_t v = 0;
        if (m < a.M && k < ktot) {
            if (k < a.K) {
                const int64_t o = int64_t(b) * a.sA1 + int64_t(m) * a.lda1 + k;
                v = __ldg(a.A1 + o);
                if (a.A1b) v += __ldg(a.A1b + o);  // an opened operand held as two shares
            } else {
                v = __ldg(a.A2 + int64_t(b) * a.sA2 + int64_t(m) * a.lda2 + (k - a.K));
            }
        }
        e[i] = v;
    }
    uint32_t p[4];
    planes4(e, p);
    uint8_t *blk = apk + ((uint64_t(b) * g.ng + grp) * g.nks + ks) * g.sa;
    const bool tail = r >= PK_BM;
    uint8_t *base = tail ? blk + 4 * PK_FULL_PLANE : blk;
    const uint32_t plane = tail ? PK_THIN_PLANE : PK_FULL_PLANE;
    const uint32_t off = kmajor_off(tail ? r - PK_BM : r, 4 * kq);
#pragma unroll
    for (int q = 0; q < 4; q++) *reinterpret_cast<uint32_t *>(base + q * plane + off) = p[q];
}

// B blocks: [batch of B][column tile][K-step] of sb bytes, P planes of
// bn x 32 bytes, K-major (column n is the "row" of the layout).  The Beaver
// operand is formed here: rows k < K hold sign*(s1*B1 - B1m), rows K..2K-1
// hold -sign*B2.  One thread = one column, four K elements.
__global__ void pk_pack_b(const __grid_constant__ GemmArgs<uint32_t> a, PkGeom g, uint8_t *bpk)
{
    const int nt = blockIdx.x, ks = blockIdx.y, bb = blockIdx.z;
    const int nl = threadIdx.x % g.bn, kq = threadIdx.x / g.bn;
    const int n = nt * g.bn + nl;
    const int ktot = a.A2 ? 2 * a.K : a.K;
    const uint32_t sgn = a.sign, s1 = a.s1;
    uint32_t e[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int k = ks * PK_BK + 4 * kq + i;
        uint32_t v = 0;
        if (n < a.N && k < ktot) {
            if (k < a.K) {
                const int64_t o = int64_t(k) * a.ldb1 + n;
                if (a.B1) {
                    uint32_t b1 = __ldg(a.B1 + int64_t(bb) * a.sB1 + o);
                    if (a.B1b) b1 += __ldg(a.B1b + int64_t(bb) * a.sB1 + o);
                    v = s1 * b1;
                }
                if (a.B1m) v -= __ldg(a.B1m + int64_t(bb) * a.sB1m + o);
                v *= sgn;
            } else {
                const int64_t o = int64_t(bb) * a.sB2 + int64_t(k - a.K) * a.ldb2 + n;
                uint32_t b2 = __ldg(a.B2 + o);
                if (a.B2b) b2 += __ldg(a.B2b + o);
                v = 0u - sgn * b2;
            }
        }
        e[i] = v;
    }
    uint32_t p[4];
    planes4(e, p);
    // the block's four planes are one contiguous chunk of sb = 4 * bn * 32 bytes:
    // assemble it in shared memory, then store it as one 16-byte word per thread
    // (a thread's own 4-byte plane words land 16 bytes apart, 32 bytes per
    // 128-byte line and store)
    __shared__ __align__(16) uint8_t img[4 * 64 * PK_BK];
    const uint32_t plane = uint32_t(g.bn) * PK_BK;
    const uint32_t off = kmajor_off(nl, 4 * kq);
#pragma unroll
    for (int q = 0; q < 4; q++) *reinterpret_cast<uint32_t *>(img + q * plane + off) = p[q];
    __syncthreads();
    uint8_t *blk = bpk + ((uint64_t(bb) * g.nnt + nt) * g.nks + ks) * g.sb;
    reinterpret_cast<uint4 *>(blk)[threadIdx.x] = reinterpret_cast<const uint4 *>(img)[threadIdx.x];
}

// ---------------------------------------------------------------- the GEMM

// Output tile in shared memory, [rows][BN + 1] words (the odd row pitch keeps
// both the row-per-thread and the column-per-lane accesses conflict-free).
template <int BN>
struct PkTile {
    static constexpr int ROWS = BN == 32 ? PK_BM + PK_THIN : PK_BM;  // tail tiles come with BN = 32
    static constexpr int PITCH = BN + 1;
    static constexpr uint32_t BYTES = uint32_t((ROWS * PITCH + BN) * 4);  // the tile, then BN bias words
    static constexpr int STAGES = BN == 32 ? 4 : 3;  // two CTAs per SM either way
    static_assert(STAGES <= PK_BAR_SLOTS, "barrier slots");
};

__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

__device__ __forceinline__ void cp_async4(uint32_t dst, const void *src, uint32_t src_bytes)
{
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}

// epilogue warps, before the accumulators are ready: the Add words of the
// CTA's output tile into shared memory with asynchronous copies (all of them
// in flight at once; zero-filled outside the matrix), one row per warp step
// and one column per lane, and the bias words of its columns.  The copies
// are waited for (cp.async.wait_all) before the tile is read.
template <int BN>
__device__ __forceinline__ void pk_prefetch(const PkArgs<uint32_t> &a, uint32_t *tile, uint32_t *bias_s, int we,
                                            int lane, int b, int row0, int n0, int rows)
{
    const uint32_t *Add = a.Add ? a.Add + int64_t(b) * a.sAdd : nullptr;
    for (int r = we; r < rows; r += 4) {
        const int m = row0 + r;
#pragma unroll
        for (int c = lane; c < BN; c += 32) {
            const int n = n0 + c;
            const bool in = Add && m < a.M && n < a.N;
            cp_async4(smem_u32(tile + r * PkTile<BN>::PITCH + c), in ? Add + int64_t(m) * a.ldAdd + n : a.C,
                      in ? 4u : 0u);
        }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    if (we == 0) {
#pragma unroll
        for (int c = lane; c < BN; c += 32) bias_s[c] = (a.bias && n0 + c < a.N) ? __ldg(a.bias + n0 + c) : 0u;
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
}

// one accumulator set (tile t): this thread's row r of the tile gets
// sum_s S_s << 8s added, from TMEM lane quadrant q (the loads are warp-wide;
// only threads with `mine` write)
template <int BN>
__device__ __forceinline__ void pk_accumulate(uint32_t *tile, const uint32_t *bias_s, uint32_t tmem, int t, int q,
                                              int r, bool mine)
{
    constexpr int P = 4;
    const uint32_t lane_base = uint32_t(32 * q) << 16;
    uint32_t *row = tile + r * PkTile<BN>::PITCH;
#pragma unroll
    for (int c = 0; c < BN / 8; c++) {
        uint32_t acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
        for (int s = 0; s < P; s++) {
            uint32_t v[8];
            tld8(tmem + lane_base + uint32_t((t * P + s) * BN + 8 * c), v);
            tld_wait();
#pragma unroll
            for (int e = 0; e < 8; e++) acc[e] += v[e] << (8 * s);
        }
        if (mine) {
#pragma unroll
            for (int e = 0; e < 8; e++) row[8 * c + e] += acc[e] + bias_s[8 * c + e];
        }
    }
}

// the finished tile to C, one row per warp step, one column per lane
template <int BN>
__device__ __forceinline__ void pk_store(const PkArgs<uint32_t> &a, const uint32_t *tile, int we, int lane, int b,
                                         int row0, int n0, int rows)
{
    uint32_t *C = a.C + int64_t(b) * a.sC;
#pragma unroll 4
    for (int r = we; r < rows; r += 4) {
        const int m = row0 + r;
        if (m >= a.M) break;
#pragma unroll
        for (int c = lane; c < BN; c += 32) {
            const int n = n0 + c;
            if (n < a.N) C[int64_t(m) * a.ldc + n] = tile[r * PkTile<BN>::PITCH + c];
        }
    }
}

template <int BN>
__global__ void __launch_bounds__(PK_THREADS) ring_gemm_pk_kernel(const __grid_constant__ PkArgs<uint32_t> a,
                                                                  uint32_t *err)
{
    constexpr int P = 4, S = PkTile<BN>::STAGES;
    // barriers at fixed offsets for both tile widths: full[4] | empty[4] | acc | TMEM address | fail flag
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint64_t *const full = reinterpret_cast<uint64_t *>(smem_raw);
    uint64_t *const empty = full + PK_BAR_SLOTS;
    uint64_t *const accb = empty + PK_BAR_SLOTS;
    uint32_t *const s_tmem = reinterpret_cast<uint32_t *>(accb + 1);
    volatile int *const s_fail = reinterpret_cast<volatile int *>(s_tmem + 1);
    uint8_t *const stages = smem_raw + 128 + ((1024u - ((smem_u32(smem_raw) + 128u) & 1023u)) & 1023u);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nt = blockIdx.x, grp = blockIdx.y, b = blockIdx.z;
    const PkGeom &g = a.g;
    const bool tail = g.thin && grp == g.ng - 1;
    const int ntiles = tail ? 2 : 1;
    const uint32_t bytes_a = tail ? g.sa : P * PK_FULL_PLANE, bytes_b = g.sb;
    const uint32_t stage_bytes = g.sa + g.sb;
    const int nks = g.nks;
    uint32_t *const tile = reinterpret_cast<uint32_t *>(stages + S * stage_bytes);
    uint32_t *const bias_s = tile + PkTile<BN>::ROWS * PkTile<BN>::PITCH;

    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(s_tmem)),
                     "r"(PK_NCOL)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (threadIdx.x == 0) {
        for (int i = 0; i < S; i++) bar_init(full + i, 1), bar_init(empty + i, 1);
        bar_init(accb, 1);
        *s_fail = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem = *s_tmem;

    const uint8_t *ablk = a.apk + (uint64_t(b) * g.ng + grp) * uint64_t(nks) * g.sa;
    const uint8_t *bblk = a.bpk + int64_t(b) * a.b_batch_bytes + uint64_t(nt) * uint64_t(nks) * g.sb;
    bool mma_issued = false;

    if (warp == 0) {
        if (lane == 0) {
            int issued = 0;
            for (int ks = 0; ks < nks; ks++) {
                const int s = ks % S;
                if (ks >= S && !bar_wait(empty + s, uint32_t((ks / S - 1) & 1))) {
                    *s_fail = 1;
                    break;
                }
                if (*s_fail) break;
                const uint32_t dst = smem_u32(stages + s * stage_bytes);
                bar_expect_tx(full + s, bytes_a + bytes_b);
                bulk_g2s(dst, ablk + uint64_t(ks) * g.sa, bytes_a, full + s);
                bulk_g2s(dst + g.sa, bblk + uint64_t(ks) * g.sb, bytes_b, full + s);
                issued = ks + 1;
            }
            // the copies this thread issued land before the CTA may leave
            for (int k = issued > S ? issued - S : 0; k < issued; k++)
                if (!bar_wait(full + k % S, uint32_t((k / S) & 1))) *s_fail = 1;
            // and so do the MMA warp's releases of the last stages (tcgen05.commit arrives on
            // empty[]): an arrive that landed after the CTA left would hit the shared memory of
            // the next CTA on this SM
            for (int k = nks > S ? nks - S : 0; k < nks; k++)
                if (!bar_wait(empty + k % S, uint32_t((k / S) & 1))) *s_fail = 1;
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t IDESC = idesc_i8(BN);
            for (int ks = 0; ks < nks; ks++) {
                const int s = ks % S;
                if (!bar_wait(full + s, uint32_t((ks / S) & 1))) {
                    *s_fail = 1;
                    break;
                }
                fence_after();
                const uint32_t sa = smem_u32(stages + s * stage_bytes), sb = sa + g.sa;
                for (int t = 0; t < ntiles; t++) {
                    const uint32_t tb = t == 0 ? sa : sa + P * PK_FULL_PLANE;
                    const uint32_t ps = t == 0 ? PK_FULL_PLANE : PK_THIN_PLANE;
#pragma unroll
                    for (int i = 0; i < P; i++) {
                        const uint64_t da = desc(tb + i * ps, 128, 256);
#pragma unroll
                        for (int j = 0; j + i < P; j++) {
                            const uint64_t db = desc(sb + j * (BN * PK_BK), 128, 256);
                            mma(tmem + uint32_t((t * P + i + j) * BN), da, db, IDESC, (ks > 0 || i > 0) ? 1u : 0u);
                        }
                    }
                }
                commit(empty + s);
                mma_issued = true;
            }
            // completes once every MMA issued above has; the epilogue waits on it
            commit(accb);
        }
        __syncwarp();
    } else {
        // epilogue: bias + Add while the mainloop runs, then the accumulators, then C
        const int q = warp & 3, we = warp - 2;
        const int rows = PK_BM + (tail ? PK_THIN : 0), row0 = grp * PK_BM, n0 = nt * BN;
        pk_prefetch<BN>(a, tile, bias_s, we, lane, b, row0, n0, rows);
        epi_sync();
        const bool ok = __all_sync(0xffffffffu, bar_wait(accb, 0) ? 1 : 0) && !*s_fail;
        if (ok) {
            fence_after();
            pk_accumulate<BN>(tile, bias_s, tmem, 0, q, 32 * q + lane, true);
            // the tail tile's rows sit in TMEM lanes 0..15 of its accumulators
            if (tail && q == 0)
                pk_accumulate<BN>(tile, bias_s, tmem, 1, 0, PK_BM + (lane & (PK_THIN - 1)), lane < PK_THIN);
        } else {
            *s_fail = 1;
        }
        epi_sync();
        if (!*s_fail) pk_store<BN>(a, tile, we, lane, b, row0, n0, rows);
        __syncwarp();
    }
    fence_before();
    __syncthreads();
    if (warp == 1) {
        // MMAs still in flight after a failure finish before their memory is freed
        if (lane == 0 && mma_issued && !bar_wait(accb, 0)) *s_fail = 1;
        __syncwarp();
        fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(PK_NCOL) : "memory");
    }
    if (threadIdx.x == 0 && *s_fail) atomicOr(err, 4u);
}

constexpr int PK_SMEM_PAD = 128 + 1024;

PkGeom pk_geometry(const GemmArgs<uint32_t> &a)
{
    PkGeom g;
    constexpr int P = 4;
    const int ktot = a.A2 ? 2 * a.K : a.K;
    g.nks = (ktot + PK_BK - 1) / PK_BK;
    const int full = a.M / PK_BM, rem = a.M % PK_BM;
    g.thin = (full >= 1 && rem > 0 && rem <= PK_THIN) ? 1 : 0;
    g.ng = g.thin ? full : (a.M + PK_BM - 1) / PK_BM;
    g.bn = g.thin ? 32 : 64;  // 2 x 4 x 32 or 1 x 4 x 64 accumulator columns = PK_NCOL
    g.nnt = (a.N + g.bn - 1) / g.bn;
    g.sa = P * PK_FULL_PLANE + (g.thin ? P * PK_THIN_PLANE : 0);
    g.sb = uint32_t(P * g.bn * PK_BK);
    const bool b_shared = a.sB1 == 0 && a.sB1m == 0 && (!a.A2 || a.sB2 == 0);
    g.batches_b = b_shared ? 1 : a.batch;
    return g;
}

template <int BN>
int pk_launch(const PkArgs<uint32_t> &pa, int batch, uint32_t *err, cudaStream_t st)
{
    // stages for this tile width: 4 x (18432 + 4096) with a tail tile, 3 x (16384 + 8192) without
    constexpr uint32_t kMax = PK_SMEM_PAD + PkTile<BN>::STAGES * (4 * PK_FULL_PLANE + (BN == 32 ? 4 * PK_THIN_PLANE : 0) +
                                                                   4 * BN * PK_BK) + PkTile<BN>::BYTES;
    const uint32_t smem = PK_SMEM_PAD + PkTile<BN>::STAGES * (pa.g.sa + pa.g.sb) + PkTile<BN>::BYTES;
    DDG_CHECK(smem <= kMax, DDG_ERR_ARG, "packed GEMM: stage set of %u bytes exceeds %u", smem, kMax);
    auto kern = ring_gemm_pk_kernel<BN>;
    static thread_local int configured_dev = -1;
    int dev = 0;
    DDG_CUDA(cudaGetDevice(&dev));
    if (configured_dev != dev) {
        DDG_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kMax));
        configured_dev = dev;
    }
    dim3 grid(pa.g.nnt, pa.g.ng, batch);
    kern<<<grid, PK_THREADS, smem, st>>>(pa, err);
    note_launch();
    DDG_CUDA(cudaGetLastError());
    return DDG_OK;
}

}  // namespace

// C = sign * (A1 . (s1 B1 - B1m) - A2 . B2) + bias + Add over Z_2^32 through
// packed operands (scratch from the device's stream-ordered pool on st)
int ring_gemm_packed(const GemmArgs<uint32_t> &a, cudaStream_t st)
{
    DDG_CHECK(a.A1 && a.C && (!a.A2 || a.B2) && (a.B1 || a.B1m), DDG_ERR_ARG, "gemm: missing operand");
    DDG_CHECK(a.batch <= 65535, DDG_ERR_ARG, "gemm batch %d too large", a.batch);
    const PkGeom g = pk_geometry(a);
    DDG_CHECK(g.ng <= 65535, DDG_ERR_ARG, "gemm: M = %d too large", a.M);
    uint32_t *err = nullptr;
    DDG_TRY(ring_gemm_err_word(&err));
    const uint64_t abytes = uint64_t(a.batch) * g.ng * g.nks * g.sa;
    const uint64_t bbytes = uint64_t(g.batches_b) * g.nnt * g.nks * g.sb;
    // the A planes go to the caller's buffer when given (kept for later GEMMs of the same A)
    void *apk = a.apk_keep, *bpk = nullptr;
    const bool own_a = apk == nullptr;
    if (own_a) DDG_CUDA(cudaMallocAsync(&apk, abytes, st));
    if (cudaMallocAsync(&bpk, bbytes, st) != cudaSuccess) {
        if (own_a) cudaFreeAsync(apk, st);
        set_last_error("cudaMallocAsync(%llu) for the packed B operand failed", (unsigned long long)bbytes);
        return DDG_ERR_CUDA;
    }
    int rc = DDG_OK;
    if (own_a || !a.apk_ready) {
        const int rows = PK_BM + (g.thin ? PK_THIN : 0);
        dim3 grid((rows + 31) / 32, g.ng * g.nks, a.batch);
        pk_pack_a<<<grid, 256, 0, st>>>(a, g, static_cast<uint8_t *>(apk));
        note_launch();
        if (cudaGetLastError() != cudaSuccess) rc = DDG_ERR_CUDA;
    }
    if (rc == DDG_OK) {
        dim3 grid(g.nnt, g.nks, g.batches_b);
        pk_pack_b<<<grid, g.bn * 8, 0, st>>>(a, g, static_cast<uint8_t *>(bpk));
        note_launch();
        if (cudaGetLastError() != cudaSuccess) rc = DDG_ERR_CUDA;
    }
    if (rc == DDG_OK) {
        PkArgs<uint32_t> pa;
        pa.apk = static_cast<const uint8_t *>(apk), pa.bpk = static_cast<const uint8_t *>(bpk);
        pa.b_batch_bytes = g.batches_b > 1 ? int64_t(g.nnt) * g.nks * g.sb : 0;
        pa.g = g;
        pa.M = a.M, pa.N = a.N;
        pa.bias = a.bias, pa.Add = a.Add, pa.ldAdd = a.ldAdd, pa.sAdd = a.sAdd;
        pa.C = a.C, pa.ldc = a.ldc, pa.sC = a.sC;
        rc = g.bn == 32 ? pk_launch<32>(pa, a.batch, err, st) : pk_launch<64>(pa, a.batch, err, st);
    }
    if (rc != DDG_OK) set_last_error("packed ring GEMM launch failed");
    if (own_a) cudaFreeAsync(apk, st);
    cudaFreeAsync(bpk, st);
    return rc;
}

uint64_t ring_gemm_packed_a_bytes(const GemmArgs<uint32_t> &a)
{
    const PkGeom g = pk_geometry(a);
    return uint64_t(a.batch) * g.ng * g.nks * g.sa;
}

}  // namespace ddg
