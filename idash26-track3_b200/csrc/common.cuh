// Shared definitions of the DeepDTAGen 2PC library: status codes, ring types,
// key-layout arithmetic.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cstdio>
#include <vector>
#include <cuda_runtime.h>

#include "../../include/ddg_fss.h"
#include "digit_plan.cuh"

namespace ddg {

inline uint64_t align256(uint64_t x) { return (x + 255u) & ~uint64_t(255); }

// status-returning CUDA check: records the first failure and returns from the
// calling function with DDG_ERR_CUDA
#define DDG_CUDA(expr)                                                                        \
    do {                                                                                      \
        cudaError_t _e = (expr);                                                              \
        if (_e != cudaSuccess) {                                                              \
            ::ddg::set_last_error("%s:%d %s: %s", __FILE__, __LINE__, #expr, cudaGetErrorString(_e)); \
            return DDG_ERR_CUDA;                                                              \
        }                                                                                     \
    } while (0)

#define DDG_CHECK(cond, code, ...)              \
    do {                                        \
        if (!(cond)) {                          \
            ::ddg::set_last_error(__VA_ARGS__); \
            return (code);                      \
        }                                       \
    } while (0)

#define DDG_TRY(expr)                \
    do {                             \
        int _s = (expr);             \
        if (_s != DDG_OK) return _s; \
    } while (0)

void set_last_error(const char *fmt, ...);

// number of kernels this library launched (all devices, all threads)
void note_launch();
uint64_t launch_count();
// a replayed CUDA graph runs kernels that were counted when it was captured
void add_launches(uint64_t n);
// record a timing event on st: an ordinary record, or, while st is being
// captured into a CUDA graph, an event-record node that records at every replay
int record_timing_event(cudaEvent_t e, cudaStream_t st);

// Optional timing of the comparison kernels (DCF gate round 1; OT garble and
// AND-tree levels): when a thread has a sink installed, every such launch is
// bracketed by CUDA events on its stream together with its algorithmic bytes
// and AES blocks.  The events come from a pool that is created once and
// reused, and the records are read back only when the caller asks for the
// totals, so that a timed forward spends no host time on them after its
// stream has drained.
struct DcfTiming {
    struct Rec {
        cudaEvent_t a, b;
        double bytes, aes, evals;
        bool done;  // the end event was recorded
    };
    std::vector<cudaEvent_t> pool;  // timing events, reused once their records are read back
    size_t used = 0;
    std::vector<Rec> recs;          // launches not yet read back
    bool enabled = false;
    int take(cudaEvent_t *e);
    void release();                 // destroy the pool (its events must be complete)
};
// keep freed stream-ordered allocations of the device's default memory pool
// cached (release threshold = infinity), once per device (forward.cu)
int keep_pool_memory(int device);

DcfTiming *dcf_timing_sink();
void set_dcf_timing_sink(DcfTiming *t);

// brackets one comparison-kernel launch with events when a sink is installed
struct TimedLaunch {
    DcfTiming *sink = nullptr;
    size_t idx = 0;
    int begin(cudaStream_t st);
    int end(cudaStream_t st, double bytes, double aes, double evals);
};

// ---------------------------------------------------------------- key layouts

// gate kinds (the comparison-based nonlinear layers)
// The RELU*_SPLIT kinds compute the same functions as GATE_RELU / GATE_RELU_ARS
// but split the (n-1)-bit comparison into a DCF-with-equality over the upper
// n-1-s bits and the s-bit low DCF: 1{x<a} = 1{U<A} ^ (1{U==A} & 1{V<B}).
// GATE_LRS_SPLIT computes GATE_LRS with its s-bit carry comparison split the
// same way into V1 (upper s - s2 bits, DCF with equality) and V2 (low s2 =
// min(7, s-1) bits, plain DCF): 2 instead of s-6 AES-128 per element.
// GATE_RELU_SPLIT3 / GATE_RELU_ARS_SPLIT3 split the (n-1)-bit comparison in
// three: U1 (upper bits, DCF with equality), U2 (the SPLIT3_MID bits above the
// low s bits, DCF with equality) and V (the low s bits, plain DCF):
// 1{x<a} = c1 + e1*(c2 + e2*cL), every sum exclusive.  15 AES per element at
// bw=32 instead of 20, for 40 / 80 key words instead of 16 / 32.
// GATE_RELU_OT / GATE_RELU_ARS_OT compute GATE_RELU_SPLIT / GATE_RELU_ARS_SPLIT
// with the same dealer words and round 2, but obtain the split comparison bits
// from garbled radix-16 digit tables and a Beaver AND tree (ot.cuh) instead of
// DCF keys: no AES tree, a few key bytes per element, more rounds.
// GATE_RELU_TT / GATE_RELU_ARS_TT / GATE_LRS_TT compute GATE_RELU_SPLIT /
// GATE_RELU_ARS_SPLIT / GATE_LRS with their dealer words and round 2; the
// comparison bits come from dealer-shared digit truth tables read at the
// public digits of x_hat and the same AND tree (no AES, no table message).
enum GateKind {
    GATE_RELU = 0, GATE_RELU_ARS = 1, GATE_ARS = 2, GATE_LRS = 3, GATE_RELU_SPLIT = 4, GATE_RELU_ARS_SPLIT = 5,
    GATE_LRS_SPLIT = 6, GATE_RELU_SPLIT3 = 7, GATE_RELU_ARS_SPLIT3 = 8, GATE_RELU_OT = 9, GATE_RELU_ARS_OT = 10,
    GATE_RELU_TT = 11, GATE_RELU_ARS_TT = 12, GATE_LRS_TT = 13, GATE_RELU_TTF = 14, GATE_RELU_ARS_TTF = 15,
    GATE_KIND_END = 16
};
constexpr int SPLIT3_MID = 6;
constexpr int SPLIT3_NMONO = 19;  // dealer-bit monomials of the three-part DReLU bit

inline bool gate_is_split3(int kind) { return kind == GATE_RELU_SPLIT3 || kind == GATE_RELU_ARS_SPLIT3; }
inline bool gate_is_ot(int kind) { return kind == GATE_RELU_OT || kind == GATE_RELU_ARS_OT; }
inline bool gate_is_tt(int kind)
{
    return kind == GATE_RELU_TT || kind == GATE_RELU_ARS_TT || kind == GATE_LRS_TT || kind == GATE_RELU_TTF ||
           kind == GATE_RELU_ARS_TTF;
}
// the kind whose dealer words and round 2 a gate uses
__host__ __device__ inline int gate_word_kind(int kind)
{
    switch (kind) {
    case GATE_RELU_OT:
    case GATE_RELU_TT: return GATE_RELU_SPLIT;
    case GATE_RELU_ARS_OT:
    case GATE_RELU_ARS_TT: return GATE_RELU_ARS_SPLIT;
    case GATE_LRS_TT: return GATE_LRS;
    case GATE_RELU_TTF: return GATE_RELU;
    case GATE_RELU_ARS_TTF: return GATE_RELU_ARS;
    default: return kind;
    }
}
// the digit plan of a TT kind
inline int tt_mode_of(int kind)
{
    return kind == GATE_LRS_TT ? PLAN_TT_LRS : (kind == GATE_RELU_TTF || kind == GATE_RELU_ARS_TTF) ? PLAN_TT_FULL
                                                                                                : PLAN_TT_RELU;
}
inline OtPlan tt_plan_of(int kind, int bw, int s) { return digit_plan(bw, s, tt_mode_of(kind)); }
// the high DCF has an equality output (three round-1 bit arrays, five with a middle DCF)
inline bool gate_is_split(int kind)
{
    return kind == GATE_RELU_SPLIT || kind == GATE_RELU_ARS_SPLIT || kind == GATE_LRS_SPLIT || gate_is_split3(kind);
}
inline bool gate_has_hi(int kind) { return kind != GATE_LRS; }
inline bool gate_has_lo(int kind) { return kind != GATE_RELU; }
inline int gate_nwords(int kind)
{
    switch (gate_word_kind(kind)) {
    case GATE_RELU: return 4;
    case GATE_RELU_ARS: return 8;
    case GATE_ARS: return 6;
    case GATE_RELU_SPLIT: return 16;
    case GATE_RELU_ARS_SPLIT: return 32;
    case GATE_LRS_SPLIT: return 7;
    case GATE_RELU_SPLIT3: return 40;
    case GATE_RELU_ARS_SPLIT3: return 80;
    default: return 4;
    }
}
// bits of the low part V2 of a GATE_LRS_SPLIT carry comparison
__host__ __device__ inline int lrs_split_lo_bits(int s) { return s - 1 < 7 ? s - 1 : 7; }
// domain bits of the high DCF and the shift that brings its input bits down
inline int gate_hi_bits(int kind, int bw, int s)
{
    if (kind == GATE_LRS_SPLIT) return s - lrs_split_lo_bits(s);
    if (gate_is_split3(kind)) return bw - 1 - s - SPLIT3_MID;
    return gate_is_split(kind) ? bw - 1 - s : bw - 1;
}
inline int gate_hi_shift(int kind, int s)
{
    if (kind == GATE_LRS_SPLIT) return lrs_split_lo_bits(s);
    if (gate_is_split3(kind)) return s + SPLIT3_MID;
    return gate_is_split(kind) ? s : 0;
}
// domain bits of the low DCF
inline int gate_lo_bits(int kind, int s) { return kind == GATE_LRS_SPLIT ? lrs_split_lo_bits(s) : s; }

// DCF key arrays of N elements, structure-of-arrays, every array 256-byte aligned:
//   root[N] (16 B) | cw[L][N] (16 B, level-major) | leaf[N] (16 B) | mu[ceil(N/32)] (u32 bits)
//   [| mu_eq[ceil(N/32)] for a DCF with equality output]
// A plain DCF's leaf covers the low min(d,7) bits (1 bit per slot); a DCF
// with equality output covers the low 6 bits with 2 bits per slot.
struct DcfLayout {
    int d = 0, L = 0;
    bool eq = false;
    uint64_t root = 0, cw = 0, leaf = 0, mu = 0, mu_eq = 0, end = 0;
};

inline int dcf_levels(int d) { return d > 7 ? d - 7 : 0; }
inline int dcfeq_levels(int d) { return d > 6 ? d - 6 : 0; }

inline DcfLayout dcf_layout(int d, uint64_t n, uint64_t base, bool eq = false)
{
    DcfLayout l;
    l.d = d;
    l.eq = eq;
    l.L = eq ? dcfeq_levels(d) : dcf_levels(d);
    l.root = align256(base);
    l.cw = align256(l.root + 16 * n);
    l.leaf = align256(l.cw + 16 * n * uint64_t(l.L));
    l.mu = align256(l.leaf + 16 * n);
    l.mu_eq = eq ? align256(l.mu + 4 * ((n + 31) / 32)) : 0;
    l.end = align256((eq ? l.mu_eq : l.mu) + 4 * ((n + 31) / 32));
    return l;
}

// one gate op: [hi DCF over hi_bits] [mid DCF] [lo DCF over lo_bits] [nwords x N ring words]
// The hi DCF reads bits [hi_shift, hi_shift + H.d) of x_hat, the middle DCF
// (three-part split kinds) bits [s, s + SPLIT3_MID), the lo DCF bits [0, Lo.d).
// OT kinds: [ot_ks: 44 u32 round keys] [ot_recv: ot_gmax x N bytes] [ot_c0: N u32] [words]
// TT kinds: [tt_tables: tt_rows x N u32] [tt_tri: tt_triw x N u32] [words]
struct GateLayout {
    int kind = 0, bw = 0, s = 0, hi_shift = 0;
    uint64_t n = 0;
    bool hi = false, mid = false, lo = false, ot = false, tt = false;
    DcfLayout H, Mi, Lo;
    int ot_gmax = 0, tt_rows = 0, tt_triw = 0;
    uint64_t ot_ks = 0, ot_recv = 0, ot_c0 = 0, tt_tables = 0, tt_tri = 0;
    int nwords = 0;
    uint64_t words = 0, bytes = 0;
};

// digits party 0 garbles in an OT gate over an n-bit ring at scale s (the
// larger half of ceil((n-1-s)/4) + ceil(s/4) radix-16 digits)
inline int ot_gmax(int bw, int s) { return ((bw - 1 - s + 3) / 4 + (s + 3) / 4 + 1) / 2; }

inline GateLayout gate_layout(int kind, int bw, int s, uint64_t n, uint64_t base = 0)
{
    GateLayout g;
    g.kind = kind, g.bw = bw, g.s = s, g.n = n;
    uint64_t off = align256(base);
    if (gate_is_tt(kind)) {
        const OtPlan P = tt_plan_of(kind, bw, s);
        g.tt = true;
        g.tt_rows = P.rows, g.tt_triw = P.tri_words();
        g.tt_tables = off;
        g.tt_tri = align256(g.tt_tables + 4 * uint64_t(g.tt_rows) * n);
        off = align256(g.tt_tri + 4 * uint64_t(g.tt_triw) * n);
        g.nwords = gate_nwords(kind);
        g.words = off;
        g.bytes = align256(g.words + uint64_t(g.nwords) * n * uint64_t(bw / 8)) - align256(base);
        return g;
    }
    if (gate_is_ot(kind)) {
        g.ot = true;
        g.ot_gmax = ot_gmax(bw, s);
        g.ot_ks = off;
        g.ot_recv = align256(g.ot_ks + 176);
        g.ot_c0 = align256(g.ot_recv + uint64_t(g.ot_gmax) * n);
        off = align256(g.ot_c0 + 4 * n);
        g.nwords = gate_nwords(kind);
        g.words = off;
        g.bytes = align256(g.words + uint64_t(g.nwords) * n * uint64_t(bw / 8)) - align256(base);
        return g;
    }
    g.hi = gate_has_hi(kind);
    g.lo = gate_has_lo(kind);
    if (g.hi) {
        g.H = dcf_layout(gate_hi_bits(kind, bw, s), n, off, gate_is_split(kind));
        g.hi_shift = gate_hi_shift(kind, s);
        off = g.H.end;
    }
    g.mid = gate_is_split3(kind);
    if (g.mid) {
        g.Mi = dcf_layout(SPLIT3_MID, n, off, true);
        off = g.Mi.end;
    }
    if (g.lo) {
        g.Lo = dcf_layout(gate_lo_bits(kind, s), n, off);
        off = g.Lo.end;
    }
    g.nwords = gate_nwords(kind);
    g.words = align256(off);
    g.bytes = align256(g.words + uint64_t(g.nwords) * n * uint64_t(bw / 8)) - align256(base);
    return g;
}

// DCF view handed to kernels (device pointers)
struct DcfView {
    const uint8_t *root, *cw, *leaf;
    const uint32_t *mu, *mu_eq;
};

struct DcfOut {
    uint8_t *root0, *root1, *cw0, *cw1, *leaf0, *leaf1;
    uint32_t *mu0, *mu1;
};

inline DcfView dcf_view(const uint8_t *key, const DcfLayout &l)
{
    return DcfView{key + l.root, key + l.cw, key + l.leaf, reinterpret_cast<const uint32_t *>(key + l.mu),
                   l.eq ? reinterpret_cast<const uint32_t *>(key + l.mu_eq) : nullptr};
}

// dealer PRG purposes
enum Purpose : uint32_t {
    P_HI_S0 = 1, P_HI_DELTA = 2, P_LO_S0 = 3, P_LO_DELTA = 4, P_ROUT = 5, P_BITS = 6,
    P_MASK = 8,    // input / output masks of linear ops
    P_MID_S0 = 9, P_MID_DELTA = 10,  // middle DCF of the three-part split gates
                                     // 0x100..0x12f: OT gates (ot.cuh), 0x140..: TT gates
    P_SHARE = 16,  // share0 of dealer word k uses purpose P_SHARE + k (k < 80)
    P_TT_LUT = 0x180,  // party 0's truth-table LUT entries
};

}  // namespace ddg
