// The affinity-branch graph as layers, and the three executors that walk it
// with the same op sequence and the same key sections in the same order:
//   SizeExec   - key bytes per party (the key-file layout),
//   DealerExec - GPU dealer: masks, correlated randomness, both parties' keys,
//   EvalExec   - one party: masked-public values, openings over its channel.
// The forward (affinity_graph) is the composition of the layer functions;
// the per-layer entry points (layers.cu) run the same functions one at a
// time, so a forward driven layer by layer reads (or writes) exactly the key
// sections of the whole forward.  Replaces DeepDTAGenAffinity::_forward
// (gpu_mpc/deepdtagen.h:183-222) with ddgSecureAdjNormEval in front of it
// (secure_adj_norm.h:394-659) and the key cursor of DDGOrcaBase /
// DDGOrcaBaseKeygen (ddg_orca_base.h:41-50, 326-374): every op reads (eval)
// or writes (dealer) the next 256-byte aligned key section.
#pragma once
#include <algorithm>
#include <vector>

#include "forward.cuh"
#include "gates.cuh"
#include "linear.cuh"
#include "ot.cuh"

namespace ddg {

enum Input { IN_X = 0, IN_ADJ = 1, IN_MASK = 2, IN_PROT = 3 };

template <typename T>
struct Tn {
    // eval: public masked value (v + v2 while an opening is still held as the
    // two parties' shares: EvalExec::val adds them); dealer: mask
    mutable T *v = nullptr;
    mutable const T *v2 = nullptr;
    uint64_t n = 0;
    const T *ms0 = nullptr;  // eval: own mask share; dealer: party 0's
    const T *ms1 = nullptr;  // dealer: party 1's
};

// ------------------------------------------------------------------ executors

template <typename T>
struct ExecBase {
    int B = 0, bw = 32, s = 12;
    int err = DDG_OK;
    uint32_t op = 1;
    uint64_t off = 0;  // key cursor
    uint64_t limit = ~uint64_t(0);  // key bytes the cursor may reach (dealer: the bound key regions)
    cudaStream_t st = nullptr;
    std::vector<void *> allocs;

    static uint64_t words(uint64_t n) { return n * sizeof(T); }
    uint64_t take(uint64_t bytes)
    {
        uint64_t o = align256(off);
        off = o + bytes;
        if (off > limit && err == DDG_OK) {
            set_last_error("key region exhausted: need %llu bytes, %llu bound", (unsigned long long)off,
                           (unsigned long long)limit);
            err = DDG_ERR_KEY;
        }
        return o;
    }
    bool ok(int status)
    {
        if (status != DDG_OK && err == DDG_OK) err = status;
        return err == DDG_OK;
    }
    void *alloc_bytes(uint64_t bytes)
    {
        if (err != DDG_OK) return nullptr;
        void *p = nullptr;
        cudaError_t e = cudaMallocAsync(&p, bytes ? bytes : 16, st);
        if (e != cudaSuccess) {
            set_last_error("cudaMallocAsync(%llu) failed: %s", (unsigned long long)bytes, cudaGetErrorString(e));
            err = DDG_ERR_CUDA;
            return nullptr;
        }
        allocs.push_back(p);
        return p;
    }
    T *alloc(uint64_t n) { return static_cast<T *>(alloc_bytes(n * sizeof(T))); }
    void free_all()
    {
        for (void *p : allocs) cudaFreeAsync(p, st);
        allocs.clear();
    }
};

// ---- size planner: advances the cursor exactly like the other two

template <typename T>
struct SizeExec : ExecBase<T> {
    using ExecBase<T>::take;
    using ExecBase<T>::words;
    T *mark = reinterpret_cast<T *>(uintptr_t(256));
    Tn<T> mk(uint64_t n) { Tn<T> t; t.n = n; return t; }
    Tn<T> reveal_input(int, uint64_t n) { take(words(n)); auto t = mk(n); t.ms0 = mark; return t; }
    Tn<T> reveal_degree(uint64_t rows, int) { take(words(rows)); auto t = mk(rows); t.ms0 = mark; return t; }
    Tn<T> reveal_public(int, uint64_t n) { return mk(n); }
    Tn<T> lut(const Tn<T> &d)
    {
        take(relu_backend() == DDG_RELU_TT ? tt_lut_layout(this->bw, d.n).bytes : lut_layout(this->bw, d.n).bytes);
        auto t = mk(d.n);
        t.ms0 = mark;
        return t;
    }
    void ensure_ms(Tn<T> &t) { if (!t.ms0) { take(words(t.n)); t.ms0 = mark; } }
    Tn<T> mul(Tn<T> &a, Tn<T> &b, Bcast, const EwShape &sh) { ensure_ms(a); ensure_ms(b); take(words(sh.n)); return mk(sh.n); }
    Tn<T> matmul(Tn<T> &A, Tn<T> &H, int K)
    {
        ensure_ms(A); ensure_ms(H);
        uint64_t n = uint64_t(this->B) * NMAX * K;
        take(words(n));
        return mk(n);
    }
    Tn<T> fc(const Tn<T> &, int l, int M) { uint64_t n = uint64_t(M) * LAYER_OUT[l]; take(words(n)); return mk(n); }
    Tn<T> gate(int kind, const Tn<T> &x) { take(gate_layout(kind, this->bw, this->s, x.n).bytes); return mk(x.n); }
    void pool_split(const Tn<T> &, int cnt, Tn<T> &even, Tn<T> &diff)
    {
        even = mk(uint64_t(this->B) * (cnt / 2) * POOL);
        diff = even;
    }
    Tn<T> pool_merge(const Tn<T> &, const Tn<T> &, const Tn<T> &, int cnt)
    {
        return mk(uint64_t(this->B) * (cnt / 2 + (cnt & 1)) * POOL);
    }
    Tn<T> concat(const Tn<T> &a, const Tn<T> &b) { return mk(a.n + b.n); }
    void output(const Tn<T> &o) { take(words(o.n)); }
};

// ---- dealer (GPU): the masks travel through the graph like values do

template <typename T>
struct DealerExec : ExecBase<T> {
    using ExecBase<T>::take;
    using ExecBase<T>::words;
    using ExecBase<T>::alloc;
    using ExecBase<T>::ok;
    uint64_t seed = 0;
    AesKey dk;
    uint8_t *k0 = nullptr, *k1 = nullptr;
    const DevWeights *w = nullptr;

    T *rand(uint64_t n)
    {
        T *r = alloc(n);
        if (r) ok(prg_fill<T>(r, n, dk, this->op++, P_MASK, this->st));
        return r;
    }
    // writes shares of v into a new section of both keys
    void share_section(const T *v, uint64_t n, const T **s0, const T **s1)
    {
        uint64_t o = take(words(n));
        T *a = reinterpret_cast<T *>(k0 + o), *b = reinterpret_cast<T *>(k1 + o);
        if (this->err == DDG_OK) ok(split_shares<T>(v, n, dk, this->op++, P_SHARE, a, b, this->st));
        if (s0) *s0 = a;
        if (s1) *s1 = b;
    }
    Tn<T> reveal_input(int, uint64_t n)
    {
        Tn<T> t;
        t.n = n;
        t.v = rand(n);
        share_section(t.v, n, &t.ms0, &t.ms1);
        return t;
    }
    Tn<T> reveal_degree(uint64_t rows, int) { return reveal_input(IN_ADJ, rows); }
    Tn<T> reveal_public(int, uint64_t n)
    {
        Tn<T> t;
        t.n = n;
        t.v = alloc(n);
        if (t.v) ok(cudaMemsetAsync(t.v, 0, words(n), this->st) == cudaSuccess ? DDG_OK : DDG_ERR_CUDA);
        return t;
    }
    Tn<T> lut(const Tn<T> &d)
    {
        Tn<T> t;
        t.n = d.n;
        if (relu_backend() == DDG_RELU_TT) {
            TtLutLayout L = tt_lut_layout(this->bw, d.n);
            uint64_t o = take(L.bytes);
            t.v = rand(d.n);
            if (this->err == DDG_OK)
                ok(tt_lut_keygen<T>(L, dk, this->op++, d.v, t.v, static_cast<const T *>(w->table), k0 + o, k1 + o,
                                    this->st));
            t.ms0 = reinterpret_cast<const T *>(k0 + o + L.rout);
            t.ms1 = reinterpret_cast<const T *>(k1 + o + L.rout);
            return t;
        }
        LutLayout L = lut_layout(this->bw, d.n);
        uint64_t o = take(L.bytes);
        t.v = rand(d.n);
        if (this->err == DDG_OK) ok(lut_keygen<T>(L, dk, this->op++, d.v, t.v, k0 + o, k1 + o, this->st));
        t.ms0 = reinterpret_cast<const T *>(k0 + o + L.rout);
        t.ms1 = reinterpret_cast<const T *>(k1 + o + L.rout);
        return t;
    }
    void ensure_ms(Tn<T> &t)
    {
        if (!t.ms0) share_section(t.v, t.n, &t.ms0, &t.ms1);
    }
    Tn<T> mul(Tn<T> &a, Tn<T> &b, Bcast bc, const EwShape &sh)
    {
        ensure_ms(a), ensure_ms(b);
        Tn<T> t;
        t.n = sh.n;
        t.v = rand(sh.n);
        T *Z = alloc(sh.n);
        if (this->err == DDG_OK) ok(beaver_ew_z<T>(sh, bc, a.v, b.v, t.v, Z, this->st));
        share_section(Z, sh.n, nullptr, nullptr);
        return t;
    }
    Tn<T> matmul(Tn<T> &A, Tn<T> &H, int K)
    {
        ensure_ms(A), ensure_ms(H);
        const uint64_t n = uint64_t(this->B) * NMAX * K;
        Tn<T> t;
        t.n = n;
        t.v = rand(n);
        T *Z = alloc(n);
        if (this->err == DDG_OK) {
            GemmArgs<T> g;
            g.M = NMAX, g.N = K, g.K = NMAX, g.batch = this->B;
            g.A1 = A.v, g.lda1 = NMAX, g.sA1 = int64_t(NMAX) * NMAX;
            g.B1 = H.v, g.ldb1 = K, g.sB1 = int64_t(NMAX) * K;
            g.Add = t.v, g.ldAdd = K, g.sAdd = int64_t(NMAX) * K;
            g.C = Z, g.ldc = K, g.sC = int64_t(NMAX) * K;
            ok(ring_gemm<T>(g, this->st));
        }
        share_section(Z, n, nullptr, nullptr);
        return t;
    }
    Tn<T> fc(const Tn<T> &x, int l, int M)
    {
        const int N = LAYER_OUT[l], K = LAYER_IN[l];
        const uint64_t n = uint64_t(M) * N;
        Tn<T> t;
        t.n = n;
        t.v = rand(n);
        T *C = alloc(n);
        if (this->err == DDG_OK) {
            GemmArgs<T> g;  // C = r_y - r_x . W
            g.M = M, g.N = N, g.K = K;
            g.A1 = x.v, g.lda1 = K;
            g.B1 = static_cast<const T *>(w->W[l]), g.ldb1 = N;
            g.sign = T(0) - T(1);
            g.Add = t.v, g.ldAdd = N;
            g.C = C, g.ldc = N;
            ok(ring_gemm<T>(g, this->st));
        }
        share_section(C, n, nullptr, nullptr);
        return t;
    }
    Tn<T> gate(int kind, const Tn<T> &x)
    {
        GateLayout L = gate_layout(kind, this->bw, this->s, x.n);
        uint64_t o = take(L.bytes);
        Tn<T> t;
        t.n = x.n;
        t.v = alloc(x.n);
        if (this->err == DDG_OK) ok(gate_keygen(L, seed, this->op, x.v, t.v, k0 + o, k1 + o, this->st));
        this->op++;
        return t;
    }
    void pool_split(const Tn<T> &cur, int cnt, Tn<T> &even, Tn<T> &diff)
    {
        const uint64_t n = uint64_t(this->B) * (cnt / 2) * POOL;
        even.n = diff.n = n;
        even.v = alloc(n), diff.v = alloc(n);
        if (this->err == DDG_OK) ok(::ddg::pool_split<T>(cur.v, even.v, diff.v, this->B, cnt, POOL, this->st));
    }
    Tn<T> pool_merge(const Tn<T> &even, const Tn<T> &r, const Tn<T> &cur, int cnt)
    {
        Tn<T> t;
        t.n = uint64_t(this->B) * (cnt / 2 + (cnt & 1)) * POOL;
        t.v = alloc(t.n);
        if (this->err == DDG_OK) ok(::ddg::pool_merge<T>(even.v, r.v, cur.v, t.v, this->B, cnt, POOL, this->st));
        return t;
    }
    Tn<T> concat(const Tn<T> &a, const Tn<T> &b)
    {
        Tn<T> t;
        t.n = a.n + b.n;
        t.v = alloc(t.n);
        if (this->err == DDG_OK) ok(concat_rows<T>(a.v, b.v, t.v, this->B, PROT, PROT, this->st));
        return t;
    }
    void output(const Tn<T> &o)
    {
        uint64_t off = take(words(o.n));
        if (this->err != DDG_OK) return;
        // the output mask goes to both evaluators in the clear (ddg_orca_base.h:511-517)
        ok(cudaMemcpyAsync(k0 + off, o.v, words(o.n), cudaMemcpyDeviceToDevice, this->st) == cudaSuccess
               ? DDG_OK : DDG_ERR_CUDA);
        ok(cudaMemcpyAsync(k1 + off, o.v, words(o.n), cudaMemcpyDeviceToDevice, this->st) == cudaSuccess
               ? DDG_OK : DDG_ERR_CUDA);
    }
};

// ---- one party's online evaluation

template <typename T>
struct EvalExec : ExecBase<T> {
    using ExecBase<T>::take;
    using ExecBase<T>::words;
    using ExecBase<T>::alloc;
    using ExecBase<T>::ok;
    Party *P = nullptr;
    int p = 0;
    // openings stay as (own share, peer share) until a consumer needs one value
    // (the level-1 and round-2 kernels of the truth-table gates, the packed
    // GEMM's operand packing, the elementwise Beaver product and the pool
    // levels add them on load); only where the peer's bytes stay valid to the
    // end of the forward (Channel::peer_stable)
    bool lazy = false;
    // the packed A operand of the Beaver products A_hat . H: the same A_hat (and
    // its mask share) in every GCN layer, so its byte planes are packed once
    uint8_t *ah_pk = nullptr;
    const T *ah_ms0 = nullptr;
    uint64_t ah_bytes = 0;
    const T *in[4] = {};
    cudaEvent_t in_ready[4] = {};  // host inputs: copy-stream event to wait on before first use
    T *out = nullptr;

    void wait_input(int which)
    {
        if (in_ready[which] && this->err == DDG_OK)
            ok(cudaStreamWaitEvent(this->st, in_ready[which], 0) == cudaSuccess ? DDG_OK : DDG_ERR_CUDA);
        in_ready[which] = nullptr;
    }

    const uint8_t *key_at(uint64_t bytes)
    {
        uint64_t o = take(bytes);
        if (this->err == DDG_OK && this->off > P->key_bytes) {
            set_last_error("key region exhausted: need %llu bytes, %llu bound", (unsigned long long)this->off,
                           (unsigned long long)P->key_bytes);
            this->err = DDG_ERR_KEY;
        }
        return P->keys + o;
    }
    const T *peer_of(const void *send, uint64_t bytes)
    {
        if (this->err != DDG_OK) return nullptr;
        void *recv = P->chan->needs_recv_buffer() ? this->alloc_bytes(bytes) : nullptr;
        const void *peer = nullptr;
        ok(P->chan->exchange(p, this->st, send, bytes, recv, &peer));
        return static_cast<const T *>(peer);
    }
    T *open(const T *share, uint64_t n)
    {
        const T *peer = peer_of(share, words(n));
        T *pub = alloc(n);
        if (this->err == DDG_OK) ok(ew_add<T>(pub, share, peer, n, this->st));
        return pub;
    }
    // open `share` into t (t.n set): the sum now, or the two addends when lazy
    void open_to(Tn<T> &t, const T *share)
    {
        if (!lazy) {
            t.v = open(share, t.n);
            return;
        }
        t.v2 = peer_of(share, words(t.n));
        t.v = const_cast<T *>(share);
    }
    // the value of t as one array (adds a held opening once, in place)
    const T *val(const Tn<T> &t)
    {
        if (t.v2 && this->err == DDG_OK) {
            T *m = alloc(t.n);
            if (this->err == DDG_OK) ok(ew_add<T>(m, t.v, t.v2, t.n, this->st));
            t.v = m, t.v2 = nullptr;
        }
        return t.v;
    }
    Tn<T> reveal_input(int which, uint64_t n)
    {
        Tn<T> t;
        t.n = n;
        t.ms0 = reinterpret_cast<const T *>(key_at(words(n)));
        T *sh = alloc(n);
        wait_input(which);
        if (this->err == DDG_OK) ok(ew_add<T>(sh, in[which], t.ms0, n, this->st));
        open_to(t, sh);
        return t;
    }
    Tn<T> reveal_degree(uint64_t rows, int cols)
    {
        Tn<T> t;
        t.n = rows;
        const T *ms = reinterpret_cast<const T *>(key_at(words(rows)));
        t.ms0 = ms;
        T *sh = alloc(rows);
        wait_input(IN_ADJ);
        if (this->err == DDG_OK) ok(rowsum_plus<T>(in[IN_ADJ], ms, sh, rows, cols, this->st));
        open_to(t, sh);
        return t;
    }
    Tn<T> reveal_public(int which, uint64_t n)
    {
        Tn<T> t;
        t.n = n;
        wait_input(which);
        t.v = open(in[which], n);
        return t;
    }
    Tn<T> lut(const Tn<T> &d)
    {
        Tn<T> t;
        t.n = d.n;
        T *sh = alloc(d.n);
        if (relu_backend() == DDG_RELU_TT) {
            TtLutLayout L = tt_lut_layout(this->bw, d.n);
            const uint8_t *k = key_at(L.bytes);
            const T *dv = val(d);
            if (this->err == DDG_OK) ok(tt_lut_eval<T>(L, dv, k, sh, this->st));
            open_to(t, sh);
            t.ms0 = reinterpret_cast<const T *>(k + L.rout);
            return t;
        }
        LutLayout L = lut_layout(this->bw, d.n);
        const uint8_t *k = key_at(L.bytes);
        const T *dv = val(d);
        if (this->err == DDG_OK)
            ok(lut_eval<T>(L, p, dv, static_cast<const T *>(P->w.table), k, sh, this->st));
        open_to(t, sh);
        t.ms0 = reinterpret_cast<const T *>(k + L.rout);
        return t;
    }
    void ensure_ms(Tn<T> &t)
    {
        if (!t.ms0) t.ms0 = reinterpret_cast<const T *>(key_at(words(t.n)));
    }
    Tn<T> mul(Tn<T> &a, Tn<T> &b, Bcast bc, const EwShape &sh)
    {
        ensure_ms(a), ensure_ms(b);
        const T *Z = reinterpret_cast<const T *>(key_at(words(sh.n)));
        T *s = alloc(sh.n);
        if (this->err == DDG_OK) ok(beaver_ew<T>(p, sh, bc, a.v, b.v, a.ms0, b.ms0, Z, s, this->st, a.v2, b.v2));
        Tn<T> t;
        t.n = sh.n;
        open_to(t, s);
        return t;
    }
    Tn<T> matmul(Tn<T> &A, Tn<T> &H, int K)
    {
        ensure_ms(A), ensure_ms(H);
        const uint64_t n = uint64_t(this->B) * NMAX * K;
        const T *Z = reinterpret_cast<const T *>(key_at(words(n)));
        T *s = alloc(n);
        if (this->err == DDG_OK) {
            // p0 * A_hat . H_hat - A_hat . [r_H] - [r_A] . H_hat + Z   (per sample)
            GemmArgs<T> g;
            g.M = NMAX, g.N = K, g.K = NMAX, g.batch = this->B;
            g.A1 = A.v, g.A1b = A.v2, g.lda1 = NMAX, g.sA1 = int64_t(NMAX) * NMAX;
            g.B1 = H.v, g.B1b = H.v2, g.ldb1 = K, g.sB1 = int64_t(NMAX) * K, g.s1 = p == 0 ? T(1) : T(0);
            g.B1m = H.ms0, g.sB1m = int64_t(NMAX) * K;
            g.A2 = A.ms0, g.lda2 = NMAX, g.sA2 = int64_t(NMAX) * NMAX;
            g.B2 = H.v, g.B2b = H.v2, g.ldb2 = K, g.sB2 = int64_t(NMAX) * K;
            g.Add = Z, g.ldAdd = K, g.sAdd = int64_t(NMAX) * K;
            g.C = s, g.ldc = K, g.sC = int64_t(NMAX) * K;
            const uint64_t ab = ring_gemm_a_pack_bytes<T>(g);
            if (ab) {
                const bool same = ah_pk && ah_ms0 == A.ms0 && ah_bytes == ab;
                if (!same) ah_pk = static_cast<uint8_t *>(this->alloc_bytes(ab)), ah_ms0 = A.ms0, ah_bytes = ab;
                g.apk_keep = ah_pk, g.apk_ready = same ? 1 : 0;
            }
            if (this->err == DDG_OK) ok(ring_gemm<T>(g, this->st));
        }
        Tn<T> t;
        t.n = n;
        open_to(t, s);
        return t;
    }
    Tn<T> fc(const Tn<T> &x, int l, int M)
    {
        const int N = LAYER_OUT[l], K = LAYER_IN[l];
        const uint64_t n = uint64_t(M) * N;
        const T *C = reinterpret_cast<const T *>(key_at(words(n)));
        const T *s = C;  // party 1's share is its key words
        if (p == 0) {
            T *s0 = alloc(n);
            if (this->err == DDG_OK) {
                GemmArgs<T> g;  // x_hat . W + b<<s + C
                g.M = M, g.N = N, g.K = K;
                g.A1 = x.v, g.A1b = x.v2, g.lda1 = K;
                g.B1 = static_cast<const T *>(P->w.W[l]), g.ldb1 = N;
                g.bias = static_cast<const T *>(P->w.b2s[l]);
                g.Add = C, g.ldAdd = N;
                g.C = s0, g.ldc = N;
                ok(ring_gemm<T>(g, this->st));
            }
            s = s0;
        }
        Tn<T> t;
        t.n = n;
        open_to(t, s);
        return t;
    }
    // AND-tree gates.  OT kinds: garbled digit tables first (one message);
    // TT kinds start from their own digit truth tables.  Then one AND-tree
    // level per round; the last level writes the masked comparison bits in the
    // split-gate layout (bits_hi = [lt | eq], bits_lo = lt; GATE_LRS_TT only
    // bits_lo), opened and consumed by round 2.
    Tn<T> gate_digits(const GateLayout &L, const uint8_t *k, const Tn<T> &x)
    {
        const OtPlan &Pl = gate_digit_plan(L);
        const uint64_t n = x.n, nw = (n + 31) / 32;
        const OtScratch sc = ot_scratch_bytes(L);
        void *state = this->alloc_bytes(sc.state);
        uint32_t *tri = nullptr;
        const uint32_t *ptab = nullptr;
        if (L.ot) val(x);  // the OT garble step reads one input array
        if (L.ot) {
            uint32_t *tab = static_cast<uint32_t *>(this->alloc_bytes(sc.tables));
            tri = static_cast<uint32_t *>(this->alloc_bytes(sc.tri));
            if (this->err == DDG_OK) ok(ot_garble(L, p, x.v, k, tab, state, tri, this->st));
            ptab = reinterpret_cast<const uint32_t *>(peer_of(tab, sc.tables));
        }
        const void *oo = nullptr, *po = nullptr;
        for (int l = 1; l <= Pl.levels; l++) {
            // openings of 1, 2 or 4 bytes per element, exchanged in whole 32-bit words
            const uint64_t ob = (uint64_t(ot_open_bytes(L, l)) * n + 3) & ~uint64_t(3);
            void *o = this->alloc_bytes(ob);
            if (this->err == DDG_OK)
                ok(ot_level(L, p, l, k, ptab, oo, po, state, tri, o, nullptr, nullptr, this->st, x.v, x.v2));
            po = peer_of(o, ob);
            oo = o;
        }
        // opened bit arrays: hi lt, hi eq, lo lt (split round 2) / full lt, lo lt / lo lt only
        const int nb = Pl.mode == PLAN_TT_FULL ? 2 : Pl.nd[0] ? 3 : 1;
        uint32_t *bits = static_cast<uint32_t *>(this->alloc_bytes(4 * nw * nb));
        uint32_t *bl = bits + (nb - 1) * nw;
        if (this->err == DDG_OK)
            ok(ot_level(L, p, Pl.levels + 1, k, ptab, oo, po, state, tri, nullptr, nb > 1 ? bits : nullptr, bl,
                        this->st, x.v, x.v2));
        const uint32_t *peer = reinterpret_cast<const uint32_t *>(peer_of(bits, 4 * nw * nb));
        T *sh = alloc(n);
        if (this->err == DDG_OK)
            ok(gate_round2(L, p, x.v, nb > 1 ? bits : nullptr, nb > 1 ? peer : nullptr, bl,
                           peer ? peer + (nb - 1) * nw : nullptr, k, sh, this->st, x.v2));
        Tn<T> t;
        t.n = n;
        open_to(t, sh);
        return t;
    }
    Tn<T> gate(int kind, const Tn<T> &x)
    {
        GateLayout L = gate_layout(kind, this->bw, this->s, x.n);
        const uint8_t *k = key_at(L.bytes);
        if (L.ot || L.tt) return gate_digits(L, k, x);
        val(x);  // the DCF rounds read one input array
        const uint64_t nw = (x.n + 31) / 32;
        // split gates also open the equality bits, three-part splits the middle DCF's two bits
        const int nh = L.hi ? (L.mid ? 4 : (L.H.eq ? 2 : 1)) : 0;
        const int nb = nh + (L.lo ? 1 : 0);
        uint32_t *bits = static_cast<uint32_t *>(this->alloc_bytes(4 * nw * nb));
        uint32_t *bh = L.hi ? bits : nullptr, *bl = L.lo ? bits + nh * nw : nullptr;
        if (this->err == DDG_OK) ok(gate_round1(L, x.v, k, bh, bl, this->st));
        const uint32_t *peer = reinterpret_cast<const uint32_t *>(peer_of(bits, 4 * nw * nb));
        const uint32_t *ph = L.hi ? peer : nullptr, *pl = L.lo ? peer + nh * nw : nullptr;
        T *s = alloc(x.n);
        if (this->err == DDG_OK) ok(gate_round2(L, p, x.v, bh, ph, bl, pl, k, s, this->st));
        Tn<T> t;
        t.n = x.n;
        open_to(t, s);
        return t;
    }
    void pool_split(const Tn<T> &cur, int cnt, Tn<T> &even, Tn<T> &diff)
    {
        const uint64_t n = uint64_t(this->B) * (cnt / 2) * POOL;
        even.n = diff.n = n;
        even.v = alloc(n), diff.v = alloc(n);
        if (this->err == DDG_OK)
            ok(::ddg::pool_split<T>(cur.v, even.v, diff.v, this->B, cnt, POOL, this->st, cur.v2));
    }
    Tn<T> pool_merge(const Tn<T> &even, const Tn<T> &r, const Tn<T> &cur, int cnt)
    {
        Tn<T> t;
        t.n = uint64_t(this->B) * (cnt / 2 + (cnt & 1)) * POOL;
        t.v = alloc(t.n);
        if (this->err == DDG_OK)
            ok(::ddg::pool_merge<T>(even.v, r.v, cur.v, t.v, this->B, cnt, POOL, this->st, r.v2, cur.v2));
        return t;
    }
    Tn<T> concat(const Tn<T> &a, const Tn<T> &b)
    {
        Tn<T> t;
        t.n = a.n + b.n;
        const T *av = val(a), *bv = val(b);
        t.v = alloc(t.n);
        if (this->err == DDG_OK) ok(concat_rows<T>(av, bv, t.v, this->B, PROT, PROT, this->st));
        return t;
    }
    void output(const Tn<T> &o)
    {
        const T *r = reinterpret_cast<const T *>(key_at(words(o.n)));
        const T *ov = val(o);
        out = alloc(o.n);
        if (this->err == DDG_OK) ok(unmask_ars<T>(ov, r, out, o.n, this->s, this->st));
    }
};

// ------------------------------------------------------------------ the graph, layer by layer

// gate kinds of the selected comparison backend (relu_backend, relu_parts)
struct GraphKinds {
    int relu, relu_ars, lrs;
};
inline GraphKinds graph_kinds()
{
    const int be = relu_backend();
    const bool three = relu_parts() == 3, ot = be == DDG_RELU_OT, tt = be == DDG_RELU_TT;
    GraphKinds k;
    k.relu = tt ? GATE_RELU_TTF : ot ? GATE_RELU_OT : three ? GATE_RELU_SPLIT3 : GATE_RELU_SPLIT;
    k.relu_ars = tt ? GATE_RELU_ARS_TTF : ot ? GATE_RELU_ARS_OT : three ? GATE_RELU_ARS_SPLIT3 : GATE_RELU_ARS_SPLIT;
    k.lrs = tt ? GATE_LRS_TT : GATE_LRS_SPLIT;
    return k;
}

// secure adjacency normalisation (ddgSecureAdjNormEval, secure_adj_norm.h:394-659):
// reveal the raw adjacency leaf and its masked degree, t = LUT[deg],
// A_hat = floor(A * t_i * t_j / 2^s) (mul #1 without truncation, mul #2 + exact floor, :498-651)
template <typename T, class E>
Tn<T> adjnorm_layer(E &x)
{
    const uint64_t nA = uint64_t(x.B) * NMAX * NMAX;
    Tn<T> A = x.reveal_input(IN_ADJ, nA);
    Tn<T> D = x.reveal_degree(uint64_t(x.B) * NMAX, NMAX);
    Tn<T> t = x.lut(D);
    EwShape sh;
    sh.n = nA, sh.R = NMAX, sh.C = NMAX;
    Tn<T> L = x.mul(A, t, BC_ROW, sh);
    Tn<T> W = x.mul(L, t, BC_COL, sh);
    return x.gate(graph_kinds().lrs, W);
}

// GCN layer l, aggregate first (GCNLayer::forward, gcn_layer.h:99-116):
// H' = ReLU(floor((floor(A_hat . H / 2^s) . W + b<<s) / 2^s))
template <typename T, class E>
Tn<T> gcn_layer(E &x, Tn<T> &Ah, Tn<T> &H, int l)
{
    const GraphKinds k = graph_kinds();
    Tn<T> Pm = x.matmul(Ah, H, LAYER_IN[l]);
    Tn<T> AX = x.gate(k.lrs, Pm);
    Tn<T> Z = x.fc(AX, l, x.B * NMAX);
    return x.gate(k.relu_ars, Z);
}

// the masked node features H3 * mask, floored (deepdtagen.h:198, DDGOrca::mul ddg_orca.h:43-63)
template <typename T, class E>
Tn<T> mask_mul_layer(E &x, Tn<T> &H, Tn<T> &M)
{
    EwShape shm;
    shm.n = H.n;
    Tn<T> prod = x.mul(H, M, BC_NONE, shm);
    return x.gate(graph_kinds().lrs, prod);
}

// masked global max-pool over the node axis (MaskedMaxPoolLayer::_forward,
// masked_maxpool_layer.h:47-166): levels of even + ReLU(odd - even) over
// node pairs (2p, 2p+1), an odd last node carried up; (B,138,376) -> (B,376)
template <typename T, class E>
Tn<T> maxpool_layer(E &x, Tn<T> cur)
{
    const int relu = graph_kinds().relu;
    int cnt = NMAX;
    while (cnt > 1) {
        Tn<T> even, diff;
        x.pool_split(cur, cnt, even, diff);
        Tn<T> r = x.gate(relu, diff);
        cur = x.pool_merge(even, r, cur, cnt);
        cnt = cnt / 2 + (cnt & 1);
    }
    return cur;
}

// activation after a head FC layer
enum FcAct { FC_ACT_NONE = 0, FC_ACT_RELU = 1, FC_ACT_TRUNC = 2 };

// one FC layer of the head (FC<T> through DDGOrcaBase::matmul 4-arg,
// ddg_orca_base.h:208-271): x . W + b<<s, then ReLU(floor(./2^s)) (act
// RELU), floor(./2^s) (TRUNC) or nothing (NONE, the output layer)
template <typename T, class E>
Tn<T> fc_layer(E &x, Tn<T> &in, int l, int rows, int act)
{
    Tn<T> z = x.fc(in, l, rows);
    if (act == FC_ACT_RELU) return x.gate(graph_kinds().relu_ars, z);
    if (act == FC_ACT_TRUNC) return x.gate(GATE_ARS, z);
    return z;
}

// GPUConcat (deepdtagen.h:45-100): reveal the public protein leaf (mask 0)
// and interleave [d2 | protein] per row
template <typename T, class E>
Tn<T> concat_protein_layer(E &x, const Tn<T> &d2)
{
    Tn<T> P = x.reveal_public(IN_PROT, uint64_t(x.B) * PROT);
    return x.concat(d2, P);
}

template <typename T, class E>
void affinity_graph(E &x)
{
    const int B = x.B;
    const uint64_t nX = uint64_t(B) * NMAX * FEAT, nM = uint64_t(B) * NMAX * POOL;
    // leaves: x, mask, raw adjacency and its masked degree, the public protein
    // (deepdtagen_inference.cu:503-529 registerLeaf; secure_adj_norm.h:414-493)
    // Each leaf is revealed right before its first use, so that host inputs
    // still in flight on the party's copy stream (features, mask, protein)
    // overlap the layers before it; the key sections follow the same order.
    Tn<T> Ah = adjnorm_layer<T>(x);
    Tn<T> H = x.reveal_input(IN_X, nX);
    for (int l = 0; l < 3; l++) H = gcn_layer<T>(x, Ah, H, l);
    Tn<T> M = x.reveal_input(IN_MASK, nM);
    Tn<T> cur = maxpool_layer<T>(x, mask_mul_layer<T>(x, H, M));
    // head (deepdtagen.h:209-220)
    Tn<T> d1 = fc_layer<T>(x, cur, 3, B, FC_ACT_RELU);
    Tn<T> d2 = fc_layer<T>(x, d1, 4, B, FC_ACT_TRUNC);
    Tn<T> f = concat_protein_layer<T>(x, d2);
    for (int l = 5; l < 8; l++) f = fc_layer<T>(x, f, l, B, FC_ACT_RELU);
    Tn<T> o = fc_layer<T>(x, f, 8, B, FC_ACT_NONE);
    x.output(o);
}

}  // namespace ddg
