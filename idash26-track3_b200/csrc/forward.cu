// The online graph of the affinity branch, walked by three executors that see
// the same op sequence and the same key sections in the same order:
//   SizeExec   - key bytes per party (the key-file layout),
//   DealerExec - GPU dealer: masks, correlated randomness, both parties' keys,
//   EvalExec   - one party: masked-public values, openings over its channel.
// Replaces DeepDTAGenAffinity::_forward (gpu_mpc/deepdtagen.h:183-222) with
// ddgSecureAdjNormEval in front of it (secure_adj_norm.h:394-659) and the
// key cursor of DDGOrcaBase / DDGOrcaBaseKeygen (ddg_orca_base.h:41-50,
// 326-374): every op reads (eval) or writes (dealer) the next 256-byte aligned
// key section.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <vector>

#include "forward.cuh"
#include "gates.cuh"
#include "ot.cuh"
#include "linear.cuh"

namespace ddg {

enum Input { IN_X = 0, IN_ADJ = 1, IN_MASK = 2, IN_PROT = 3 };

template <typename T>
struct Tn {
    T *v = nullptr;          // eval: public masked value; dealer: mask
    uint64_t n = 0;
    const T *ms0 = nullptr;  // eval: own mask share; dealer: party 0's
    const T *ms1 = nullptr;  // dealer: party 1's
};

// ------------------------------------------------------------------ weights

int DevWeights::load(const int64_t *h_blob, uint64_t n, int bw_, int s_, int device_)
{
    DDG_CHECK(n == weights_elems(), DDG_ERR_ARG, "weights blob has %llu int64 values, expected %llu",
              (unsigned long long)n, (unsigned long long)weights_elems());
    release();
    bw = bw_, s = s_, device = device_;
    DDG_CUDA(cudaSetDevice(device));
    const int es = bw / 8;
    int64_t *tmp = nullptr;
    DDG_CUDA(cudaMalloc(&tmp, n * sizeof(int64_t)));
    DDG_CUDA(cudaMemcpy(tmp, h_blob, n * sizeof(int64_t), cudaMemcpyHostToDevice));
    uint64_t off = 0;
    int st = DDG_OK;
    for (int l = 0; l < NLAYERS && st == DDG_OK; l++) {
        const uint64_t nw = uint64_t(LAYER_IN[l]) * LAYER_OUT[l], nb = LAYER_OUT[l];
        DDG_CUDA(cudaMalloc(&W[l], nw * es));
        DDG_CUDA(cudaMalloc(&b2s[l], nb * es));
        if (bw == 32) {
            st = i64_to_ring<uint32_t>(tmp + off, (uint32_t *)W[l], nw, 0, nullptr);
            if (st == DDG_OK) st = i64_to_ring<uint32_t>(tmp + off + nw, (uint32_t *)b2s[l], nb, s, nullptr);
        } else {
            st = i64_to_ring<uint64_t>(tmp + off, (uint64_t *)W[l], nw, 0, nullptr);
            if (st == DDG_OK) st = i64_to_ring<uint64_t>(tmp + off + nw, (uint64_t *)b2s[l], nb, s, nullptr);
        }
        off += nw + nb;
    }
    // public 8-bit degree table: t[0] = 0, t[d] = llround(2^s / sqrt(d)), d <= NMAX (secure_adj_norm.h:139-184)
    uint64_t tab[256] = {0};
    for (int d = 1; d <= NMAX; d++) tab[d] = uint64_t(std::llround(std::ldexp(1.0, s) / std::sqrt(double(d))));
    DDG_CUDA(cudaMalloc(&table, 256 * es));
    if (bw == 32) {
        uint32_t t32[256];
        for (int i = 0; i < 256; i++) t32[i] = uint32_t(tab[i]);
        DDG_CUDA(cudaMemcpy(table, t32, sizeof(t32), cudaMemcpyHostToDevice));
    } else {
        DDG_CUDA(cudaMemcpy(table, tab, sizeof(tab), cudaMemcpyHostToDevice));
    }
    DDG_CUDA(cudaDeviceSynchronize());
    cudaFree(tmp);
    return st;
}

void DevWeights::release()
{
    for (int l = 0; l < NLAYERS; l++) {
        if (W[l]) cudaFree(W[l]);
        if (b2s[l]) cudaFree(b2s[l]);
        W[l] = b2s[l] = nullptr;
    }
    if (table) cudaFree(table);
    table = nullptr;
}

int Party::ensure_copy_stream()
{
    if (copy_stream) return DDG_OK;
    DDG_CUDA(cudaStreamCreateWithFlags(&copy_stream, cudaStreamNonBlocking));
    for (auto &ev : in_ev) DDG_CUDA(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
    return DDG_OK;
}

void Party::release_inputs()
{
    for (int i = 0; i < 4; i++)
        if (in_buf[i]) cudaFree(in_buf[i]), in_buf[i] = nullptr, in_cap[i] = 0;
    for (auto &ev : in_ev)
        if (ev) cudaEventDestroy(ev), ev = nullptr;
    if (copy_stream) cudaStreamDestroy(copy_stream), copy_stream = nullptr;
}

int Party::ensure_input(int which, uint64_t bytes)
{
    if (in_cap[which] >= bytes) return DDG_OK;
    if (in_buf[which]) cudaFree(in_buf[which]);
    in_buf[which] = nullptr;
    DDG_CUDA(cudaMalloc(&in_buf[which], bytes ? bytes : 16));
    in_cap[which] = bytes;
    return DDG_OK;
}

int keep_pool_memory(int device)
{
    static std::atomic<bool> done[64] = {};
    if (device >= 0 && device < 64 && done[device].load()) return DDG_OK;
    cudaMemPool_t pool;
    DDG_CUDA(cudaDeviceGetDefaultMemPool(&pool, device));
    uint64_t thr = ~uint64_t(0);
    DDG_CUDA(cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &thr));
    if (device >= 0 && device < 64) done[device].store(true);
    return DDG_OK;
}

// ------------------------------------------------------------------ executors

template <typename T>
struct ExecBase {
    int B = 0, bw = 32, s = 12;
    int err = DDG_OK;
    uint32_t op = 1;
    uint64_t off = 0;  // key cursor
    cudaStream_t st = nullptr;
    std::vector<void *> allocs;

    static uint64_t words(uint64_t n) { return n * sizeof(T); }
    uint64_t take(uint64_t bytes)
    {
        uint64_t o = align256(off);
        off = o + bytes;
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
    Tn<T> reveal_input(int which, uint64_t n)
    {
        Tn<T> t;
        t.n = n;
        t.ms0 = reinterpret_cast<const T *>(key_at(words(n)));
        T *sh = alloc(n);
        wait_input(which);
        if (this->err == DDG_OK) ok(ew_add<T>(sh, in[which], t.ms0, n, this->st));
        t.v = open(sh, n);
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
        t.v = open(sh, rows);
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
            if (this->err == DDG_OK) ok(tt_lut_eval<T>(L, d.v, k, sh, this->st));
            t.v = open(sh, d.n);
            t.ms0 = reinterpret_cast<const T *>(k + L.rout);
            return t;
        }
        LutLayout L = lut_layout(this->bw, d.n);
        const uint8_t *k = key_at(L.bytes);
        if (this->err == DDG_OK)
            ok(lut_eval<T>(L, p, d.v, static_cast<const T *>(P->w.table), k, sh, this->st));
        t.v = open(sh, d.n);
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
        if (this->err == DDG_OK) ok(beaver_ew<T>(p, sh, bc, a.v, b.v, a.ms0, b.ms0, Z, s, this->st));
        Tn<T> t;
        t.n = sh.n;
        t.v = open(s, sh.n);
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
            g.A1 = A.v, g.lda1 = NMAX, g.sA1 = int64_t(NMAX) * NMAX;
            g.B1 = H.v, g.ldb1 = K, g.sB1 = int64_t(NMAX) * K, g.s1 = p == 0 ? T(1) : T(0);
            g.B1m = H.ms0, g.sB1m = int64_t(NMAX) * K;
            g.A2 = A.ms0, g.lda2 = NMAX, g.sA2 = int64_t(NMAX) * NMAX;
            g.B2 = H.v, g.ldb2 = K, g.sB2 = int64_t(NMAX) * K;
            g.Add = Z, g.ldAdd = K, g.sAdd = int64_t(NMAX) * K;
            g.C = s, g.ldc = K, g.sC = int64_t(NMAX) * K;
            ok(ring_gemm<T>(g, this->st));
        }
        Tn<T> t;
        t.n = n;
        t.v = open(s, n);
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
                g.A1 = x.v, g.lda1 = K;
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
        t.v = open(s, n);
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
        if (L.ot) {
            uint32_t *tab = static_cast<uint32_t *>(this->alloc_bytes(sc.tables));
            tri = static_cast<uint32_t *>(this->alloc_bytes(sc.tri));
            if (this->err == DDG_OK) ok(ot_garble(L, p, x.v, k, tab, state, tri, this->st));
            ptab = reinterpret_cast<const uint32_t *>(peer_of(tab, sc.tables));
        }
        const uint32_t *oo = nullptr, *po = nullptr;
        for (int l = 1; l <= Pl.levels; l++) {
            uint32_t *o = static_cast<uint32_t *>(this->alloc_bytes(4 * n));
            if (this->err == DDG_OK)
                ok(ot_level(L, p, l, k, ptab, oo, po, state, tri, o, nullptr, nullptr, this->st, x.v));
            po = reinterpret_cast<const uint32_t *>(peer_of(o, 4 * n));
            oo = o;
        }
        // opened bit arrays: hi lt, hi eq, lo lt (split round 2) / full lt, lo lt / lo lt only
        const int nb = Pl.mode == PLAN_TT_FULL ? 2 : Pl.nd[0] ? 3 : 1;
        uint32_t *bits = static_cast<uint32_t *>(this->alloc_bytes(4 * nw * nb));
        uint32_t *bl = bits + (nb - 1) * nw;
        if (this->err == DDG_OK)
            ok(ot_level(L, p, Pl.levels + 1, k, ptab, oo, po, state, tri, nullptr, nb > 1 ? bits : nullptr, bl,
                        this->st, x.v));
        const uint32_t *peer = reinterpret_cast<const uint32_t *>(peer_of(bits, 4 * nw * nb));
        T *sh = alloc(n);
        if (this->err == DDG_OK)
            ok(gate_round2(L, p, x.v, nb > 1 ? bits : nullptr, nb > 1 ? peer : nullptr, bl,
                           peer ? peer + (nb - 1) * nw : nullptr, k, sh, this->st));
        Tn<T> t;
        t.n = n;
        t.v = open(sh, n);
        return t;
    }
    Tn<T> gate(int kind, const Tn<T> &x)
    {
        GateLayout L = gate_layout(kind, this->bw, this->s, x.n);
        const uint8_t *k = key_at(L.bytes);
        if (L.ot || L.tt) return gate_digits(L, k, x);
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
        t.v = open(s, x.n);
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
        const T *r = reinterpret_cast<const T *>(key_at(words(o.n)));
        out = alloc(o.n);
        if (this->err == DDG_OK) ok(unmask_ars<T>(o.v, r, out, o.n, this->s, this->st));
    }
};

// ------------------------------------------------------------------ the graph

// comparison split of the ReLU gates: 3 parts (default; fewest AES) or 2
// (smaller keys: 94.8 vs 111.8 MB per sample and party at bw=32).  Key sizes
// differ, so dealer and evaluators must run with the same setting.
static std::atomic<int> g_relu_parts{3};
void set_relu_parts(int parts) { g_relu_parts.store(parts == 2 ? 2 : 3); }
static int relu_parts(int) { return g_relu_parts.load(); }
// comparison backend of the ReLU (and truncation) gates: dealer truth tables
// per digit with a Beaver AND tree (GATE_RELU*_TT and GATE_LRS_TT at the
// truncation sites; default: no AES online), OT-leaf digit tables with the
// same tree (GATE_RELU*_OT: 2 AES and ~8 key bytes per element and party
// besides the words) or DCF keys (split per relu_parts)
static std::atomic<int> g_relu_backend{DDG_RELU_TT};
void set_relu_backend(int backend)
{
    g_relu_backend.store(backend == DDG_RELU_OT || backend == DDG_RELU_TT ? backend : DDG_RELU_DCF);
}
int relu_backend() { return g_relu_backend.load(); }

template <typename T, class E>
static void affinity_graph(E &x)
{
    const int B = x.B;
    const int be = g_relu_backend.load();
    const bool three = relu_parts(x.bw) == 3, ot = be == DDG_RELU_OT, tt = be == DDG_RELU_TT;
    const int RELU = tt ? GATE_RELU_TTF : ot ? GATE_RELU_OT : three ? GATE_RELU_SPLIT3 : GATE_RELU_SPLIT;
    const int RELU_ARS = tt ? GATE_RELU_ARS_TTF : ot ? GATE_RELU_ARS_OT : three ? GATE_RELU_ARS_SPLIT3 : GATE_RELU_ARS_SPLIT;
    const int LRS = tt ? GATE_LRS_TT : GATE_LRS_SPLIT;
    const uint64_t nX = uint64_t(B) * NMAX * FEAT, nA = uint64_t(B) * NMAX * NMAX, nM = uint64_t(B) * NMAX * POOL;
    // leaves: x, mask, raw adjacency and its masked degree, the public protein
    // (deepdtagen_inference.cu:503-529 registerLeaf; secure_adj_norm.h:414-493)
    // Each leaf is revealed right before its first use, so that host inputs
    // still in flight on the party's copy stream (features, mask, protein)
    // overlap the layers before it; the key sections follow the same order.
    Tn<T> A = x.reveal_input(IN_ADJ, nA);
    Tn<T> D = x.reveal_degree(uint64_t(B) * NMAX, NMAX);
    // A_hat = floor(A * t_i * t_j / 2^s), t = LUT[deg] (secure_adj_norm.h:498-651)
    Tn<T> t = x.lut(D);
    EwShape sh;
    sh.n = nA, sh.R = NMAX, sh.C = NMAX;
    Tn<T> L = x.mul(A, t, BC_ROW, sh);
    Tn<T> W = x.mul(L, t, BC_COL, sh);
    Tn<T> Ah = x.gate(LRS, W);
    // GCN x3, aggregate first (gcn_layer.h:107-116)
    Tn<T> X = x.reveal_input(IN_X, nX);
    Tn<T> H = X;
    for (int l = 0; l < 3; l++) {
        Tn<T> Pm = x.matmul(Ah, H, LAYER_IN[l]);
        Tn<T> AX = x.gate(LRS, Pm);
        Tn<T> Z = x.fc(AX, l, B * NMAX);
        H = x.gate(RELU_ARS, Z);
    }
    // masked global max-pool (deepdtagen.h:198-202, masked_maxpool_layer.h:72-126)
    EwShape shm;
    shm.n = nM;
    Tn<T> M = x.reveal_input(IN_MASK, nM);
    Tn<T> prod = x.mul(H, M, BC_NONE, shm);
    Tn<T> cur = x.gate(LRS, prod);
    int cnt = NMAX;
    while (cnt > 1) {
        Tn<T> even, diff;
        x.pool_split(cur, cnt, even, diff);
        Tn<T> r = x.gate(RELU, diff);
        cur = x.pool_merge(even, r, cur, cnt);
        cnt = cnt / 2 + (cnt & 1);
    }
    // head (deepdtagen.h:209-220)
    Tn<T> d1 = x.gate(RELU_ARS, x.fc(cur, 3, B));
    Tn<T> d2 = x.gate(GATE_ARS, x.fc(d1, 4, B));
    Tn<T> P = x.reveal_public(IN_PROT, uint64_t(B) * PROT);
    Tn<T> f = x.concat(d2, P);
    for (int l = 5; l < 8; l++) f = x.gate(RELU_ARS, x.fc(f, l, B));
    Tn<T> o = x.fc(f, 8, B);
    x.output(o);
}

// ------------------------------------------------------------------ entry points

uint64_t forward_key_bytes(int bw, int s, int B)
{
    if (bw == 32) {
        SizeExec<uint32_t> e;
        e.B = B, e.bw = bw, e.s = s;
        affinity_graph<uint32_t>(e);
        return align256(e.off);
    }
    SizeExec<uint64_t> e;
    e.B = B, e.bw = bw, e.s = s;
    affinity_graph<uint64_t>(e);
    return align256(e.off);
}

template <typename T>
static int dealer_t(int bw, int s, int B, uint64_t seed, const DevWeights &w, uint8_t *k0, uint8_t *k1,
                    cudaStream_t st)
{
    DealerExec<T> e;
    e.B = B, e.bw = bw, e.s = s, e.st = st, e.seed = seed, e.dk = dealer_key(seed), e.k0 = k0, e.k1 = k1, e.w = &w;
    affinity_graph<T>(e);
    if (e.err == DDG_OK) {
        cudaError_t ce = cudaStreamSynchronize(st);
        if (ce != cudaSuccess) {
            set_last_error("dealer: %s", cudaGetErrorString(ce));
            e.err = DDG_ERR_CUDA;
        }
    }
    if (e.err == DDG_OK) e.err = ring_gemm_tc_check(st);
    e.free_all();
    return e.err;
}

int dealer_forward(int bw, int s, int B, uint64_t seed, const DevWeights &w, uint8_t *k0, uint8_t *k1,
                   cudaStream_t st)
{
    DDG_TRY(keep_pool_memory(w.device));
    DDG_TRY(aes_device_init());
    return bw == 32 ? dealer_t<uint32_t>(bw, s, B, seed, w, k0, k1, st)
                    : dealer_t<uint64_t>(bw, s, B, seed, w, k0, k1, st);
}

// capture: the stream is being captured into a CUDA graph (forward_capture):
// the output goes to the device buffer capture_out (when not null) instead of
// the host, and nothing waits for the device
template <typename T>
static int eval_t(Party &P, int B, const void *x_sh, const void *adj_sh, const void *mask_sh, const void *prot_sh,
                  bool on_host, int64_t *h_out_raw, double *h_aff, bool capture = false, void *capture_out = nullptr)
{
    EvalExec<T> e;
    e.B = B, e.bw = P.bw, e.s = P.s, e.st = P.stream, e.P = &P, e.p = P.party;
    const uint64_t sizes[4] = {uint64_t(B) * NMAX * FEAT, uint64_t(B) * NMAX * NMAX, uint64_t(B) * NMAX * POOL,
                               uint64_t(B) * PROT};
    const void *src[4] = {x_sh, adj_sh, mask_sh, prot_sh};
    if (on_host) {
        // host -> device on the party's copy stream, in order of first use; the
        // graph waits on each input's event right before revealing it
        DDG_TRY(P.ensure_copy_stream());
        DDG_CUDA(cudaEventRecord(P.in_ev[4], P.stream));
        DDG_CUDA(cudaStreamWaitEvent(P.copy_stream, P.in_ev[4], 0));  // buffers free: the last forward is done
        for (int i : {int(IN_ADJ), int(IN_X), int(IN_MASK), int(IN_PROT)}) {
            DDG_TRY(P.ensure_input(i, sizes[i] * sizeof(T)));
            DDG_CUDA(cudaMemcpyAsync(P.in_buf[i], src[i], sizes[i] * sizeof(T), cudaMemcpyHostToDevice,
                                     P.copy_stream));
            DDG_CUDA(cudaEventRecord(P.in_ev[i], P.copy_stream));
            e.in[i] = static_cast<const T *>(P.in_buf[i]);
            e.in_ready[i] = P.in_ev[i];
        }
    } else {
        for (int i = 0; i < 4; i++) e.in[i] = static_cast<const T *>(src[i]);
    }
    const uint64_t sent0 = P.chan->bytes_sent[P.party], rounds0 = P.chan->rounds[P.party];
    if (P.timing.enabled) {
        // one reference event per timing session: every timed launch of every
        // forward since enabling is read against it.  A capture does not record
        // it (a replay would move it); ddg_forward_graph_launch records it
        // before the first replay of a session instead.
        if (!P.ref_event) DDG_CUDA(cudaEventCreate(&P.ref_event));
        if (!P.ref_live && !capture) {
            DDG_TRY(record_timing_event(P.ref_event, P.stream));
            P.ref_live = true;
        }
        set_dcf_timing_sink(&P.timing);
    }
    affinity_graph<T>(e);
    set_dcf_timing_sink(nullptr);
    std::vector<T> h(B);
    if (e.err == DDG_OK && !capture)
        e.ok(cudaMemcpyAsync(h.data(), e.out, B * sizeof(T), cudaMemcpyDeviceToHost, P.stream) == cudaSuccess
                 ? DDG_OK : DDG_ERR_CUDA);
    if (e.err == DDG_OK && capture && capture_out)
        e.ok(cudaMemcpyAsync(capture_out, e.out, B * sizeof(T), cudaMemcpyDeviceToDevice, P.stream) == cudaSuccess
                 ? DDG_OK : DDG_ERR_CUDA);
    // the peer may still read buffers this party allocated: join before freeing
    int bs = P.chan->barrier(P.party, P.stream);
    if (e.err == DDG_OK) e.err = bs;
    e.free_all();
    if (capture) {
        if (e.err != DDG_OK) {
            if (auto *lp = dynamic_cast<LocalPairChannel *>(P.chan)) lp->fail();
            return e.err;
        }
        P.stats.bytes_sent = P.chan->bytes_sent[P.party] - sent0;
        P.stats.rounds = P.chan->rounds[P.party] - rounds0;
        P.stats.key_bytes_used = e.off;
        return DDG_OK;
    }
    cudaError_t ce = cudaStreamSynchronize(P.stream);
    if (e.err == DDG_OK && ce != cudaSuccess) {
        set_last_error("forward: %s", cudaGetErrorString(ce));
        e.err = DDG_ERR_CUDA;
    }
    if (e.err == DDG_OK) e.err = ring_gemm_tc_check(P.stream);
    // the caller may reuse its host buffers once this returns
    if (P.copy_stream) {
        ce = cudaStreamSynchronize(P.copy_stream);
        if (e.err == DDG_OK && ce != cudaSuccess) {
            set_last_error("forward input copy: %s", cudaGetErrorString(ce));
            e.err = DDG_ERR_CUDA;
        }
    }
    if (e.err != DDG_OK) {
        if (auto *lp = dynamic_cast<LocalPairChannel *>(P.chan)) lp->fail();
        return e.err;
    }
    P.stats.bytes_sent = P.chan->bytes_sent[P.party] - sent0;
    P.stats.rounds = P.chan->rounds[P.party] - rounds0;
    P.stats.key_bytes_used = e.off;
    for (int i = 0; i < B; i++) {
        using S = typename std::conditional<sizeof(T) == 4, int32_t, int64_t>::type;
        const int64_t v = int64_t(S(h[i]));
        if (h_out_raw) h_out_raw[i] = v;
        // AFFINITY = int32(value) / 2^s (deepdtagen_inference.cu:594-606)
        if (h_aff) h_aff[i] = double(int32_t(uint32_t(uint64_t(v)))) / double(1ull << P.s);
    }
    return DDG_OK;
}

double union_ms(std::vector<std::pair<double, double>> v)
{
    std::sort(v.begin(), v.end());
    double tot = 0, cs = -1, ce = -1;
    for (auto &iv : v) {
        if (iv.first > ce) {
            if (ce > cs) tot += ce - cs;
            cs = iv.first, ce = iv.second;
        } else if (iv.second > ce) {
            ce = iv.second;
        }
    }
    if (ce > cs) tot += ce - cs;
    return tot;
}

// read back the party's pending timed launches (their forwards have finished:
// the forward drains its stream before returning) into its intervals and
// totals, and hand their events back to the pool
static int settle_recs(Party &P, const std::vector<DcfTiming::Rec> &recs)
{
    for (const auto &r : recs) {
        if (!r.done) continue;  // a launch that failed between its two events
        float a = 0, b = 0;
        DDG_CUDA(cudaEventElapsedTime(&a, P.ref_event, r.a));
        DDG_CUDA(cudaEventElapsedTime(&b, P.ref_event, r.b));
        P.intervals.emplace_back(double(a), double(b));
        P.dcf.launches += 1, P.dcf.bytes += r.bytes, P.dcf.aes += r.aes, P.dcf.sum_ms += double(b - a);
    }
    return DDG_OK;
}

// also adds the launches of the last replay of a CUDA graph that holds this
// party's timed launches, once per replay that ran since the last read-back
int settle_timing(Party &P)
{
    DcfTiming &t = P.timing;
    const bool graph = P.timing.enabled && P.graph_recs && P.graph_fresh;
    if (t.recs.empty() && !graph) return DDG_OK;
    DDG_CHECK(P.ref_live, DDG_ERR_STATE, "timed launches without a reference event");
    DDG_CUDA(cudaSetDevice(P.device));
    DDG_TRY(settle_recs(P, t.recs));
    t.recs.clear(), t.used = 0;
    if (graph) {
        DDG_TRY(settle_recs(P, *P.graph_recs));
        P.graph_fresh = false;
    }
    // forwards of one party never overlap, so the union over the whole
    // session is the sum of the per-forward unions
    P.dcf.union_ms = union_ms(P.intervals);
    return DDG_OK;
}

int reset_timing(Party &P, bool on)
{
    P.timing.enabled = on;
    P.timing.recs.clear(), P.timing.used = 0;
    P.dcf = DcfAcc();
    P.intervals.clear();
    P.ref_live = false;
    P.graph_fresh = false;
    if (!on) return DDG_OK;
    // events for ~28 forwards' comparison launches up front; the pool grows on
    // demand beyond that, while the host is ahead of the device
    DDG_CUDA(cudaSetDevice(P.device));
    while (P.timing.pool.size() < 4096) {
        cudaEvent_t e = nullptr;
        DDG_CUDA(cudaEventCreate(&e));
        P.timing.pool.push_back(e);
    }
    return DDG_OK;
}

// union of several parties' comparison-launch intervals since timing was
// enabled, on the timeline of ps[0] (all on one device); stored on ps[0]
int parties_dcf_union(Party *const *ps, int n)
{
    for (int i = 0; i < n; i++) {
        if (!ps[i]->timing.enabled || !ps[i]->ref_live) return DDG_OK;
        DDG_TRY(settle_timing(*ps[i]));
    }
    std::vector<std::pair<double, double>> all = ps[0]->intervals;
    for (int i = 1; i < n; i++) {
        DDG_CHECK(ps[i]->device == ps[0]->device, DDG_ERR_ARG, "DCF interval union needs one device");
        float off = 0;
        DDG_CUDA(cudaEventElapsedTime(&off, ps[0]->ref_event, ps[i]->ref_event));
        for (auto &iv : ps[i]->intervals) all.emplace_back(iv.first + off, iv.second + off);
    }
    ps[0]->dcf.pair_union_ms = union_ms(all);
    return DDG_OK;
}

int forward_capture(Party &P, int B, const void *x_sh, const void *adj_sh, const void *mask_sh, const void *prot_sh,
                    void *d_out)
{
    DDG_CHECK(P.chan, DDG_ERR_STATE, "party %d has no channel", P.party);
    DDG_CHECK(P.keys, DDG_ERR_STATE, "party %d has no keys bound", P.party);
    DDG_CHECK(P.w.table, DDG_ERR_STATE, "party %d has no weights", P.party);
    DDG_CUDA(cudaSetDevice(P.device));
    return P.bw == 32 ? eval_t<uint32_t>(P, B, x_sh, adj_sh, mask_sh, prot_sh, false, nullptr, nullptr, true, d_out)
                      : eval_t<uint64_t>(P, B, x_sh, adj_sh, mask_sh, prot_sh, false, nullptr, nullptr, true, d_out);
}

int forward_eval(Party &P, int B, const void *x_sh, const void *adj_sh, const void *mask_sh, const void *prot_sh,
                 bool on_host, int64_t *h_out_raw, double *h_aff)
{
    DDG_CHECK(P.chan, DDG_ERR_STATE, "party %d has no channel", P.party);
    DDG_CHECK(P.keys, DDG_ERR_STATE, "party %d has no keys bound", P.party);
    DDG_CHECK(P.w.table, DDG_ERR_STATE, "party %d has no weights", P.party);
    DDG_CUDA(cudaSetDevice(P.device));
    DDG_TRY(keep_pool_memory(P.device));
    DDG_TRY(aes_device_init());
    return P.bw == 32 ? eval_t<uint32_t>(P, B, x_sh, adj_sh, mask_sh, prot_sh, on_host, h_out_raw, h_aff)
                      : eval_t<uint64_t>(P, B, x_sh, adj_sh, mask_sh, prot_sh, on_host, h_out_raw, h_aff);
}

}  // namespace ddg
