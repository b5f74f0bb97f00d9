// extern "C" entry points of libddg.so (declared in include/ddg_fss.h).
#include "aes_dev.cuh"
#include "gates.cuh"

using namespace ddg;

static int check_gate_args(int kind, int bw, int scale)
{
    DDG_CHECK(kind >= DDG_GATE_RELU && kind <= DDG_GATE_LRS, DDG_ERR_ARG, "gate kind %d out of range", kind);
    DDG_CHECK(bw == 32 || bw == 64, DDG_ERR_ARG, "bw must be 32 or 64 (got %d)", bw);
    DDG_CHECK(scale >= 1 && scale < bw - 1, DDG_ERR_ARG, "scale %d out of range for bw %d", scale, bw);
    return DDG_OK;
}

extern "C" {

const char *ddg_last_error(void) { return ddg::last_error(); }

int ddg_version(void) { return 1; }

uint64_t ddg_gate_key_bytes(int kind, int bw, int scale, uint64_t n)
{
    if (check_gate_args(kind, bw, scale) != DDG_OK) return 0;
    return gate_layout(kind, bw, scale, n).bytes;
}

int ddg_gate_key_layout(int kind, int bw, int scale, uint64_t n, uint64_t *out)
{
    DDG_TRY(check_gate_args(kind, bw, scale));
    DDG_CHECK(out != nullptr, DDG_ERR_ARG, "null out");
    GateLayout L = gate_layout(kind, bw, scale, n);
    uint64_t v[12] = {L.H.root, L.H.cw, L.H.leaf, L.H.mu, L.Lo.root, L.Lo.cw, L.Lo.leaf, L.Lo.mu,
                      L.words, L.bytes, uint64_t(L.H.L), uint64_t(L.Lo.L)};
    for (int i = 0; i < 12; i++) out[i] = v[i];
    return DDG_OK;
}

int ddg_gate_keygen(int kind, int bw, int scale, uint64_t n, uint64_t seed, uint32_t op_id, const void *d_rin,
                    void *d_rout, void *d_key0, void *d_key1, void *stream)
{
    DDG_TRY(check_gate_args(kind, bw, scale));
    DDG_CHECK(n == 0 || (d_rin && d_rout && d_key0 && d_key1), DDG_ERR_ARG, "null pointer");
    return gate_keygen(gate_layout(kind, bw, scale, n), seed, op_id, d_rin, d_rout, d_key0, d_key1,
                       static_cast<cudaStream_t>(stream));
}

int ddg_gate_round1(int kind, int bw, int scale, uint64_t n, const void *d_xhat, const void *d_key,
                    uint32_t *d_bits_hi, uint32_t *d_bits_lo, void *stream)
{
    DDG_TRY(check_gate_args(kind, bw, scale));
    GateLayout L = gate_layout(kind, bw, scale, n);
    DDG_CHECK(n == 0 || (d_xhat && d_key), DDG_ERR_ARG, "null pointer");
    DDG_CHECK(n == 0 || !L.hi || d_bits_hi, DDG_ERR_ARG, "gate needs d_bits_hi");
    DDG_CHECK(n == 0 || !L.lo || d_bits_lo, DDG_ERR_ARG, "gate needs d_bits_lo");
    return gate_round1(L, d_xhat, d_key, d_bits_hi, d_bits_lo, static_cast<cudaStream_t>(stream));
}

int ddg_gate_round2(int kind, int bw, int scale, uint64_t n, int party, const void *d_xhat,
                    const uint32_t *d_hi_own, const uint32_t *d_hi_peer, const uint32_t *d_lo_own,
                    const uint32_t *d_lo_peer, const void *d_key, void *d_share, void *stream)
{
    DDG_TRY(check_gate_args(kind, bw, scale));
    DDG_CHECK(party == 0 || party == 1, DDG_ERR_ARG, "party must be 0 or 1");
    GateLayout L = gate_layout(kind, bw, scale, n);
    DDG_CHECK(n == 0 || (d_xhat && d_key && d_share), DDG_ERR_ARG, "null pointer");
    DDG_CHECK(n == 0 || !L.hi || (d_hi_own && d_hi_peer), DDG_ERR_ARG, "gate needs high-DCF bits");
    DDG_CHECK(n == 0 || !L.lo || (d_lo_own && d_lo_peer), DDG_ERR_ARG, "gate needs low-DCF bits");
    return gate_round2(L, party, d_xhat, d_hi_own, d_hi_peer, d_lo_own, d_lo_peer, d_key, d_share,
                       static_cast<cudaStream_t>(stream));
}

int ddg_aes_chain(uint64_t threads, int iters, uint32_t *d_out, void *stream)
{
    DDG_CHECK(threads > 0 && iters > 0 && d_out, DDG_ERR_ARG, "bad aes_chain arguments");
    return aes_chain(threads, iters, d_out, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
