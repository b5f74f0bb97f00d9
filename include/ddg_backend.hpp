/*
 * ddg_backend.hpp -- a C++ adapter with the shape of the reference's
 * Backend<T> evaluator (DDGOrcaBase / DDGOrca / DDGOrcaBatched,
 * gpu_mpc/ddg_orca_base.h:170-323, ddg_orca.h:43-123) and of its layer calls
 * (ddgSecureAdjNormEval, secure_adj_norm.h:394-405; GCNLayer::forward,
 * gcn_layer.h:99-103; MaskedMaxPoolLayer::_forward, masked_maxpool_layer.h:
 * 23-47) over libddg.so's C ABI (ddg_fss.h).  Header only; link -lddg.
 *
 * One object is one evaluator.  `keyBuf` is the reference's key cursor: every
 * call reads the next key section and advances it; both parties make the same
 * calls in the same order, as the reference's two evaluators do.  Tensors are
 * ddg_wire values (device buffer of the masked-public value + the party's mask
 * share); the caller owns every buffer.  Openings go through the party's
 * channel: NCCL, CUDA IPC, an in-process pair, or the caller's own transport
 * (`Transport`, the seam of GpuPeer::reconstructInPlace, gpu_comms.h:291-302).
 * Every method returns the library's status code (DDG_OK = 0); a failure's
 * message is ddg_last_error().
 */
#ifndef DDG_BACKEND_HPP
#define DDG_BACKEND_HPP

#include <cstdint>

#include "ddg_fss.h"

namespace ddg_ref {

// The caller's transport: exchange() must leave the peer's `bytes` of the
// same opening in d_recv (device) for work queued on `stream` afterwards.
struct Transport {
    virtual ~Transport() {}
    virtual int exchange(int party, const void *d_send, void *d_recv, uint64_t bytes, void *stream) = 0;
};

class Backend {
public:
    // party 0 or 1, ring width bw (32 or 64), scale (12 in the reference),
    // the device, the weights.bin blob (int64, nine layers) and the device key
    // region of one forward (the reference's key arena)
    Backend(int party, int bw, int scale, int device, const int64_t *weights, uint64_t n_weights, const void *d_keys,
            uint64_t key_bytes)
    {
        status_ = ddg_party_create(&p_, party, bw, scale, device);
        if (status_ == DDG_OK) status_ = ddg_party_set_weights(p_, weights, n_weights);
        if (status_ == DDG_OK) status_ = ddg_party_bind_keys(p_, d_keys, key_bytes);
        keyBuf.offset = 0, keyBuf.ops = 0, keyBuf.reserved = 0;
    }
    ~Backend() { ddg_party_destroy(p_); }
    Backend(const Backend &) = delete;
    Backend &operator=(const Backend &) = delete;

    int status() const { return status_; }
    ddg_party *party() { return p_; }

    // channels (the reference's GpuPeer constructor connects a TCP peer)
    int connect_nccl(const void *unique_id128, int nranks, int rank, int peer_rank)
    {
        return ddg_party_connect_nccl(p_, unique_id128, nranks, rank, peer_rank);
    }
    int connect(Transport *t)
    {
        comm_.user = t;
        comm_.exchange = [](void *user, int party, const void *s, void *r, uint64_t bytes, void *st) {
            return static_cast<Transport *>(user)->exchange(party, s, r, bytes, st);
        };
        return ddg_party_connect_callback(p_, &comm_);
    }

    // registerLeaf + revealIfLeaf (ddg_orca_base.h:72-80): a secret-shared input
    int input(const void *d_share, uint64_t n, ddg_wire &out) { return ddg_op_input_eval(p_, &keyBuf, n, d_share, &out); }
    // matmul, 3-arg (secret x secret, per sample): A_hat . x
    int matmul(int batch, int k, ddg_wire &a_hat, ddg_wire &x, ddg_wire &out)
    {
        return ddg_op_matmul_eval(p_, &keyBuf, batch, k, &a_hat, &x, &out);
    }
    // matmul, 4-arg (secret x public weights of layer `layer`, bias at 2*scale)
    int matmul(ddg_wire &x, int layer, int rows, ddg_wire &out)
    {
        return ddg_op_fc_eval(p_, &keyBuf, layer, rows, DDG_ACT_NONE, &x, &out);
    }
    // FC + ReLU(floor(./2^scale)) of the GCN and head layers
    int fc_relu(ddg_wire &x, int layer, int rows, ddg_wire &out)
    {
        return ddg_op_fc_eval(p_, &keyBuf, layer, rows, DDG_ACT_RELU, &x, &out);
    }
    // mul (Beaver, then exact floor by 2^scale for a non-negative product, as
    // DDGOrca::mul truncates)
    int mul(ddg_wire &a, ddg_wire &b, ddg_wire &out) { return ddg_op_mul_eval(p_, &keyBuf, 0, 1, 1, &a, &b, 1, &out); }
    // relu with the gate kind of the selected backend (DDG_GATE_RELU_TTF by default)
    int relu(ddg_wire &in, ddg_wire &out, int kind = DDG_GATE_RELU_TTF)
    {
        return ddg_op_gate_eval(p_, &keyBuf, kind, &in, &out);
    }
    // truncateForward by scale: exact floor; non-negative inputs take the
    // cheaper unsigned gate (DDG_GATE_LRS_TT), others the signed one (DDG_GATE_ARS)
    int truncateForward(ddg_wire &in, ddg_wire &out, bool nonnegative)
    {
        return ddg_op_gate_eval(p_, &keyBuf, nonnegative ? DDG_GATE_LRS_TT : DDG_GATE_ARS, &in, &out);
    }
    // output (ddg_orca_base.h:296-302): revealed values at scale, AFFINITY
    int output(int batch, ddg_wire &o, int64_t *raw, double *affinity)
    {
        return ddg_op_output_eval(p_, &keyBuf, batch, &o, raw, affinity);
    }

    // the layer calls of the reference's graph
    int secureAdjNormEval(int batch, const void *d_adj_share, ddg_wire &a_hat)
    {
        return ddg_adjnorm_eval(p_, &keyBuf, batch, d_adj_share, &a_hat);
    }
    int gcnLayerForward(int layer, int batch, ddg_wire &x, ddg_wire &a_hat, ddg_wire &out)
    {
        return ddg_gcn_layer_eval(p_, &keyBuf, layer, batch, &a_hat, &x, &out);
    }
    int maskedMaxPool(int batch, ddg_wire &masked, ddg_wire &out)
    {
        return ddg_maxpool_eval(p_, &keyBuf, batch, &masked, &out);
    }
    int concatProtein(int batch, ddg_wire &d2, const void *d_protein_share, ddg_wire &out)
    {
        return ddg_op_concat_protein_eval(p_, &keyBuf, batch, &d2, d_protein_share, &out);
    }

    ddg_cursor keyBuf;  // the reference's u8* keyBuf, as a byte offset into the key region

private:
    ddg_party *p_ = nullptr;
    ddg_comm comm_{};
    int status_ = DDG_OK;
};

}  // namespace ddg_ref

#endif /* DDG_BACKEND_HPP */
