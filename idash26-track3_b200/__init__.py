"""B200-native online phase of the two-party DeepDTAGen affinity inference.

The compute lives in ``libddg.so`` (hand-written sm_100a CUDA behind the C ABI
declared in include/ddg_fss.h).  This package is the host-side mirror used by
tests, the bench and Python callers: it loads the library through ctypes,
declares every entry point's signature, and wraps status codes into
exceptions.  There is no CPU fallback: if the library is missing or fails to
load, every call raises.

Import it with ``importlib.import_module("idash26-track3_b200")`` (the
directory name is not a Python identifier).
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libddg.so")

(GATE_RELU, GATE_RELU_ARS, GATE_ARS, GATE_LRS, GATE_RELU_SPLIT, GATE_RELU_ARS_SPLIT, GATE_LRS_SPLIT,
 GATE_RELU_SPLIT3, GATE_RELU_ARS_SPLIT3, GATE_RELU_OT, GATE_RELU_ARS_OT, GATE_RELU_TT, GATE_RELU_ARS_TT,
 GATE_LRS_TT, GATE_RELU_TTF, GATE_RELU_ARS_TTF) = range(16)
# comparison backends of the forward's ReLU gates (relu_backend)
RELU_DCF, RELU_OT, RELU_TT = 0, 1, 2

DDG_OK = 0
_STATUS = {1: "DDG_ERR_ARG", 2: "DDG_ERR_CUDA", 3: "DDG_ERR_KEY", 4: "DDG_ERR_PEER", 5: "DDG_ERR_STATE",
           6: "DDG_ERR_OVERFLOW"}


class DdgError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{_STATUS.get(code, code)}: {msg}")
        self.code = code


_lib = None

_u64, _u32, _i32, _vp = ctypes.c_uint64, ctypes.c_uint32, ctypes.c_int, ctypes.c_void_p


class Cursor(ctypes.Structure):
    """ddg_cursor: key bytes consumed / written so far, dealer ops so far."""
    _fields_ = [("offset", _u64), ("ops", _u32), ("reserved", _u32)]


class Wire(ctypes.Structure):
    """ddg_wire: one evaluator's masked-public tensor and its mask share."""
    _fields_ = [("d_value", _vp), ("n", _u64), ("d_mask_share", _vp)]


class MaskWire(ctypes.Structure):
    """ddg_mask_wire: the dealer's mask of a tensor and both parties' shares of it."""
    _fields_ = [("d_mask", _vp), ("n", _u64), ("d_share0", _vp), ("d_share1", _vp)]


# int exchange(void *user, int party, const void *d_send, void *d_recv, uint64_t bytes, void *stream)
COMM_EXCHANGE = ctypes.CFUNCTYPE(_i32, _vp, _i32, _vp, _vp, _u64, _vp)


class Comm(ctypes.Structure):
    """ddg_comm: the caller's transport for the openings."""
    _fields_ = [("user", _vp), ("exchange", COMM_EXCHANGE)]


ACT_NONE, ACT_RELU, ACT_TRUNC = 0, 1, 2
_C, _W, _M = ctypes.POINTER(Cursor), ctypes.POINTER(Wire), ctypes.POINTER(MaskWire)

# name -> (restype, argtypes); kept in the order of include/ddg_fss.h
SIGNATURES = {
    "ddg_last_error": (ctypes.c_char_p, []),
    "ddg_version": (_i32, []),
    "ddg_gate_key_bytes": (_u64, [_i32, _i32, _i32, _u64]),
    "ddg_gate_key_layout": (_i32, [_i32, _i32, _i32, _u64, ctypes.POINTER(_u64)]),
    "ddg_gate_keygen": (_i32, [_i32, _i32, _i32, _u64, _u64, _u32, _vp, _vp, _vp, _vp, _vp]),
    "ddg_gate_round1": (_i32, [_i32, _i32, _i32, _u64, _vp, _vp, _vp, _vp, _vp]),
    "ddg_gate_round2": (_i32, [_i32, _i32, _i32, _u64, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "ddg_ot_key_layout": (_i32, [_i32, _i32, _i32, _u64, ctypes.POINTER(_u64)]),
    "ddg_tt_key_layout": (_i32, [_i32, _i32, _i32, _u64, ctypes.POINTER(_u64)]),
    "ddg_gate_eval_pair_noalloc": (_i32, [_i32, _i32, _i32, _u64, _vp, _vp, _vp, _vp, _vp]),
    "ddg_lut_key_bytes": (_u64, [_i32, _u64]),
    "ddg_lut_keygen": (_i32, [_i32, _u64, _u64, _u32, _vp, _vp, _vp, _vp, _vp]),
    "ddg_lut_eval": (_i32, [_i32, _u64, _i32, _vp, _vp, _vp, _vp, _vp]),
    "ddg_tt_lut_key_bytes": (_u64, [_i32, _u64]),
    "ddg_tt_lut_keygen": (_i32, [_i32, _u64, _u64, _u32, _vp, _vp, _vp, _vp, _vp, _vp]),
    "ddg_tt_lut_eval": (_i32, [_i32, _u64, _vp, _vp, _vp, _vp]),
    "ddg_mul_share": (_i32, [_i32, _i32, _u64, _i32, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "ddg_matmul_share": (_i32, [_i32, _i32, _i32, _i32, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "ddg_fc_share": (_i32, [_i32, _i32, _i32, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp]),
    "ddg_gemm_path": (_i32, [_i32]),
    "ddg_gemm_status": (_i32, []),
    "ddg_aes_chain": (_i32, [_u64, _i32, _vp, _vp]),
    "ddg_aes_chain_variant": (_i32, [_u64, _i32, _i32, _vp, _vp]),
    "ddg_aes_tables": (_i32, [_i32]),
    "ddg_relu_split": (_i32, [_i32]),
    "ddg_relu_backend": (_i32, [_i32]),
    "ddg_gate_eval_pair": (_i32, [_i32, _i32, _i32, _u64, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "ddg_gate_round1_arrays": (_i32, [_i32, _i32, _i32]),
    "ddg_party_create": (_i32, [ctypes.POINTER(_vp), _i32, _i32, _i32, _i32]),
    "ddg_party_destroy": (_i32, [_vp]),
    "ddg_party_set_weights": (_i32, [_vp, _vp, _u64]),
    "ddg_party_bind_keys": (_i32, [_vp, _vp, _u64]),
    "ddg_party_stream": (_i32, [_vp, ctypes.POINTER(_vp)]),
    "ddg_party_stats": (_i32, [_vp, ctypes.POINTER(_u64)]),
    "ddg_pair_local": (_i32, [_vp, _vp]),
    "ddg_nccl_unique_id": (_i32, [_vp]),
    "ddg_party_connect_nccl": (_i32, [_vp, _vp, _i32, _i32, _i32]),
    "ddg_party_set_timeout": (_i32, [_vp, _i32]),
    "ddg_party_connect_ipc": (_i32, [_vp, ctypes.c_char_p, _u64]),
    "ddg_party_connect_ipc_push": (_i32, [_vp, ctypes.c_char_p, _u64]),
    "ddg_party_exchange_probe": (_i32, [_vp, _u64, _i32, ctypes.POINTER(ctypes.c_double)]),
    "ddg_forward_max_exchange_bytes": (_u64, [_i32, _i32, _i32]),
    "ddg_forward_key_bytes": (_u64, [_i32, _i32, _i32]),
    "ddg_forward_eval": (_i32, [_vp, _i32, _vp, _vp, _vp, _vp, _i32, _vp, _vp]),
    "ddg_forward_eval_pair": (_i32, [_vp, _vp, _i32, ctypes.POINTER(_vp), ctypes.POINTER(_vp), _i32, _vp, _vp]),
    "ddg_forward_graph_create": (_i32, [_vp, _vp, _i32, ctypes.POINTER(_vp), ctypes.POINTER(_vp),
                                        ctypes.POINTER(_vp)]),
    "ddg_party_graph_create": (_i32, [_vp, _i32, ctypes.POINTER(_vp), _i32, ctypes.POINTER(_vp)]),
    "ddg_forward_graph_create_ex": (_i32, [_vp, _vp, _i32, ctypes.POINTER(_vp), ctypes.POINTER(_vp), _i32,
                                           ctypes.POINTER(_vp)]),
    "ddg_forward_graph_launch": (_i32, [_vp, _vp, _vp]),
    "ddg_forward_graph_enqueue": (_i32, [_vp]),
    "ddg_forward_graph_sync": (_i32, [_vp, _vp, _vp]),
    "ddg_forward_pipeline_create": (_i32, [_vp, _vp, _i32, ctypes.POINTER(_vp)]),
    "ddg_forward_pipeline_submit": (_i32, [_vp, ctypes.POINTER(_vp), ctypes.POINTER(_vp), _vp, _vp]),
    "ddg_forward_pipeline_wait": (_i32, [_vp]),
    "ddg_forward_pipeline_destroy": (_i32, [_vp]),
    "ddg_forward_graph_destroy": (_i32, [_vp]),
    "ddg_dealer_forward": (_i32, [_i32, _i32, _i32, _u64, _vp, _u64, _i32, _vp, _vp, _vp]),
    "ddg_party_connect_callback": (_i32, [_vp, ctypes.POINTER(Comm)]),
    "ddg_op_input_eval": (_i32, [_vp, _C, _u64, _vp, _W]),
    "ddg_adjnorm_eval": (_i32, [_vp, _C, _i32, _vp, _W]),
    "ddg_gcn_layer_eval": (_i32, [_vp, _C, _i32, _i32, _W, _W, _W]),
    "ddg_op_matmul_eval": (_i32, [_vp, _C, _i32, _i32, _W, _W, _W]),
    "ddg_op_mul_eval": (_i32, [_vp, _C, _i32, _i32, _i32, _W, _W, _i32, _W]),
    "ddg_op_gate_eval": (_i32, [_vp, _C, _i32, _W, _W]),
    "ddg_maxpool_eval": (_i32, [_vp, _C, _i32, _W, _W]),
    "ddg_op_fc_eval": (_i32, [_vp, _C, _i32, _i32, _i32, _W, _W]),
    "ddg_op_concat_protein_eval": (_i32, [_vp, _C, _i32, _W, _vp, _W]),
    "ddg_op_output_eval": (_i32, [_vp, _C, _i32, _W, _vp, _vp]),
    "ddg_dealer_create": (_i32, [ctypes.POINTER(_vp), _i32, _i32, _i32, _u64, _vp, _u64]),
    "ddg_dealer_bind_keys": (_i32, [_vp, _vp, _vp, _u64]),
    "ddg_dealer_stream": (_i32, [_vp, ctypes.POINTER(_vp)]),
    "ddg_dealer_destroy": (_i32, [_vp]),
    "ddg_op_input_keygen": (_i32, [_vp, _C, _u64, _M]),
    "ddg_adjnorm_keygen": (_i32, [_vp, _C, _i32, _M]),
    "ddg_gcn_layer_keygen": (_i32, [_vp, _C, _i32, _i32, _M, _M, _M]),
    "ddg_op_matmul_keygen": (_i32, [_vp, _C, _i32, _i32, _M, _M, _M]),
    "ddg_op_mul_keygen": (_i32, [_vp, _C, _i32, _i32, _i32, _M, _M, _i32, _M]),
    "ddg_op_gate_keygen": (_i32, [_vp, _C, _i32, _M, _M]),
    "ddg_maxpool_keygen": (_i32, [_vp, _C, _i32, _M, _M]),
    "ddg_op_fc_keygen": (_i32, [_vp, _C, _i32, _i32, _i32, _M, _M]),
    "ddg_op_concat_protein_keygen": (_i32, [_vp, _C, _i32, _M, _M]),
    "ddg_op_output_keygen": (_i32, [_vp, _C, _M]),
    "ddg_launch_count": (_u64, []),
    "ddg_key_chunk_bytes": (_u64, [_i32, _i32, _i32]),
    "ddg_key_checksum": (_i32, [_vp, _u64, ctypes.POINTER(_u64), _vp]),
    "ddg_key_chunk_seal": (_i32, [_vp, _i32, _i32, _i32, _u64, _vp]),
    "ddg_key_chunk_verify": (_i32, [_vp, _i32, _i32, _i32, ctypes.POINTER(_u64), _vp]),
    "ddg_keystream_create": (_i32, [ctypes.POINTER(_vp), _vp, _i32]),
    "ddg_keystream_destroy": (_i32, [_vp]),
    "ddg_keystream_add_host_chunk": (_i32, [_vp, _vp]),
    "ddg_keystream_open_file": (_i32, [_vp, ctypes.c_char_p, _i32]),
    "ddg_keystream_set_verify": (_i32, [_vp, _i32]),
    "ddg_keystream_stats": (_i32, [_vp, ctypes.POINTER(ctypes.c_double)]),
    "ddg_forward_eval_streamed": (_i32, [_vp, _i32, _vp, _vp, _vp, _vp, _i32, _vp, _vp]),
    "ddg_forward_eval_pair_streamed": (_i32, [_vp, _vp, _i32, ctypes.POINTER(_vp), ctypes.POINTER(_vp), _i32, _vp,
                                              _vp]),
    "ddg_party_enable_dcf_timing": (_i32, [_vp, _i32]),
    "ddg_party_dcf_timing": (_i32, [_vp, ctypes.POINTER(ctypes.c_double)]),
    "ddg_parties_dcf_union": (_i32, [ctypes.POINTER(_vp), _i32]),
}


def lib():
    """The loaded libddg.so (raises if it is missing: build with __graft_entry__.build())."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing; run __graft_entry__.build() first")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def check(status: int):
    if status != DDG_OK:
        raise DdgError(status, (lib().ddg_last_error() or b"").decode(errors="replace"))
    return status


def gate_key_bytes(kind: int, bw: int, scale: int, n: int) -> int:
    return int(lib().ddg_gate_key_bytes(kind, bw, scale, n))


def gate_key_layout(kind: int, bw: int, scale: int, n: int) -> dict:
    """Byte offsets of one party's gate key (see ddg_gate_key_layout)."""
    out = (_u64 * 22)()
    check(lib().ddg_gate_key_layout(kind, bw, scale, n, out))
    keys = ("hi_root", "hi_cw", "hi_leaf", "hi_mu", "lo_root", "lo_cw", "lo_leaf", "lo_mu", "words", "bytes",
            "hi_levels", "lo_levels", "hi_mu_eq", "hi_bits", "hi_shift", "lo_bits", "mid_root", "mid_cw", "mid_leaf",
            "mid_mu", "mid_mu_eq", "mid_levels")
    return {k: int(v) for k, v in zip(keys, out)}


def ot_key_layout(kind: int, bw: int, scale: int, n: int) -> dict:
    """Byte offsets and plan of one party's OT-gate key (see ddg_ot_key_layout)."""
    out = (_u64 * 10)()
    check(lib().ddg_ot_key_layout(kind, bw, scale, n, out))
    keys = ("ks", "recv", "c0", "words", "bytes", "slots", "digits", "g0", "levels", "combines")
    return {k: int(v) for k, v in zip(keys, out)}


def tt_key_layout(kind: int, bw: int, scale: int, n: int) -> dict:
    """Byte offsets and plan of one party's truth-table gate key (see ddg_tt_key_layout)."""
    out = (_u64 * 8)()
    check(lib().ddg_tt_key_layout(kind, bw, scale, n, out))
    keys = ("tables", "rows", "tri", "tri_words", "words", "bytes", "digits", "levels")
    return {k: int(v) for k, v in zip(keys, out)}


def gate_round1_arrays(kind: int, bw: int, scale: int) -> int:
    """ceil(n/32)-word bit arrays of a kind's comparison bits (round-1 layout)."""
    return int(lib().ddg_gate_round1_arrays(kind, bw, scale))


def gate_eval_pair(kind, bw, scale, n, d_xhat, d_key0, d_key1, d_bits0, d_bits1, d_share0, d_share1, stream=None):
    """Both parties of one gate on one device (every round, openings in place); see ddg_gate_eval_pair."""
    check(lib().ddg_gate_eval_pair(kind, bw, scale, n, d_xhat, d_key0, d_key1, d_bits0, d_bits1, d_share0,
                                   d_share1, stream))


def gate_keygen(kind, bw, scale, n, seed, op_id, d_rin, d_rout, d_key0, d_key1, stream=None):
    check(lib().ddg_gate_keygen(kind, bw, scale, n, seed, op_id, d_rin, d_rout, d_key0, d_key1, stream))


def gate_round1(kind, bw, scale, n, d_xhat, d_key, d_bits_hi, d_bits_lo, stream=None):
    check(lib().ddg_gate_round1(kind, bw, scale, n, d_xhat, d_key, d_bits_hi, d_bits_lo, stream))


def gate_round2(kind, bw, scale, n, party, d_xhat, d_hi_own, d_hi_peer, d_lo_own, d_lo_peer, d_key, d_share,
                stream=None):
    check(lib().ddg_gate_round2(kind, bw, scale, n, party, d_xhat, d_hi_own, d_hi_peer, d_lo_own, d_lo_peer, d_key,
                                d_share, stream))


# ---------------------------------------------------------------- parties

def forward_key_bytes(bw: int, scale: int, batch: int) -> int:
    return int(lib().ddg_forward_key_bytes(bw, scale, batch))


def dealer_forward(bw, scale, batch, seed, weights_blob, device, d_key0, d_key1, stream=None):
    """GPU dealer: both parties' keys for one forward of `batch` samples.
    `weights_blob` is the int64 weights.bin content (numpy array)."""
    import numpy as np

    blob = np.ascontiguousarray(weights_blob, dtype=np.int64)
    check(lib().ddg_dealer_forward(bw, scale, batch, seed, blob.ctypes.data, blob.size, device, d_key0, d_key1,
                                   stream))


class Party:
    """One evaluator (party 0 or 1) of the online phase: mirrors the reference's
    DDGOrcaBatched backend object (gpu_mpc/ddg_orca_batched.h:87-206) plus its
    GpuPeer.  Keys are a device region bound with bind_keys(); weights are the
    int64 weights.bin blob."""

    def __init__(self, party: int, bw: int, scale: int = 12, device: int = 0):
        h = _vp()
        check(lib().ddg_party_create(ctypes.byref(h), party, bw, scale, device))
        self.h, self.party, self.bw, self.scale, self.device = h, party, bw, scale, device

    def close(self):
        if self.h:
            lib().ddg_party_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_weights(self, blob):
        import numpy as np

        b = np.ascontiguousarray(blob, dtype=np.int64)
        check(lib().ddg_party_set_weights(self.h, b.ctypes.data, b.size))

    def bind_keys(self, d_ptr: int, nbytes: int):
        check(lib().ddg_party_bind_keys(self.h, d_ptr, nbytes))

    @property
    def stream(self) -> int:
        s = _vp()
        check(lib().ddg_party_stream(self.h, ctypes.byref(s)))
        return s.value or 0

    def stats(self) -> dict:
        out = (_u64 * 3)()
        check(lib().ddg_party_stats(self.h, out))
        return {"bytes_sent": int(out[0]), "rounds": int(out[1]), "key_bytes_used": int(out[2])}

    def enable_dcf_timing(self, on: bool = True):
        check(lib().ddg_party_enable_dcf_timing(self.h, int(on)))

    def dcf_timing(self) -> dict:
        out = (ctypes.c_double * 6)()
        check(lib().ddg_party_dcf_timing(self.h, out))
        keys = ("launches", "bytes", "aes_blocks", "sum_ms", "union_ms", "pair_union_ms")
        return dict(zip(keys, [float(v) for v in out]))

    def connect_nccl(self, unique_id: bytes, nranks: int, rank: int, peer_rank: int):
        buf = ctypes.create_string_buffer(bytes(unique_id), 128)
        check(lib().ddg_party_connect_nccl(self.h, buf, nranks, rank, peer_rank))

    def connect_ipc(self, name: str, slot_bytes: int, push: bool = False):
        """Two party processes on one node: openings through CUDA IPC (see
        ddg_party_connect_ipc); push=True hands them over on the device
        (ddg_party_connect_ipc_push; the parties on different GPUs)."""
        fn = lib().ddg_party_connect_ipc_push if push else lib().ddg_party_connect_ipc
        check(fn(self.h, name.encode(), slot_bytes))

    def connect_callback(self, exchange):
        """Openings through the caller's transport: exchange(party, d_send,
        d_recv, nbytes, stream) -> 0 on success (see ddg_comm)."""

        def tramp(user, party, d_send, d_recv, nbytes, stream):
            try:
                return int(exchange(party, d_send, d_recv, nbytes, stream) or 0)
            except Exception:  # any failure of the transport fails the opening
                return 1

        self._comm_fn = COMM_EXCHANGE(tramp)  # kept alive as long as the party
        self._comm = Comm(None, self._comm_fn)
        check(lib().ddg_party_connect_callback(self.h, ctypes.byref(self._comm)))

    def set_timeout(self, ms: int):
        check(lib().ddg_party_set_timeout(self.h, ms))

    def exchange_probe(self, nbytes: int, iters: int) -> float:
        """ms per opening of nbytes through this party's channel (both parties call it together)."""
        out = ctypes.c_double()
        check(lib().ddg_party_exchange_probe(self.h, nbytes, iters, ctypes.byref(out)))
        return out.value

    def forward(self, batch, x, adj, mask, prot, on_host=False):
        """One online forward.  x/adj/mask/prot: this party's shares (device
        pointers, or host pointers with on_host=True).  Returns (raw ring
        outputs as int64, affinities) on party 0, (None, None) on party 1."""
        import numpy as np

        raw = np.zeros(batch, dtype=np.int64)
        aff = np.zeros(batch, dtype=np.float64)
        check(lib().ddg_forward_eval(self.h, batch, x, adj, mask, prot, int(on_host), raw.ctypes.data,
                                     aff.ctypes.data))
        return (raw, aff) if self.party == 0 else (None, None)


class Dealer:
    """The layer-by-layer GPU dealer (ddg_dealer_*): both parties' keys written
    at a cursor by the ddg_*_keygen entry points."""

    def __init__(self, bw: int, scale: int, device: int, seed: int, weights_blob):
        import numpy as np

        blob = np.ascontiguousarray(weights_blob, dtype=np.int64)
        h = _vp()
        check(lib().ddg_dealer_create(ctypes.byref(h), bw, scale, device, seed, blob.ctypes.data, blob.size))
        self.h = h

    def bind_keys(self, d_key0: int, d_key1: int, nbytes: int):
        check(lib().ddg_dealer_bind_keys(self.h, d_key0, d_key1, nbytes))

    def close(self):
        if self.h:
            check(lib().ddg_dealer_destroy(self.h))
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def nccl_unique_id() -> bytes:
    buf = ctypes.create_string_buffer(128)
    check(lib().ddg_nccl_unique_id(buf))
    return buf.raw


def pair_local(p0: Party, p1: Party):
    check(lib().ddg_pair_local(p0.h, p1.h))


def forward_pair(p0: Party, p1: Party, batch, inputs0, inputs1, on_host=False):
    """Both parties of an in-process pair, each on its own host thread.
    inputs0/1: (x, adj, mask, protein) share pointers. Returns (raw, affinity)."""
    import numpy as np

    a0 = (_vp * 4)(*inputs0)
    a1 = (_vp * 4)(*inputs1)
    raw = np.zeros(batch, dtype=np.int64)
    aff = np.zeros(batch, dtype=np.float64)
    check(lib().ddg_forward_eval_pair(p0.h, p1.h, batch, a0, a1, int(on_host), raw.ctypes.data, aff.ctypes.data))
    return raw, aff


class ForwardGraph:
    """One pair forward of device-resident inputs captured into a CUDA graph
    (ddg_forward_graph_create) and replayed by launch(); see ddg_fss.h.  Run one
    ordinary forward_pair of the pair before creating it, and close it before
    the parties."""

    def __init__(self, p0: Party, p1, batch, inputs0, inputs1=None, on_host=False):
        """on_host: inputs are pinned host buffers copied in by every replay.
        p1 None: p0's own forward alone (ddg_party_graph_create), for a party
        whose peer is another process over a push-mode IPC channel."""
        self.batch = batch
        a0 = (_vp * 4)(*inputs0)
        h = _vp()
        if p1 is None:
            check(lib().ddg_party_graph_create(p0.h, batch, a0, int(on_host), ctypes.byref(h)))
        else:
            a1 = (_vp * 4)(*inputs1)
            check(lib().ddg_forward_graph_create_ex(p0.h, p1.h, batch, a0, a1, int(on_host), ctypes.byref(h)))
        self.h = h

    def launch(self, outputs=True):
        """Replay the forward; returns (raw, affinity) of the (first) party's reveal, or None."""
        import numpy as np

        if not outputs:
            check(lib().ddg_forward_graph_launch(self.h, None, None))
            return None
        raw = np.zeros(self.batch, dtype=np.int64)
        aff = np.zeros(self.batch, dtype=np.float64)
        check(lib().ddg_forward_graph_launch(self.h, raw.ctypes.data, aff.ctypes.data))
        return raw, aff

    def enqueue(self):
        """Queue one replay without waiting (ddg_forward_graph_enqueue)."""
        check(lib().ddg_forward_graph_enqueue(self.h))

    def sync(self, outputs=True):
        """Wait for the replays queued; (raw, affinity) of the last one, or None."""
        import numpy as np

        if not outputs:
            check(lib().ddg_forward_graph_sync(self.h, None, None))
            return None
        raw = np.zeros(self.batch, dtype=np.int64)
        aff = np.zeros(self.batch, dtype=np.float64)
        check(lib().ddg_forward_graph_sync(self.h, raw.ctypes.data, aff.ctypes.data))
        return raw, aff

    def close(self):
        if self.h:
            check(lib().ddg_forward_graph_destroy(self.h))
            self.h = None


class ForwardPipeline:
    """Pipelined forwards of an in-process pair on pinned host input shares
    (ddg_forward_pipeline_*; see ddg_fss.h): submit() queues one step (its
    input copies overlap the previous step's forward) and returns the (raw,
    affinity) arrays that the step fills once delivered, by a later submit()
    or by wait().  Run one ordinary forward_pair first, with DCF timing off."""

    def __init__(self, p0: Party, p1: Party, batch: int):
        self.batch = batch
        h = _vp()
        check(lib().ddg_forward_pipeline_create(p0.h, p1.h, batch, ctypes.byref(h)))
        self.h = h
        self._keep = [None, None]  # the arrays of the steps in flight, per staging set
        self._k = 0

    def submit(self, inputs0, inputs1):
        import numpy as np

        raw = np.zeros(self.batch, dtype=np.int64)
        aff = np.zeros(self.batch, dtype=np.float64)
        a0, a1 = (_vp * 4)(*inputs0), (_vp * 4)(*inputs1)
        check(lib().ddg_forward_pipeline_submit(self.h, a0, a1, raw.ctypes.data, aff.ctypes.data))
        self._keep[self._k & 1] = (raw, aff)
        self._k += 1
        return raw, aff

    def wait(self):
        check(lib().ddg_forward_pipeline_wait(self.h))

    def close(self):
        if self.h:
            check(lib().ddg_forward_pipeline_destroy(self.h))
            self.h = None


def forward_max_exchange_bytes(bw: int, scale: int, batch: int) -> int:
    return int(lib().ddg_forward_max_exchange_bytes(bw, scale, batch))


def launch_count() -> int:
    return int(lib().ddg_launch_count())


GEMM_TENSOR, GEMM_CUDA_CORES, GEMM_TENSOR_BK, GEMM_TENSOR_WIDE, GEMM_TENSOR_SYNC, GEMM_TENSOR_INKERNEL = 0, 1, 2, 3, 4, 5


def gemm_path(path: int):
    """Ring GEMM engine: GEMM_TENSOR (default, tcgen05 limb products),
    GEMM_CUDA_CORES, or the tensor-core layout/tile variants."""
    check(lib().ddg_gemm_path(path))


def aes_tables(tables: int):
    """AES engine of every FSS kernel: 4 (default) or 2 staged round tables."""
    check(lib().ddg_aes_tables(tables))


def relu_split(parts: int):
    """Comparison split of the forward's ReLU gates: 3 (default, fewest AES) or 2
    (smaller keys).  Dealer and evaluators must use the same setting (it changes
    the key layout)."""
    check(lib().ddg_relu_split(parts))


def relu_backend(backend: int):
    """Comparison backend of the forward's ReLU gates: RELU_TT (default; dealer digit truth tables +
    Beaver AND tree, GATE_RELU*_TT, and GATE_LRS_TT at the truncation sites), RELU_OT (garbled
    radix-16 digit tables + the same tree, GATE_RELU*_OT) or RELU_DCF (DCF keys, split per relu_split).
    Dealer and evaluators must use the same setting (it changes the key layout)."""
    check(lib().ddg_relu_backend(backend))


def gemm_status():
    """Raise DdgError if a tensor-core GEMM gave up on a bounded wait (clears the flag)."""
    check(lib().ddg_gemm_status())


# ---------------------------------------------------------------- key chunks / streaming

def key_chunk_bytes(bw: int, scale: int, batch: int) -> int:
    return int(lib().ddg_key_chunk_bytes(bw, scale, batch))


def key_chunk_seal(d_chunk: int, bw: int, scale: int, batch: int, index: int, stream=None):
    check(lib().ddg_key_chunk_seal(d_chunk, bw, scale, batch, index, stream))


def key_chunk_verify(d_chunk: int, bw: int, scale: int, batch: int, stream=None) -> int:
    idx = _u64()
    check(lib().ddg_key_chunk_verify(d_chunk, bw, scale, batch, ctypes.byref(idx), stream))
    return int(idx.value)


class KeyStream:
    """Double-buffered key feed of one party (chunks in pinned host memory or a key file)."""

    def __init__(self, party: Party, batch: int):
        h = _vp()
        check(lib().ddg_keystream_create(ctypes.byref(h), party.h, batch))
        self.h, self.party, self.batch = h, party, batch

    def add_host_chunk(self, h_ptr: int):
        check(lib().ddg_keystream_add_host_chunk(self.h, h_ptr))

    def open_file(self, path: str, nchunks: int):
        check(lib().ddg_keystream_open_file(self.h, path.encode(), nchunks))

    def set_verify(self, on: bool = True):
        check(lib().ddg_keystream_set_verify(self.h, int(on)))

    def stats(self) -> dict:
        out = (ctypes.c_double * 5)()
        check(lib().ddg_keystream_stats(self.h, out))
        return dict(zip(("chunks", "bytes", "copy_ms", "read_ms", "wait_ms"), [float(v) for v in out]))

    def forward(self, x, adj, mask, prot, on_host=False):
        import numpy as np

        raw = np.zeros(self.batch, dtype=np.int64)
        aff = np.zeros(self.batch, dtype=np.float64)
        check(lib().ddg_forward_eval_streamed(self.h, self.batch, x, adj, mask, prot, int(on_host), raw.ctypes.data,
                                              aff.ctypes.data))
        return (raw, aff) if self.party.party == 0 else (None, None)

    def close(self):
        if self.h:
            lib().ddg_keystream_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def forward_pair_streamed(ks0: KeyStream, ks1: KeyStream, inputs0, inputs1, on_host=False):
    import numpy as np

    B = ks0.batch
    a0 = (_vp * 4)(*inputs0)
    a1 = (_vp * 4)(*inputs1)
    raw = np.zeros(B, dtype=np.int64)
    aff = np.zeros(B, dtype=np.float64)
    check(lib().ddg_forward_eval_pair_streamed(ks0.h, ks1.h, B, a0, a1, int(on_host), raw.ctypes.data,
                                               aff.ctypes.data))
    return raw, aff


def dealer_chunks(bw: int, scale: int, batch: int, seeds, weights_blob, device: int = 0):
    """GPU dealer -> sealed key chunks of both parties in pinned host memory.

    Returns [(chunk0, chunk1)] per seed: torch uint8 pinned tensors of
    key_chunk_bytes(bw, scale, batch) bytes, chunk index = position in `seeds`."""
    import torch

    cb = key_chunk_bytes(bw, scale, batch)
    kb = forward_key_bytes(bw, scale, batch)
    dev = torch.device("cuda", device)
    d0 = torch.empty(cb, dtype=torch.uint8, device=dev)
    d1 = torch.empty(cb, dtype=torch.uint8, device=dev)
    out = []
    for i, seed in enumerate(seeds):
        dealer_forward(bw, scale, batch, seed, weights_blob, device, d0.data_ptr(), d1.data_ptr())
        pair = []
        for d in (d0, d1):
            key_chunk_seal(d.data_ptr(), bw, scale, batch, i)
            h = torch.empty(cb, dtype=torch.uint8, pin_memory=True)
            h.copy_(d)
            pair.append(h)
        out.append(tuple(pair))
    assert kb <= cb
    return out


def write_key_file(path: str, chunks) -> None:
    """Chunks back to back (chunk k at k * key_chunk_bytes), as the reference's
    dealer pwrites them (deepdtagen_inference.cu:383-398)."""
    with open(path, "wb") as f:
        for c in chunks:
            f.write(c.numpy().tobytes())


def parties_dcf_union(parties):
    arr = (_vp * len(parties))(*[p.h for p in parties])
    check(lib().ddg_parties_dcf_union(arr, len(parties)))


def forward_lanes(parties, batch_per_lane, inputs, on_host=False):
    """Run one forward on each of several parties of this process concurrently
    (one host thread each; the library releases the GIL).  inputs[i] =
    (x, adj, mask, protein) pointers of lane i.  Returns the lanes' (raw, aff)."""
    import threading

    results, errors = [None] * len(parties), [None] * len(parties)

    def run(i):
        try:
            results[i] = parties[i].forward(batch_per_lane, *inputs[i], on_host=on_host)
        except Exception as e:  # re-raised in the caller
            errors[i] = e

    ts = [threading.Thread(target=run, args=(i,)) for i in range(len(parties))]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    for e in errors:
        if e is not None:
            raise e
    return results
