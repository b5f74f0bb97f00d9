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

GATE_RELU, GATE_RELU_ARS, GATE_ARS, GATE_LRS = 0, 1, 2, 3

DDG_OK = 0
_STATUS = {1: "DDG_ERR_ARG", 2: "DDG_ERR_CUDA", 3: "DDG_ERR_KEY", 4: "DDG_ERR_PEER", 5: "DDG_ERR_STATE",
           6: "DDG_ERR_OVERFLOW"}


class DdgError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{_STATUS.get(code, code)}: {msg}")
        self.code = code


_lib = None

_u64, _u32, _i32, _vp = ctypes.c_uint64, ctypes.c_uint32, ctypes.c_int, ctypes.c_void_p

# name -> (restype, argtypes); kept in the order of include/ddg_fss.h
SIGNATURES = {
    "ddg_last_error": (ctypes.c_char_p, []),
    "ddg_version": (_i32, []),
    "ddg_gate_key_bytes": (_u64, [_i32, _i32, _i32, _u64]),
    "ddg_gate_key_layout": (_i32, [_i32, _i32, _i32, _u64, ctypes.POINTER(_u64)]),
    "ddg_gate_keygen": (_i32, [_i32, _i32, _i32, _u64, _u64, _u32, _vp, _vp, _vp, _vp, _vp]),
    "ddg_gate_round1": (_i32, [_i32, _i32, _i32, _u64, _vp, _vp, _vp, _vp, _vp]),
    "ddg_gate_round2": (_i32, [_i32, _i32, _i32, _u64, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "ddg_aes_chain": (_i32, [_u64, _i32, _vp, _vp]),
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
    out = (_u64 * 12)()
    check(lib().ddg_gate_key_layout(kind, bw, scale, n, out))
    keys = ("hi_root", "hi_cw", "hi_leaf", "hi_mu", "lo_root", "lo_cw", "lo_leaf", "lo_mu", "words", "bytes",
            "hi_levels", "lo_levels")
    return {k: int(v) for k, v in zip(keys, out)}


def gate_keygen(kind, bw, scale, n, seed, op_id, d_rin, d_rout, d_key0, d_key1, stream=None):
    check(lib().ddg_gate_keygen(kind, bw, scale, n, seed, op_id, d_rin, d_rout, d_key0, d_key1, stream))


def gate_round1(kind, bw, scale, n, d_xhat, d_key, d_bits_hi, d_bits_lo, stream=None):
    check(lib().ddg_gate_round1(kind, bw, scale, n, d_xhat, d_key, d_bits_hi, d_bits_lo, stream))


def gate_round2(kind, bw, scale, n, party, d_xhat, d_hi_own, d_hi_peer, d_lo_own, d_lo_peer, d_key, d_share,
                stream=None):
    check(lib().ddg_gate_round2(kind, bw, scale, n, party, d_xhat, d_hi_own, d_hi_peer, d_lo_own, d_lo_peer, d_key,
                                d_share, stream))
