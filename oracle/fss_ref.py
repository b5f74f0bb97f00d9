"""ctypes view of oracle/fss_ref.c -- TEST INFRASTRUCTURE ONLY.

Imported by tests/, by ``__graft_entry__.smoke()`` and by bench.py's
cpu_baseline leg as the checker of the CUDA FSS kernels.  Nothing in the
product package imports it.

The C file restates, in plain byte-oriented C, this build's FSS scheme
(AES-128, the half-tree DCF/DPF, the comparison gates and the 8-bit DPF
look-up table); see the header of fss_ref.c for the published algorithms it
follows and for the reference call sites it replaces
(gpu_mpc/ddg_orca.h:83-123, gpu_mpc/secure_adj_norm.h:498-520).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "libfss_ref.so")

(GATE_RELU, GATE_RELU_ARS, GATE_ARS, GATE_LRS, GATE_RELU_SPLIT, GATE_RELU_ARS_SPLIT, GATE_LRS_SPLIT,
 GATE_RELU_SPLIT3, GATE_RELU_ARS_SPLIT3, GATE_RELU_OT, GATE_RELU_ARS_OT, GATE_RELU_TT, GATE_RELU_ARS_TT,
 GATE_LRS_TT, GATE_RELU_TTF, GATE_RELU_ARS_TTF) = range(16)
GATE_NWORDS = {GATE_RELU: 4, GATE_RELU_ARS: 8, GATE_ARS: 6, GATE_LRS: 4, GATE_RELU_SPLIT: 16,
               GATE_RELU_ARS_SPLIT: 32, GATE_LRS_SPLIT: 7, GATE_RELU_SPLIT3: 40, GATE_RELU_ARS_SPLIT3: 80,
               GATE_RELU_OT: 16, GATE_RELU_ARS_OT: 32, GATE_RELU_TT: 16, GATE_RELU_ARS_TT: 32, GATE_LRS_TT: 4,
               GATE_RELU_TTF: 4, GATE_RELU_ARS_TTF: 8}
# OT-leaf kinds and the SPLIT kind whose words and round 2 they use
OT_KINDS = (GATE_RELU_OT, GATE_RELU_ARS_OT)
OT_WORD_KIND = {GATE_RELU_OT: GATE_RELU_SPLIT, GATE_RELU_ARS_OT: GATE_RELU_ARS_SPLIT}
# truth-table kinds and the kind whose words and round 2 they use
TT_KINDS = (GATE_RELU_TT, GATE_RELU_ARS_TT, GATE_LRS_TT, GATE_RELU_TTF, GATE_RELU_ARS_TTF)
TT_WORD_KIND = {GATE_RELU_TT: GATE_RELU_SPLIT, GATE_RELU_ARS_TT: GATE_RELU_ARS_SPLIT, GATE_LRS_TT: GATE_LRS,
                GATE_RELU_TTF: GATE_RELU, GATE_RELU_ARS_TTF: GATE_RELU_ARS}
# kinds whose high DCF also outputs equality (three round-1 bit arrays or more)
SPLIT_KINDS = (GATE_RELU_SPLIT, GATE_RELU_ARS_SPLIT, GATE_LRS_SPLIT, GATE_RELU_SPLIT3, GATE_RELU_ARS_SPLIT3)
# kinds with a middle DCF with equality output (five round-1 bit arrays)
SPLIT3_KINDS = (GATE_RELU_SPLIT3, GATE_RELU_ARS_SPLIT3)


def build() -> str:
    src = os.path.join(_HERE, "fss_ref.c")
    if not os.path.exists(_SO) or os.path.getmtime(_SO) < os.path.getmtime(src):
        subprocess.check_call(["make", "-s", "-C", _HERE, "libfss_ref.so"])
    return _SO


class GateKey(ctypes.Structure):
    _fields_ = [
        ("hi_root", ctypes.c_uint8 * 16),
        ("hi_cw", (ctypes.c_uint8 * 16) * 56),
        ("hi_leaf", ctypes.c_uint8 * 16),
        ("hi_mu", ctypes.c_int32),
        ("hi_mu_eq", ctypes.c_int32),
        ("lo_root", ctypes.c_uint8 * 16),
        ("lo_cw", (ctypes.c_uint8 * 16) * 56),
        ("lo_leaf", ctypes.c_uint8 * 16),
        ("lo_mu", ctypes.c_int32),
        ("mid_root", ctypes.c_uint8 * 16),
        ("mid_cw", (ctypes.c_uint8 * 16) * 56),
        ("mid_leaf", ctypes.c_uint8 * 16),
        ("mid_mu", ctypes.c_int32),
        ("mid_mu_eq", ctypes.c_int32),
        ("w", ctypes.c_uint64 * 80),
    ]


class OtKey(ctypes.Structure):
    _fields_ = [
        ("ks", ctypes.c_uint8 * 176),
        ("recv", ctypes.c_uint8 * 18),
        ("c0", ctypes.c_uint32),
        ("w", ctypes.c_uint64 * 32),
    ]


class TtKey(ctypes.Structure):
    _fields_ = [
        ("tab", ctypes.c_uint32 * 24),
        ("tri", ctypes.c_uint32 * 3),
        ("w", ctypes.c_uint64 * 32),
    ]


class LutKey(ctypes.Structure):
    _fields_ = [
        ("root", ctypes.c_uint8 * 16),
        ("cw", (ctypes.c_uint8 * 16) * 8),
        ("cwv", ctypes.c_uint8 * 16),
        ("rout", ctypes.c_uint64),
    ]


class AesKs(ctypes.Structure):
    _fields_ = [("rk", ctypes.c_uint8 * 176)]


_lib = None


def lib():
    global _lib
    if _lib is None:
        L = ctypes.CDLL(build())
        u8p = ctypes.POINTER(ctypes.c_uint8)
        L.ref_aes128_expand.argtypes = [u8p, ctypes.POINTER(AesKs)]
        L.ref_aes128_encrypt.argtypes = [ctypes.POINTER(AesKs), u8p, u8p]
        L.ref_hash_h.argtypes = [u8p, u8p]
        L.ref_hash_c.argtypes = [u8p, u8p]
        L.ref_dealer_key.argtypes = [ctypes.c_uint64, ctypes.POINTER(AesKs)]
        L.ref_prg.argtypes = [ctypes.POINTER(AesKs), ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint64, u8p]
        L.ref_dcf_keygen.argtypes = [ctypes.c_int, ctypes.c_uint64, u8p, u8p, u8p, u8p, u8p, u8p]
        L.ref_dcf_eval.argtypes = [ctypes.c_int, ctypes.c_uint64, u8p, u8p, u8p]
        L.ref_dcf_eval.restype = ctypes.c_int
        L.ref_gate_keygen.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_uint64, ctypes.c_uint32,
                                      ctypes.c_uint64, ctypes.c_uint64, ctypes.POINTER(GateKey),
                                      ctypes.POINTER(GateKey)]
        L.ref_gate_keygen.restype = ctypes.c_uint64
        L.ref_gate_round1.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_uint64,
                                      ctypes.POINTER(GateKey)]
        L.ref_gate_round1.restype = ctypes.c_int
        L.ref_gate_round2.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_uint64,
                                      ctypes.c_int, ctypes.POINTER(GateKey)]
        L.ref_dcfeq_keygen.argtypes = [ctypes.c_int, ctypes.c_uint64, u8p, u8p, u8p, u8p, u8p, u8p]
        L.ref_dcfeq_eval.argtypes = [ctypes.c_int, ctypes.c_uint64, u8p, u8p, u8p]
        L.ref_dcfeq_eval.restype = ctypes.c_int
        L.ref_gate_round2.restype = ctypes.c_uint64
        L.ref_lut_keygen.argtypes = [ctypes.c_int, ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint64,
                                     ctypes.c_uint64, ctypes.c_uint64, ctypes.POINTER(LutKey),
                                     ctypes.POINTER(LutKey)]
        L.ref_lut_eval.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_uint64, ctypes.POINTER(ctypes.c_uint64),
                                   ctypes.POINTER(LutKey)]
        L.ref_lut_eval.restype = ctypes.c_uint64
        L.ref_invsqrt_table.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_uint64)]
        L.ref_ot_plan_info.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_int)]
        L.ref_ot_plan_info.restype = ctypes.c_int
        L.ref_ot_keygen.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_uint64, ctypes.c_uint32,
                                    ctypes.c_uint64, ctypes.c_uint64, ctypes.POINTER(OtKey), ctypes.POINTER(OtKey)]
        L.ref_ot_keygen.restype = ctypes.c_uint64
        u32p = ctypes.POINTER(ctypes.c_uint32)
        L.ref_tt_plan_info.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_int)]
        L.ref_tt_plan_info.restype = ctypes.c_int
        L.ref_tt_tri_positions.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_int)]
        L.ref_tt_tri_positions.restype = ctypes.c_int
        L.ref_tt_keygen.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_uint64, ctypes.c_uint32,
                                    ctypes.c_uint64, ctypes.c_uint64, ctypes.POINTER(TtKey), ctypes.POINTER(TtKey)]
        L.ref_tt_keygen.restype = ctypes.c_uint64
        L.ref_tt_eval_pair.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_uint64,
                                       ctypes.POINTER(TtKey), ctypes.POINTER(TtKey), ctypes.POINTER(ctypes.c_int),
                                       ctypes.POINTER(ctypes.c_int)]
        L.ref_ot_eval_pair.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_uint64, ctypes.c_uint64,
                                       ctypes.POINTER(OtKey), ctypes.POINTER(OtKey), ctypes.POINTER(ctypes.c_int),
                                       ctypes.POINTER(ctypes.c_int), u32p, u32p]
        _lib = L
    return _lib


def _buf(b: bytes):
    return (ctypes.c_uint8 * len(b)).from_buffer_copy(b)


def aes128(key: bytes, pt: bytes) -> bytes:
    ks = AesKs()
    lib().ref_aes128_expand(_buf(key), ctypes.byref(ks))
    out = (ctypes.c_uint8 * 16)()
    lib().ref_aes128_encrypt(ctypes.byref(ks), _buf(pt), out)
    return bytes(out)


def hash_h(x: bytes) -> bytes:
    out = (ctypes.c_uint8 * 16)()
    lib().ref_hash_h(_buf(x), out)
    return bytes(out)


def hash_c(x: bytes) -> bytes:
    out = (ctypes.c_uint8 * 16)()
    lib().ref_hash_c(_buf(x), out)
    return bytes(out)


def prg(seed: int, op: int, purpose: int, idx: int) -> bytes:
    ks = AesKs()
    lib().ref_dealer_key(seed, ctypes.byref(ks))
    out = (ctypes.c_uint8 * 16)()
    lib().ref_prg(ctypes.byref(ks), op, purpose, idx, out)
    return bytes(out)


def dcf_keygen(d: int, alpha: int, s0: bytes, delta: bytes):
    L = max(d - 7, 0)
    r0, r1 = (ctypes.c_uint8 * 16)(), (ctypes.c_uint8 * 16)()
    cw = (ctypes.c_uint8 * (16 * max(L, 1)))()
    leaf = (ctypes.c_uint8 * 16)()
    lib().ref_dcf_keygen(d, alpha, _buf(s0), _buf(delta), r0, r1, cw, leaf)
    return bytes(r0), bytes(r1), bytes(cw)[: 16 * L], bytes(leaf)


def dcf_eval(d: int, x: int, root: bytes, cw: bytes, leaf: bytes) -> int:
    return lib().ref_dcf_eval(d, x, _buf(root), _buf(cw if cw else b"\0" * 16), _buf(leaf))


def dcfeq_keygen(d: int, alpha: int, s0: bytes, delta: bytes):
    L = max(d - 6, 0)
    r0, r1 = (ctypes.c_uint8 * 16)(), (ctypes.c_uint8 * 16)()
    cw = (ctypes.c_uint8 * (16 * max(L, 1)))()
    leaf = (ctypes.c_uint8 * 16)()
    lib().ref_dcfeq_keygen(d, alpha, _buf(s0), _buf(delta), r0, r1, cw, leaf)
    return bytes(r0), bytes(r1), bytes(cw)[: 16 * L], bytes(leaf)


def dcfeq_eval(d: int, x: int, root: bytes, cw: bytes, leaf: bytes) -> int:
    """party's shares: bit0 of 1{x < alpha}, bit1 of 1{x == alpha}"""
    return lib().ref_dcfeq_eval(d, x, _buf(root), _buf(cw if cw else b"\0" * 16), _buf(leaf))


def gate_keygen(kind: int, n: int, s: int, seed: int, op: int, i: int, r_in: int):
    k0, k1 = GateKey(), GateKey()
    r_out = lib().ref_gate_keygen(kind, n, s, seed, op, i, r_in, ctypes.byref(k0), ctypes.byref(k1))
    return k0, k1, r_out


def gate_round1(kind: int, n: int, s: int, xhat: int, key: GateKey) -> int:
    return lib().ref_gate_round1(kind, n, s, xhat, ctypes.byref(key))


def gate_round2(kind: int, n: int, s: int, party: int, xhat: int, bits: int, key: GateKey) -> int:
    """bits: opened round-1 bits, bit0 = high compare, bit1 = low compare, bit2 = high equality,
    bit3 / bit4 = middle compare / equality (three-part split kinds)."""
    return lib().ref_gate_round2(kind, n, s, party, xhat, bits, ctypes.byref(key))


def gate_eval_pair(kind: int, n: int, s: int, xhat: int, k0: GateKey, k1: GateKey) -> int:
    """Both parties, both rounds, with the openings done in place: returns y_hat."""
    b0 = gate_round1(kind, n, s, xhat, k0)
    b1 = gate_round1(kind, n, s, xhat, k1)
    o = b0 ^ b1
    y0 = gate_round2(kind, n, s, 0, xhat, o, k0)
    y1 = gate_round2(kind, n, s, 1, xhat, o, k1)
    return (y0 + y1) & ((1 << n) - 1)


def ot_plan_info(n: int, s: int) -> dict:
    o = (ctypes.c_int * 6)()
    if not lib().ref_ot_plan_info(n, s, o):
        raise ValueError(f"no OT plan for n={n} s={s}")
    return dict(zip(("digits", "g0", "levels", "combines", "naux", "tri0"), list(o)))


def ot_keygen(kind: int, n: int, s: int, seed: int, op: int, i: int, r_in: int):
    k0, k1 = OtKey(), OtKey()
    r_out = lib().ref_ot_keygen(kind, n, s, seed, op, i, r_in, ctypes.byref(k0), ctypes.byref(k1))
    return k0, k1, r_out


def ot_eval_pair(kind: int, n: int, s: int, xhat: int, i: int, k0: OtKey, k1: OtKey):
    """Both parties' OT comparison protocol for element i: (bits0, bits1, tables0, tables1), bits in the
    round-1 encoding (bit0 hi compare, bit1 lo compare, bit2 hi equality), tables = each party's garbled words."""
    b0, b1 = ctypes.c_int(), ctypes.c_int()
    t0, t1 = (ctypes.c_uint32 * 18)(), (ctypes.c_uint32 * 18)()
    lib().ref_ot_eval_pair(kind, n, s, xhat, i, ctypes.byref(k0), ctypes.byref(k1), ctypes.byref(b0),
                           ctypes.byref(b1), t0, t1)
    info = ot_plan_info(n, s)
    return b0.value, b1.value, list(t0)[: info["g0"]], list(t1)[: info["digits"] - info["g0"]]


def ot_round2(kind: int, n: int, s: int, party: int, xhat: int, bits: int, key: OtKey) -> int:
    """round 2 of an OT kind = round 2 of its SPLIT kind over the opened bits and the key's words"""
    g = GateKey()
    for j in range(32):
        g.w[j] = key.w[j]
    return gate_round2(OT_WORD_KIND[kind], n, s, party, xhat, bits, g)


def ot_gate_pair(kind: int, n: int, s: int, xhat: int, i: int, k0: OtKey, k1: OtKey) -> int:
    """Both parties, every round: returns y_hat = y + r_out."""
    b0, b1, _, _ = ot_eval_pair(kind, n, s, xhat, i, k0, k1)
    o = b0 ^ b1
    return (ot_round2(kind, n, s, 0, xhat, o, k0) + ot_round2(kind, n, s, 1, xhat, o, k1)) & ((1 << n) - 1)


def tt_plan_info(kind: int, n: int, s: int) -> dict:
    o = (ctypes.c_int * 4)()
    if not lib().ref_tt_plan_info(kind, n, s, o):
        raise ValueError(f"no truth-table plan for kind={kind} n={n} s={s}")
    return dict(zip(("digits", "rows", "levels", "combines"), list(o)))


def tt_tri_positions(kind: int, n: int, s: int) -> dict:
    """Where the plan keeps each combine's triple bits in a party's triple
    words: tpa[q] (a, b, b' at +0..2), tpc[q] (c, c' at +0..1), mu (the full
    compare's lo mask bit)."""
    o = (ctypes.c_int * 40)()
    if not lib().ref_tt_tri_positions(kind, n, s, o):
        raise ValueError(f"no truth-table plan for kind={kind} n={n} s={s}")
    nc = o[0]
    return {"tpa": [o[1 + 2 * q] for q in range(nc)], "tpc": [o[2 + 2 * q] for q in range(nc)], "mu": o[1 + 2 * nc]}


def tt_keygen(kind: int, n: int, s: int, seed: int, op: int, i: int, r_in: int):
    k0, k1 = TtKey(), TtKey()
    r_out = lib().ref_tt_keygen(kind, n, s, seed, op, i, r_in, ctypes.byref(k0), ctypes.byref(k1))
    return k0, k1, r_out


def tt_eval_pair(kind: int, n: int, s: int, xhat: int, k0: TtKey, k1: TtKey):
    """Both parties' truth-table comparison for one element: (bits0, bits1) in the round-1 encoding
    (bit0 hi compare, bit1 lo compare, bit2 hi equality; the carry kind only bit1)."""
    b0, b1 = ctypes.c_int(), ctypes.c_int()
    lib().ref_tt_eval_pair(kind, n, s, xhat, ctypes.byref(k0), ctypes.byref(k1), ctypes.byref(b0), ctypes.byref(b1))
    return b0.value, b1.value


def tt_round2(kind: int, n: int, s: int, party: int, xhat: int, bits: int, key: TtKey) -> int:
    g = GateKey()
    for j in range(32):
        g.w[j] = key.w[j]
    return gate_round2(TT_WORD_KIND[kind], n, s, party, xhat, bits, g)


def tt_gate_pair(kind: int, n: int, s: int, xhat: int, k0: TtKey, k1: TtKey) -> int:
    """Both parties, every round: returns y_hat = y + r_out."""
    b0, b1 = tt_eval_pair(kind, n, s, xhat, k0, k1)
    o = b0 ^ b1
    return (tt_round2(kind, n, s, 0, xhat, o, k0) + tt_round2(kind, n, s, 1, xhat, o, k1)) & ((1 << n) - 1)


def lut_keygen(n: int, seed: int, op: int, i: int, alpha: int, r_out: int):
    k0, k1 = LutKey(), LutKey()
    lib().ref_lut_keygen(n, seed, op, i, alpha, r_out, ctypes.byref(k0), ctypes.byref(k1))
    return k0, k1


def lut_eval(n: int, party: int, xhat: int, table, key: LutKey) -> int:
    t = (ctypes.c_uint64 * 256)(*[int(v) for v in table])
    return lib().ref_lut_eval(n, party, xhat, t, ctypes.byref(key))


def invsqrt_table(scale: int, nmax: int) -> np.ndarray:
    t = (ctypes.c_uint64 * 256)()
    lib().ref_invsqrt_table(scale, nmax, t)
    return np.array(list(t), dtype=np.uint64)


def gate_key_bytes(key: GateKey) -> dict:
    """Flatten one element's key into the SoA fields the CUDA layout stores."""
    return {
        "hi_root": bytes(key.hi_root), "hi_cw": bytes(key.hi_cw), "hi_leaf": bytes(key.hi_leaf),
        "hi_mu": key.hi_mu, "hi_mu_eq": key.hi_mu_eq, "lo_root": bytes(key.lo_root), "lo_cw": bytes(key.lo_cw),
        "lo_leaf": bytes(key.lo_leaf), "lo_mu": key.lo_mu, "mid_root": bytes(key.mid_root),
        "mid_cw": bytes(key.mid_cw), "mid_leaf": bytes(key.mid_leaf), "mid_mu": key.mid_mu,
        "mid_mu_eq": key.mid_mu_eq, "w": list(key.w),
    }
