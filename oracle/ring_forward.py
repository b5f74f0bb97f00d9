"""Plaintext integer forward of the affinity branch -- TEST INFRASTRUCTURE ONLY.

Used by tests/, ``__graft_entry__.smoke()`` and bench.py's cpu_baseline leg as
the oracle the two-party CUDA path must reproduce.  Nothing in the product
imports it.

Two modes over the ring Z_2^n (n = 32 or 64, scale s = 12):

``protocol_forward``  -- the exact integer function the reference's 2PC graph
    computes, in its op order (this is what the MPC output must equal bit for
    bit):
      * secure adjacency normalisation (gpu_mpc/secure_adj_norm.h:394-659):
        deg = rowsum(A_raw); t = T[deg] with T[0]=0,
        T[d]=llround(2^s/sqrt(d)) (d<=138, table at :139-184);
        left = A*t_i (no truncation, :609-624); A_hat = floor(left*t_j / 2^s)
        (TrFloor, :626-651);
      * GCN layer, aggregate-first (gpu_mpc/gcn_layer.h:107-116,
        sytorch/layers/layers.h:67-90): AX = floor(A_hat@H / 2^s) per sample,
        Z = AX@W + (b<<s) (bias at 2s, deepdtagen_inference.cu:169-178),
        H' = ReLU(floor(Z / 2^s));
      * masked max-pool (deepdtagen.h:198-202, masked_maxpool_layer.h:72-126):
        masked = floor(H3*mask / 2^s), then levels of
        even + ReLU(odd - even) over node pairs (2p, 2p+1), an odd last node
        carried to the next level;
      * head (deepdtagen.h:209-220): ReLU(trunc(FC)) for dfc1, ffc1-3;
        trunc(FC) for dfc2; concat [d2 | protein] per row (:45-100); fout
        without truncation;
      * output (ddg_orca_base.h:296-302): arithmetic shift of the revealed
        2s-scale value by s; AFFINITY = int32(value)/2^s
        (deepdtagen_inference.cu:594-606).
    Truncations are exact floors (the reference's TrFloor semantics).  At the
    sites whose operands are non-negative (A_hat, A_hat@H, H3*mask) the
    value must lie in [0, 2^(n-1)); ``protocol_forward`` checks that and
    raises if a ring overflow breaks it.

``ff_forward`` -- restatement of reference/fixed_forward.py:55-95
    (FixedAffinity._drug_path_fx / _fusion_fx): X@W first, then A_hat@,
    float-normalised A_hat quantised, sentinel masked max.  It exists only to
    pin the shared primitives against golden vectors produced by the
    reference code itself (tests/golden/).
"""
from __future__ import annotations

import math

import numpy as np

NMAX = 138


def invsqrt_table(scale: int = 12, nmax: int = NMAX) -> np.ndarray:
    t = np.zeros(256, dtype=np.uint64)
    q = math.ldexp(1.0, scale)
    for d in range(1, min(nmax, 255) + 1):
        t[d] = int(math.floor(q / math.sqrt(d) + 0.5))  # llround on a positive value
    return t


class Ring:
    def __init__(self, n: int):
        assert n in (32, 64)
        self.n = n
        self.M = np.uint64((1 << n) - 1) if n < 64 else np.uint64(0xFFFFFFFFFFFFFFFF)

    def red(self, x):
        return np.asarray(x, dtype=np.uint64) & self.M

    def signed(self, x) -> np.ndarray:
        x = self.red(x)
        if self.n == 64:
            return x.view(np.int64)
        v = x.astype(np.int64)
        return np.where(v >= (1 << 31), v - (1 << 32), v)

    def from_signed(self, v) -> np.ndarray:
        return self.red(np.asarray(v, dtype=np.int64).view(np.uint64))

    def mm(self, a, b):
        """(…,m,k)@(…,k,p) mod 2^n; numpy's integer matmul wraps mod 2^64."""
        return self.red(np.matmul(np.asarray(a, np.uint64), np.asarray(b, np.uint64)))

    def ars(self, x, s):
        return self.from_signed(self.signed(x) >> s)

    def relu(self, x):
        sx = self.signed(x)
        return self.from_signed(np.where(sx >= 0, sx, 0))

    def relu_ars(self, x, s):
        return self.from_signed(np.maximum(self.signed(x) >> s, 0))

    def lrs_nonneg(self, x, s, site: str):
        sx = self.signed(x)
        if (sx < 0).any():
            raise OverflowError(f"{site}: value outside [0, 2^(n-1)) -- ring overflow")
        return self.red(sx >> s)


def maxpool_tree(R: Ring, cur: np.ndarray) -> np.ndarray:
    """cur (B, count, F) -> (B, F) by levels of even + ReLU(odd - even)."""
    while cur.shape[1] > 1:
        cnt = cur.shape[1]
        pairs = cnt // 2
        even = cur[:, 0:2 * pairs:2]
        odd = cur[:, 1:2 * pairs:2]
        nxt = R.red(even + R.relu(R.red(odd - even)))
        if cnt % 2:
            nxt = np.concatenate([nxt, cur[:, cnt - 1:cnt]], axis=1)
        cur = nxt
    return cur[:, 0]


def protocol_forward(x_ring, adj_ring, mask_ring, protein_ring, qlayers, n: int, s: int = 12,
                     nmax: int = NMAX, trace: dict | None = None):
    """Integer forward.  Inputs are ring arrays: x (B,nmax,94) at s, adj (B,nmax,nmax)
    0/1 at scale 0, mask (B,nmax,376) at s, protein (B,128) at s; qlayers = nine
    (W (in,out) int64, b int64).  Returns (out_ring (B,), affinity float64 (B,))."""
    R = Ring(n)
    A = R.red(adj_ring)
    B = A.shape[0]
    T = invsqrt_table(s, nmax)
    deg = R.red(A.sum(axis=-1))
    t = T[(deg & np.uint64(255)).astype(np.int64)]
    left = R.red(A * t[:, :, None])
    w = R.red(left * t[:, None, :])
    A_hat = R.lrs_nonneg(w, s, "adj-norm")
    tr = trace if trace is not None else {}
    tr["deg"], tr["inv"], tr["adj_left"], tr["adj_prod"], tr["A_hat"] = deg, t, left, w, A_hat

    def fc(x, W, b):
        return R.red(R.mm(x, R.from_signed(W)) + R.from_signed(b << s))

    H = R.red(x_ring)
    for li in range(3):
        W, b = qlayers[li]
        P = R.mm(A_hat, H)
        AX = R.lrs_nonneg(P, s, f"gcn{li}.AX")
        Z = fc(AX, W, b)
        H = R.relu_ars(Z, s)
        tr[f"gcn{li}.P"], tr[f"gcn{li}.AX"], tr[f"gcn{li}.Z"], tr[f"gcn{li}.H"] = P, AX, Z, H
    prod = R.red(H * R.red(mask_ring))
    masked = R.lrs_nonneg(prod, s, "mask-mul")
    pooled = maxpool_tree(R, masked)
    tr["mask_prod"], tr["masked"], tr["pooled"] = prod, masked, pooled
    W, b = qlayers[3]
    d1 = R.relu_ars(fc(pooled, W, b), s)
    W, b = qlayers[4]
    d2z = fc(d1, W, b)
    d2 = R.ars(d2z, s)
    fused = np.concatenate([d2, R.red(protein_ring)], axis=1)
    tr["d1"], tr["d2z"], tr["d2"], tr["fused"] = d1, d2z, d2, fused
    h = fused
    for li in (5, 6, 7):
        W, b = qlayers[li]
        h = R.relu_ars(fc(h, W, b), s)
        tr[f"f{li - 4}"] = h
    W, b = qlayers[8]
    o2s = fc(h, W, b)
    out = R.ars(o2s, s)[:, 0]
    tr["out2s"], tr["out"] = o2s[:, 0], out
    aff = (out.astype(np.uint64) & np.uint64(0xFFFFFFFF)).astype(np.uint32).view(np.int32).astype(np.float64)
    return out, aff / float(1 << s)


# ---------------------------------------------------------------- fixed_forward restatement

def to_fixed(x, scale: int) -> np.ndarray:
    """round half away from zero (reference/fixedpoint.py:28-41)."""
    x = np.asarray(x, dtype=np.float64) * float(1 << scale)
    return np.where(x >= 0, np.floor(x + 0.5), np.ceil(x - 0.5)).astype(np.int64)


def _wrap(x, bw: int):
    if bw >= 64:
        return x
    m = (1 << bw) - 1
    xm = np.asarray(x, np.int64) & m
    return np.where(xm >= (1 << (bw - 1)), xm - (1 << bw), xm)


def _fmm(a, b, s):
    """fixed_matmul: exact integer product then floor shift (values fit int64 here)."""
    return np.matmul(np.asarray(a, np.int64), np.asarray(b, np.int64)) >> s


def ff_forward(X, A_hat_float, mask, pvec_float, float_layers, s: int = 12, bw: int = 64):
    """One sample, reference/fixed_forward.py semantics. float_layers = nine
    (W (out,in) f32, b f32). Returns (pmvo_fx (128,), out_fx (1,), pooled (376,))."""
    q = [(to_fixed(W, s), to_fixed(b, s)) for W, b in float_layers]
    Xf, Af = to_fixed(X, s), to_fixed(A_hat_float, s)
    sentinel = np.int64(-(1 << (bw - 2)))
    H = Xf
    for W, b in q[:3]:
        XW = _wrap(_fmm(H, W.T, s), bw)
        o = _wrap(_fmm(Af, XW, s), bw)
        H = np.maximum(_wrap(o + b, bw), 0)
    keep = np.asarray(mask).reshape(-1, 1) != 0
    pooled = np.where(keep, H, sentinel).max(axis=0)

    def lin(x, W, b):
        return _wrap(_wrap(_fmm(np.atleast_2d(x), W.T, s), bw) + b, bw).reshape(-1)

    h = np.maximum(lin(pooled, *q[3]), 0)
    pmvo = lin(h, *q[4])
    h = np.concatenate([pmvo, to_fixed(pvec_float, s)])
    for k in range(5, 9):
        h = lin(h, *q[k])
        if k < 8:
            h = np.maximum(h, 0)
    return pmvo, h, pooled
