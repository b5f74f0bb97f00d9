"""Per-op parity of the linear layers and the DPF LUT through the C ABI.

LUT: keys and shares against oracle/fss_ref.c; reconstruction against the
public table for every degree 0..138 (secure_adj_norm.h:139-184).  Beaver
product, Beaver matmul and FC: each party's share against the formula in
numpy ring arithmetic, and the reconstruction against the plaintext product.
"""
import numpy as np
import pytest

from oracle import fss_ref as F
from oracle.ring_forward import invsqrt_table
from tests.gpu_util import dev_bytes, from_dev, ptr, ring_dt, to_dev


def rnd(rng, bw, shape):
    dt = ring_dt(bw)
    return rng.integers(0, np.iinfo(dt).max, size=shape, dtype=dt, endpoint=True)


def sync():
    import torch

    torch.cuda.synchronize()


@pytest.mark.gpu
@pytest.mark.parametrize("bw", [32, 64])
def test_lut_matches_oracle(ddg, cuda, bw):
    L = ddg.lib()
    dt = ring_dt(bw)
    rng = np.random.default_rng(bw)
    degs = np.concatenate([np.arange(139), rng.integers(0, 139, size=61)]).astype(dt)
    n = degs.size
    r_deg, r_out = rnd(rng, bw, n), rnd(rng, bw, n)
    kb = int(L.ddg_lut_key_bytes(bw, n))
    k0, k1 = dev_bytes(kb), dev_bytes(kb)
    d_a, d_ro = to_dev(r_deg), to_dev(r_out)
    ddg.check(L.ddg_lut_keygen(bw, n, 3, 11, ptr(d_a), ptr(d_ro), ptr(k0), ptr(k1), None))
    table = invsqrt_table(12, 138).astype(dt)
    d_t = to_dev(table)
    xh = (degs + r_deg).astype(dt)
    d_x = to_dev(xh)
    sh = [dev_bytes(n * bw // 8) for _ in range(2)]
    for p, k in ((0, k0), (1, k1)):
        ddg.check(L.ddg_lut_eval(bw, n, p, ptr(d_x), ptr(d_t), ptr(k), ptr(sh[p]), None))
    sync()
    s0, s1 = from_dev(sh[0], dt, n), from_dev(sh[1], dt, n)
    assert np.array_equal((s0 + s1 - r_out).astype(dt), table[degs.astype(np.int64)])
    tab = [int(v) for v in table]
    for i in range(0, n, 7):
        o0, o1 = F.lut_keygen(bw, 3, 11, i, int(r_deg[i]) & 255, int(r_out[i]))
        assert int(s0[i]) == F.lut_eval(bw, 0, int(xh[i]), tab, o0)
        assert int(s1[i]) == F.lut_eval(bw, 1, int(xh[i]), tab, o1)


@pytest.mark.gpu
@pytest.mark.parametrize("bw", [32, 64])
def test_tt_lut_matches_restated_keys(ddg, cuda, bw):
    """Truth-table LUT: every key entry equals its restatement (party 0's entry u of
    lookup i = slot u mod (16 / word) of AES_dealer(i + (u div slots) * n || op || 0x180), party
    1's = table[(u - alpha) mod 256] + r_out - party 0's), the shares are the entries at
    x_hat mod 256, and they reconstruct table[degree] + r_out for every degree 0..138."""
    L = ddg.lib()
    dt = ring_dt(bw)
    W = bw // 8
    rng = np.random.default_rng(bw + 5)
    degs = np.concatenate([np.arange(139), rng.integers(0, 139, size=61)]).astype(dt)
    n = degs.size
    r_deg, r_out = rnd(rng, bw, n), rnd(rng, bw, n)
    kb = int(L.ddg_tt_lut_key_bytes(bw, n))
    k0, k1 = dev_bytes(kb), dev_bytes(kb)
    table = invsqrt_table(12, 138).astype(dt)
    d_a, d_ro, d_t = to_dev(r_deg), to_dev(r_out), to_dev(table)
    ddg.check(L.ddg_tt_lut_keygen(bw, n, 3, 11, ptr(d_a), ptr(d_ro), ptr(d_t), ptr(k0), ptr(k1), None))
    xh = (degs + r_deg).astype(dt)
    d_x = to_dev(xh)
    sh = [dev_bytes(n * W) for _ in range(2)]
    for p, k in ((0, k0), (1, k1)):
        ddg.check(L.ddg_tt_lut_eval(bw, n, ptr(d_x), ptr(k), ptr(sh[p]), None))
    sync()
    s0, s1 = from_dev(sh[0], dt, n), from_dev(sh[1], dt, n)
    assert np.array_equal((s0 + s1 - r_out).astype(dt), table[degs.astype(np.int64)])
    t0 = k0.cpu().numpy()[: 256 * n * W].view(dt).reshape(256, n)
    t1 = k1.cpu().numpy()[: 256 * n * W].view(dt).reshape(256, n)
    M = (1 << bw) - 1
    per = 16 // W
    for i in list(range(0, n, 17)) + [n - 1]:
        a = int(r_deg[i]) & 255
        for u in range(0, 256, 37):
            blk = F.prg(3, 11, 0x180, (u // per) * n + i)
            e0 = int.from_bytes(blk[W * (u % per): W * (u % per) + W], "little")
            assert int(t0[u, i]) == e0
            assert int(t1[u, i]) == (int(table[(u - a) & 255]) + int(r_out[i]) - e0) & M
        u = int(xh[i]) & 255
        assert int(s0[i]) == int(t0[u, i]) and int(s1[i]) == int(t1[u, i])


@pytest.mark.gpu
@pytest.mark.parametrize("bw", [32, 64])
@pytest.mark.parametrize("bcast", [0, 1, 2])
def test_mul_share(ddg, cuda, bw, bcast):
    L = ddg.lib()
    dt = ring_dt(bw)
    rng = np.random.default_rng(bcast + bw)
    Bt, R, C = 3, 5, 7
    n = Bt * R * C
    x, rx = rnd(rng, bw, n), rnd(rng, bw, n)
    ylen = n if bcast == 0 else (Bt * R if bcast == 1 else Bt * C)
    y, ry, rz = rnd(rng, bw, ylen), rnd(rng, bw, ylen), rnd(rng, bw, n)
    e = np.arange(n)
    yi = e if bcast == 0 else (e // C if bcast == 1 else (e // (R * C)) * C + e % C)
    Z = (rx * ry[yi] + rz).astype(dt)
    msx0, msy0, z0 = rnd(rng, bw, n), rnd(rng, bw, ylen), rnd(rng, bw, n)
    parts = [(msx0, msy0, z0), ((rx - msx0).astype(dt), (ry - msy0).astype(dt), (Z - z0).astype(dt))]
    xh, yh = (x + rx).astype(dt), (y + ry).astype(dt)
    outs = []
    for p in (0, 1):
        bufs = [to_dev(a) for a in (xh, yh) + parts[p]]
        out = dev_bytes(n * bw // 8)
        ddg.check(L.ddg_mul_share(bw, p, n, bcast, R, C, *[ptr(b) for b in bufs], ptr(out), None))
        sync()
        outs.append(from_dev(out, dt, n))
        ms_x, ms_y, zz = parts[p]
        want = ((1 - p) * xh * yh[yi] - xh * ms_y[yi] - ms_x * yh[yi] + zz).astype(dt)
        assert np.array_equal(outs[p], want)
    assert np.array_equal((outs[0] + outs[1] - rz).astype(dt), (x * y[yi]).astype(dt))


@pytest.mark.gpu
@pytest.mark.parametrize("bw", [32, 64])
@pytest.mark.parametrize("shape", [(2, 138, 138, 94), (1, 1, 5, 3), (3, 65, 17, 70)])
def test_matmul_share(ddg, cuda, bw, shape):
    L = ddg.lib()
    dt = ring_dt(bw)
    Bt, M, K, N = shape
    rng = np.random.default_rng(M + K + N + bw)
    A, rA = rnd(rng, bw, (Bt, M, K)), rnd(rng, bw, (Bt, M, K))
    Bm, rB = rnd(rng, bw, (Bt, K, N)), rnd(rng, bw, (Bt, K, N))
    rC = rnd(rng, bw, (Bt, M, N))
    Z = (np.matmul(rA.astype(np.uint64), rB.astype(np.uint64)).astype(dt) + rC).astype(dt)
    msA0, msB0, z0 = rnd(rng, bw, rA.shape), rnd(rng, bw, rB.shape), rnd(rng, bw, Z.shape)
    parts = [(msA0, msB0, z0), ((rA - msA0).astype(dt), (rB - msB0).astype(dt), (Z - z0).astype(dt))]
    Ah, Bh = (A + rA).astype(dt), (Bm + rB).astype(dt)
    tot = np.zeros((Bt, M, N), dtype=dt)
    for p in (0, 1):
        bufs = [to_dev(a) for a in (Ah, Bh) + parts[p]]
        out = dev_bytes(Bt * M * N * bw // 8)
        ddg.check(L.ddg_matmul_share(bw, p, Bt, M, K, N, *[ptr(b) for b in bufs], ptr(out), None))
        sync()
        tot = (tot + from_dev(out, dt).reshape(-1)[: Bt * M * N].reshape(Bt, M, N)).astype(dt)
    want = (np.matmul(A.astype(np.uint64), Bm.astype(np.uint64)).astype(dt) + rC).astype(dt)
    assert np.array_equal(tot, want)


@pytest.mark.gpu
@pytest.mark.parametrize("bw", [32, 64])
def test_fc_share(ddg, cuda, bw):
    L = ddg.lib()
    dt = ring_dt(bw)
    rng = np.random.default_rng(bw)
    M, K, N = 70, 94, 188
    x, rx, ry = rnd(rng, bw, (M, K)), rnd(rng, bw, (M, K)), rnd(rng, bw, (M, N))
    W = rng.integers(-3000, 3000, size=(K, N)).astype(np.int64).astype(np.uint64).astype(dt)
    b2s = (rng.integers(-3000, 3000, size=N).astype(np.int64) << 12).astype(np.uint64).astype(dt)
    C = (ry - np.matmul(rx.astype(np.uint64), W.astype(np.uint64)).astype(dt)).astype(dt)
    c0 = rnd(rng, bw, C.shape)
    c1 = (C - c0).astype(dt)
    xh = (x + rx).astype(dt)
    tot = np.zeros((M, N), dtype=dt)
    for p, cp in ((0, c0), (1, c1)):
        bufs = [to_dev(a) for a in (xh, W, b2s, cp)]
        out = dev_bytes(M * N * bw // 8)
        ddg.check(L.ddg_fc_share(bw, p, M, K, N, *[ptr(b) for b in bufs], ptr(out), None))
        sync()
        tot = (tot + from_dev(out, dt, M * N).reshape(M, N)).astype(dt)
    want = (np.matmul(x.astype(np.uint64), W.astype(np.uint64)).astype(dt) + b2s + ry).astype(dt)
    assert np.array_equal(tot, want)
