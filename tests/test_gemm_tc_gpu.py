"""Tensor-core ring GEMM (tcgen05 kind::i8 limb products) through the C ABI.

Every engine path (tensor cores with operand B MN-major or K-major in shared
memory, wide tiles, and the CUDA-core kernel) must produce the same ring
product as numpy's wrapping uint64 matmul, bit for bit: the Beaver per-sample
product of DDGOrcaBase::matmul 3-arg (gpu_mpc/ddg_orca_base.h:170-205) and
the FC of DDGOrcaBase::matmul 4-arg (ddg_orca_base.h:208-271).  Shapes cover
ragged M/N/K (not multiples of the 128 x BN x 32 tile), multi-tile M, batch,
M = 1, and all-ones operands at the largest reduction length the limb sums
allow (each int32 partial sum then sits just below 2^31).
"""
import numpy as np
import pytest

from tests.gpu_util import dev_bytes, from_dev, ptr, ring_dt, to_dev

PATHS = [0, 5, 4, 2, 3, 1]


def rnd(rng, bw, shape):
    dt = ring_dt(bw)
    return rng.integers(0, np.iinfo(dt).max, size=shape, dtype=dt, endpoint=True)


def mm(a, b, dt):
    return np.matmul(a.astype(np.uint64), b.astype(np.uint64)).astype(dt)


@pytest.fixture
def engine(ddg):
    yield ddg
    ddg.gemm_path(0)


def beaver(ddg, bw, Bt, M, K, N, A, rA, Bm, rB, rC, rng):
    """Both parties' shares through ddg_matmul_share; returns their sum."""
    L = ddg.lib()
    dt = ring_dt(bw)
    Z = (mm(rA, rB, dt) + rC).astype(dt)
    msA0, msB0, z0 = rnd(rng, bw, rA.shape), rnd(rng, bw, rB.shape), rnd(rng, bw, Z.shape)
    parts = [(msA0, msB0, z0), ((rA - msA0).astype(dt), (rB - msB0).astype(dt), (Z - z0).astype(dt))]
    Ah, Bh = (A + rA).astype(dt), (Bm + rB).astype(dt)
    tot = np.zeros((Bt, M, N), dtype=dt)
    import torch

    for p in (0, 1):
        bufs = [to_dev(a) for a in (Ah, Bh) + parts[p]]
        out = dev_bytes(Bt * M * N * bw // 8)
        ddg.check(L.ddg_matmul_share(bw, p, Bt, M, K, N, *[ptr(b) for b in bufs], ptr(out), None))
        torch.cuda.synchronize()
        sh = from_dev(out, dt, Bt * M * N).reshape(Bt, M, N)
        ms_a, ms_b, zz = parts[p]
        want = ((1 - p) * mm(Ah, Bh, dt) - mm(Ah, ms_b, dt) - mm(ms_a, Bh, dt) + zz).astype(dt)
        assert np.array_equal(sh, want), f"party {p} share differs"
        tot = (tot + sh).astype(dt)
    ddg.gemm_status()
    return tot


@pytest.mark.gpu
@pytest.mark.parametrize("path", PATHS)
@pytest.mark.parametrize("bw", [32, 64])
@pytest.mark.parametrize("shape", [(2, 138, 138, 94), (1, 1, 5, 3), (3, 65, 17, 70), (1, 300, 40, 130),
                                   (2, 129, 33, 65), (3, 160, 45, 130), (2, 138, 276, 312)])
def test_beaver_matmul_paths(engine, cuda, path, bw, shape):
    engine.gemm_path(path)
    dt = ring_dt(bw)
    Bt, M, K, N = shape
    rng = np.random.default_rng(M * 7 + K + N + bw + path)
    A, rA = rnd(rng, bw, (Bt, M, K)), rnd(rng, bw, (Bt, M, K))
    Bm, rB = rnd(rng, bw, (Bt, K, N)), rnd(rng, bw, (Bt, K, N))
    rC = rnd(rng, bw, (Bt, M, N))
    tot = beaver(engine, bw, Bt, M, K, N, A, rA, Bm, rB, rC, rng)
    assert np.array_equal(tot, (mm(A, Bm, dt) + rC).astype(dt))


@pytest.mark.gpu
@pytest.mark.parametrize("path", PATHS)
@pytest.mark.parametrize("bw", [32, 64])
@pytest.mark.parametrize("shape", [(70, 94, 188), (300, 282, 376), (1, 1024, 128), (256, 256, 1), (5, 3, 2),
                                   (150, 94, 70), (257, 40, 33)])
def test_fc_paths(engine, cuda, path, bw, shape):
    engine.gemm_path(path)
    L = engine.lib()
    dt = ring_dt(bw)
    M, K, N = shape
    rng = np.random.default_rng(M + K + N + bw)
    x, rx, ry = rnd(rng, bw, (M, K)), rnd(rng, bw, (M, K)), rnd(rng, bw, (M, N))
    W = rng.integers(-3000, 3000, size=(K, N)).astype(np.int64).astype(np.uint64).astype(dt)
    b2s = (rng.integers(-3000, 3000, size=N).astype(np.int64) << 12).astype(np.uint64).astype(dt)
    C = (ry - mm(rx, W, dt)).astype(dt)
    c0 = rnd(rng, bw, C.shape)
    xh = (x + rx).astype(dt)
    bufs = [to_dev(a) for a in (xh, W, b2s, c0)]
    out = dev_bytes(M * N * bw // 8)
    engine.check(L.ddg_fc_share(bw, 0, M, K, N, *[ptr(b) for b in bufs], ptr(out), None))
    import torch

    torch.cuda.synchronize()
    engine.gemm_status()
    got = from_dev(out, dt, M * N).reshape(M, N)
    assert np.array_equal(got, (mm(xh, W, dt) + b2s + c0).astype(dt))


@pytest.mark.gpu
@pytest.mark.parametrize("path", [0, 4, 2, 3])
@pytest.mark.parametrize("bw,K", [(32, 4096), (64, 2048)])
def test_limb_sums_at_the_exactness_bound(engine, cuda, path, bw, K):
    """Party 0's Beaver share with every byte of both concatenated operands at
    255: A_hat = [r_A]0 = -1, B_hat = 1, [r_B]0 = 2, so s1*B_hat - [r_B]0 = -1
    and -B_hat = -1.  The reduction length is 2K, at the bound, and the top
    limb sum P * 2K * 255^2 sits just under 2^31."""
    import torch

    engine.gemm_path(path)
    L = engine.lib()
    dt = ring_dt(bw)
    M, N = 130, 70
    top = np.iinfo(dt).max
    rng = np.random.default_rng(K + bw)
    Ah = np.full((1, M, K), top, dtype=dt)
    msA = np.full((1, M, K), top, dtype=dt)
    Bh = np.ones((1, K, N), dtype=dt)
    msB = np.full((1, K, N), 2, dtype=dt)
    z = rnd(rng, bw, (1, M, N))
    bufs = [to_dev(a) for a in (Ah, Bh, msA, msB, z)]
    out = dev_bytes(M * N * bw // 8)
    engine.check(L.ddg_matmul_share(bw, 0, 1, M, K, N, *[ptr(b) for b in bufs], ptr(out), None))
    torch.cuda.synchronize()
    engine.gemm_status()
    got = from_dev(out, dt, M * N).reshape(1, M, N)
    want = (mm(Ah, Bh, dt) - mm(Ah, msB, dt) - mm(msA, Bh, dt) + z).astype(dt)
    assert np.array_equal(got, want)


@pytest.mark.gpu
@pytest.mark.parametrize("bw", [32, 64])
def test_fc_at_layer_size_matches_numpy(engine, cuda, bw):
    """GCN layer 3 FC at B = 32 samples (M = 4416, K = 282, N = 376) on the
    tensor cores and on the CUDA cores: each equals numpy's wrapping product
    x_hat . W + bias2s + C0 (party 0 of DDGOrcaBase::matmul 4-arg) bit for bit."""
    import torch

    L = engine.lib()
    dt = ring_dt(bw)
    M, K, N = 32 * 138, 282, 376
    rng = np.random.default_rng(bw)
    xh, W, c0 = rnd(rng, bw, (M, K)), rnd(rng, bw, (K, N)), rnd(rng, bw, (M, N))
    b2s = rnd(rng, bw, N)
    want = (mm(xh, W, dt) + b2s[None, :] + c0).astype(dt).reshape(-1)
    bufs = [to_dev(a) for a in (xh, W, b2s, c0)]
    for path in (0, 1):
        engine.gemm_path(path)
        out = dev_bytes(M * N * bw // 8)
        engine.check(L.ddg_fc_share(bw, 0, M, K, N, *[ptr(b) for b in bufs], ptr(out), None))
        torch.cuda.synchronize()
        got = from_dev(out, dt, M * N)
        assert np.array_equal(got, want), f"path {path}: {np.count_nonzero(got != want)} elements differ"
    engine.gemm_status()
