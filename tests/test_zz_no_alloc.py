"""ddg_gate_eval_pair_noalloc: the allocation-free gate evaluation.

Some callers cannot call cudaMalloc (a host framework that owns all device
memory, pipelines that must not take cudaMalloc's implicit synchronisation,
fixed memory budgets).  For them the library evaluates one gate for both
parties with its scratch in a file-scope device array.  This file checks,
through the C ABI, that two calls in a row give exactly the result of the
existing entry points (ddg_gate_round1 / ddg_gate_round2 per party with
caller-allocated buffers, then adding the shares), and that sizes above the
stated limit are rejected.  It sorts last so a stop-at-first-failure run has
already run every other test.
"""
import numpy as np
import pytest

from tests.gpu_util import dev_bytes, from_dev, ptr, ring_dt, to_dev

S = 12
MAX_N = 262144


def keys_and_input(ddg, kind, bw, n, seed):
    """Masked input x_hat = x + r_in and both parties' keys; returns the plain
    x and the dealer's output mask r_out as well."""
    dt = ring_dt(bw)
    rng = np.random.default_rng(seed)
    hi = np.iinfo(dt).max
    x = rng.integers(0, hi, size=n, dtype=dt, endpoint=True)
    if kind == 3:
        x &= dt(hi >> 1)
    r = rng.integers(0, hi, size=n, dtype=dt, endpoint=True)
    kb = ddg.gate_key_bytes(kind, bw, S, n)
    k0, k1 = dev_bytes(kb), dev_bytes(kb)
    d_r, d_ro = to_dev(r), dev_bytes(n * bw // 8)
    ddg.gate_keygen(kind, bw, S, n, seed, 5, ptr(d_r), ptr(d_ro), ptr(k0), ptr(k1))
    return to_dev((x + r).astype(dt)), k0, k1, x, from_dev(d_ro, dt, n).copy()


def plaintext(kind, bw, x):
    """The gate's function on the plain input: ReLU, ReLU(floor(x/2^s)),
    floor(x/2^s) signed, floor(x/2^s) for x in [0, 2^(bw-1))."""
    dt = ring_dt(bw)
    sx = x.view(np.int32 if bw == 32 else np.int64).astype(np.int64)
    y = {0: np.maximum(sx, 0), 1: np.maximum(sx >> S, 0), 2: sx >> S, 3: sx >> S}[kind]
    return y.astype(np.int64).view(np.uint64).astype(dt)


def existing_entry_points(ddg, kind, bw, n, d_x, k0, k1):
    dt = ring_dt(bw)
    w = (n + 31) // 32
    bits = {(p, h): dev_bytes(4 * w) for p in (0, 1) for h in ("hi", "lo")}
    for p, k in ((0, k0), (1, k1)):
        ddg.gate_round1(kind, bw, S, n, ptr(d_x), ptr(k), ptr(bits[p, "hi"]), ptr(bits[p, "lo"]))
    sh = [dev_bytes(n * bw // 8) for _ in range(2)]
    for p, k in ((0, k0), (1, k1)):
        q = 1 - p
        ddg.gate_round2(kind, bw, S, n, p, ptr(d_x), ptr(bits[p, "hi"]), ptr(bits[q, "hi"]), ptr(bits[p, "lo"]),
                        ptr(bits[q, "lo"]), ptr(k), ptr(sh[p]))
    import torch

    torch.cuda.synchronize()
    return (from_dev(sh[0], dt, n) + from_dev(sh[1], dt, n)).astype(dt)


def noalloc(ddg, kind, bw, n, d_x, k0, k1):
    out = dev_bytes(n * bw // 8)
    ddg.check(ddg.lib().ddg_gate_eval_pair_noalloc(kind, bw, S, n, ptr(d_x), ptr(k0), ptr(k1), ptr(out), None))
    import torch

    torch.cuda.synchronize()
    return from_dev(out, ring_dt(bw), n)


# consecutive calls share the scratch array; the order makes every ARS / LRS
# call follow a call of another kind (LRS writes no high-comparison bits and
# ARS reads both halves, so stale words from the call before would show), and
# the first call fills the whole array
CALLS = ((1, MAX_N, 11), (3, 40_001, 12), (2, 100_003, 13), (0, 77, 14), (3, MAX_N, 15), (2, 33, 16))


@pytest.mark.gpu
@pytest.mark.parametrize("bw", [32, 64])
def test_noalloc_calls_in_a_row_match_existing_entry_points(ddg, cuda, bw):
    for kind, n, seed in CALLS:
        d_x, k0, k1, x, r_out = keys_and_input(ddg, kind, bw, n, seed)
        want = existing_entry_points(ddg, kind, bw, n, d_x, k0, k1)
        got = noalloc(ddg, kind, bw, n, d_x, k0, k1)
        assert np.array_equal(got, want), (kind, n)
        # and the gate's function itself: y_hat = f(x) + r_out
        assert np.array_equal(got, (plaintext(kind, bw, x) + r_out).astype(ring_dt(bw))), (kind, n)


@pytest.mark.gpu
def test_noalloc_rejects_sizes_above_limit(ddg, cuda):
    with pytest.raises(ddg.DdgError) as e:
        ddg.check(ddg.lib().ddg_gate_eval_pair_noalloc(0, 32, S, MAX_N + 1, 1, 1, 1, 1, None))
    assert e.value.code == 1 and "no-allocation limit" in str(e.value)
