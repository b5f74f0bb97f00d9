"""Gate kernels (DCF + select / truncation) against the C oracle, through the C ABI.

Mirrors the reference's own primitive tests (gpu_mpc/lss/lss_test.cpp:330-389:
ReLU / compare / MSB checked bit-exact on random and boundary inputs, both
parties, openings done in the test): here every party's key bytes, round-1
bits and round-2 shares are compared with oracle/fss_ref.c element by element,
and the reconstructed outputs with the plaintext function.
"""
import numpy as np
import pytest

from oracle import fss_ref as F
from oracle.ring_forward import Ring
from tests.gpu_util import dev_bytes, from_dev, ptr, ring_dt, to_dev

S = 12
KINDS = [F.GATE_RELU, F.GATE_RELU_ARS, F.GATE_ARS, F.GATE_LRS, F.GATE_RELU_SPLIT, F.GATE_RELU_ARS_SPLIT,
         F.GATE_LRS_SPLIT, F.GATE_RELU_SPLIT3, F.GATE_RELU_ARS_SPLIT3]
LRS_KINDS = (F.GATE_LRS, F.GATE_LRS_SPLIT)


def plain(kind, x, bw):
    R = Ring(bw)
    if kind in (F.GATE_RELU, F.GATE_RELU_SPLIT, F.GATE_RELU_SPLIT3):
        return R.relu(x)
    if kind in (F.GATE_RELU_ARS, F.GATE_RELU_ARS_SPLIT, F.GATE_RELU_ARS_SPLIT3):
        return R.relu_ars(x, S)
    if kind == F.GATE_ARS:
        return R.ars(x, S)
    return R.red(R.signed(x) >> S)


def boundary(bw, kind):
    M = (1 << bw) - 1
    v = [0, 1, 2, M, M - 1, 1 << (bw - 1), (1 << (bw - 1)) - 1, (1 << (bw - 1)) + 1, (1 << S) - 1, 1 << S,
         (1 << S) + 1, M - (1 << S) + 1, M - (1 << S)]
    if kind in LRS_KINDS:
        v = [x & (M >> 1) for x in v]
    return v


def make_inputs(bw, kind, n, seed):
    rng = np.random.default_rng(seed)
    dt = ring_dt(bw)
    hi = np.iinfo(dt).max
    x = rng.integers(0, hi, size=n, dtype=dt, endpoint=True)
    if kind in LRS_KINDS:
        x &= dt(hi >> 1)
    b = boundary(bw, kind)
    x[: min(len(b), n)] = np.array(b[: min(len(b), n)], dtype=dt)
    r = rng.integers(0, hi, size=n, dtype=dt, endpoint=True)
    r[:4] = np.array([0, hi, 1 << (bw - 1), (1 << S) - 1][: min(4, n)], dtype=dt)[: min(4, n)]
    # every 5th element: x_hat agrees with r on the bits above the low `S` (split-compare equality branch)
    sel = np.arange(n) % 5 == 4
    lowmask = dt((1 << S) - 1)
    xh = (r & ~lowmask) | (rng.integers(0, 1 << S, size=n, dtype=dt) & lowmask)
    x[sel] = (xh - r).astype(dt)[sel]
    # every 7th element: x_hat agrees with r on carry bits 5..11 (split LRS equality branch)
    sel2 = np.arange(n) % 7 == 3
    m31 = dt(31)
    xh2 = (r & ~m31) | (rng.integers(0, 32, size=n, dtype=dt) & m31)
    xh2 = (xh2 + (rng.integers(0, 1 << 16, size=n, dtype=dt) << dt(12))).astype(dt)
    x[sel2] = (xh2 - r).astype(dt)[sel2]
    # every 11th element: x_hat agrees with r on bits 18..bw-2 (three-part split: U1 equal)
    sel3 = np.arange(n) % 11 == 6
    lo18 = dt((1 << 18) - 1)
    xh3 = (r & ~lo18) | (rng.integers(0, 1 << 18, size=n, dtype=dt) & lo18)
    x[sel3] = (xh3 - r).astype(dt)[sel3]
    if kind in LRS_KINDS:
        x &= dt(hi >> 1)
    return x, r


def run_gate(ddg, kind, bw, n, x, r, seed=5, op=3):
    dt = ring_dt(bw)
    kb = ddg.gate_key_bytes(kind, bw, S, n)
    k0, k1 = dev_bytes(kb), dev_bytes(kb)
    d_r, d_ro = to_dev(r), dev_bytes(n * (bw // 8))
    ddg.gate_keygen(kind, bw, S, n, seed, op, ptr(d_r), ptr(d_ro), ptr(k0), ptr(k1))
    xh = (x + r).astype(dt)
    d_x = to_dev(xh)
    words = (n + 31) // 32
    bits = {(p, h): dev_bytes(16 * words) for p in (0, 1) for h in ("hi", "lo")}  # up to 4 arrays of bits
    for p, k in ((0, k0), (1, k1)):
        ddg.gate_round1(kind, bw, S, n, ptr(d_x), ptr(k), ptr(bits[p, "hi"]), ptr(bits[p, "lo"]))
    shares = [dev_bytes(n * (bw // 8)) for _ in range(2)]
    for p, k in ((0, k0), (1, k1)):
        q = 1 - p
        ddg.gate_round2(kind, bw, S, n, p, ptr(d_x), ptr(bits[p, "hi"]), ptr(bits[q, "hi"]), ptr(bits[p, "lo"]),
                        ptr(bits[q, "lo"]), ptr(k), ptr(shares[p]))
    import torch

    torch.cuda.synchronize()
    return dict(k0=k0.cpu().numpy(), k1=k1.cpu().numpy(), rout=from_dev(d_ro, dt, n),
                bits={kk: from_dev(v, np.uint32, 4 * words) for kk, v in bits.items()},
                y0=from_dev(shares[0], dt, n), y1=from_dev(shares[1], dt, n), xh=xh)


def key_fields(blob, lay, n, e, bw):
    """One element's key out of the SoA blob, in the oracle's per-element form."""
    f = {}
    for side in ("hi", "mid", "lo"):
        L = lay[f"{side}_levels"]
        if lay[f"{side}_root"] == 0 and lay[f"{side}_cw"] == 0:
            continue
        root = blob[lay[f"{side}_root"] + 16 * e: lay[f"{side}_root"] + 16 * e + 16].tobytes()
        cw = b"".join(blob[lay[f"{side}_cw"] + 16 * (j * n + e): lay[f"{side}_cw"] + 16 * (j * n + e) + 16].tobytes()
                      for j in range(L))
        leaf = blob[lay[f"{side}_leaf"] + 16 * e: lay[f"{side}_leaf"] + 16 * e + 16].tobytes()
        mu = (int(blob[lay[f"{side}_mu"]:].view(np.uint32)[e // 32]) >> (e % 32)) & 1
        mu_eq = (int(blob[lay[f"{side}_mu_eq"]:].view(np.uint32)[e // 32]) >> (e % 32)) & 1 if (
            side in ("hi", "mid") and lay[f"{side}_mu_eq"]) else 0
        f[side] = (root, cw, leaf, mu, mu_eq)
    return f


@pytest.mark.gpu
@pytest.mark.parametrize("bw", [32, 64])
@pytest.mark.parametrize("kind", KINDS)
def test_gate_keys_bits_shares_match_oracle(ddg, cuda, bw, kind):
    n = 300
    x, r = make_inputs(bw, kind, n, seed=kind * 10 + bw)
    out = run_gate(ddg, kind, bw, n, x, r)
    lay = ddg.gate_key_layout(kind, bw, S, n)
    nw = F.GATE_NWORDS[kind]
    dt = ring_dt(bw)
    w0 = out["k0"][lay["words"]:].view(dt)
    w1 = out["k1"][lay["words"]:].view(dt)
    for e in range(n):
        k0, k1, ry = F.gate_keygen(kind, bw, S, 5, 3, e, int(r[e]))
        assert int(out["rout"][e]) == ry
        for blob, ref in ((out["k0"], k0), (out["k1"], k1)):
            g = key_fields(blob, lay, n, e, bw)
            rb = F.gate_key_bytes(ref)
            if "hi" in g:
                L = lay["hi_levels"]
                assert g["hi"][0] == rb["hi_root"] and g["hi"][1] == rb["hi_cw"][: 16 * L]
                assert g["hi"][2] == rb["hi_leaf"] and g["hi"][3] == rb["hi_mu"]
                assert g["hi"][4] == (rb["hi_mu_eq"] if kind in F.SPLIT_KINDS else 0)
            if "lo" in g:
                L = lay["lo_levels"]
                assert g["lo"][0] == rb["lo_root"] and g["lo"][1] == rb["lo_cw"][: 16 * L]
                assert g["lo"][2] == rb["lo_leaf"] and g["lo"][3] == rb["lo_mu"]
            if "mid" in g:
                L = lay["mid_levels"]
                assert g["mid"][0] == rb["mid_root"] and g["mid"][1] == rb["mid_cw"][: 16 * L]
                assert g["mid"][2] == rb["mid_leaf"] and g["mid"][3] == rb["mid_mu"]
                assert g["mid"][4] == rb["mid_mu_eq"]
        for wi in range(nw):
            assert int(w0[wi * n + e]) == k0.w[wi] and int(w1[wi * n + e]) == k1.w[wi]
        b0 = F.gate_round1(kind, bw, S, int(out["xh"][e]), k0)
        b1 = F.gate_round1(kind, bw, S, int(out["xh"][e]), k1)
        words = (n + 31) // 32
        for p, bb in ((0, b0), (1, b1)):
            if kind != F.GATE_LRS:
                assert (int(out["bits"][p, "hi"][e // 32]) >> (e % 32)) & 1 == bb & 1
            if kind in F.SPLIT_KINDS:
                assert (int(out["bits"][p, "hi"][words + e // 32]) >> (e % 32)) & 1 == (bb >> 2) & 1
            if kind in F.SPLIT3_KINDS:
                assert (int(out["bits"][p, "hi"][2 * words + e // 32]) >> (e % 32)) & 1 == (bb >> 3) & 1
                assert (int(out["bits"][p, "hi"][3 * words + e // 32]) >> (e % 32)) & 1 == (bb >> 4) & 1
            if kind != F.GATE_RELU:
                assert (int(out["bits"][p, "lo"][e // 32]) >> (e % 32)) & 1 == (bb >> 1) & 1
        o = b0 ^ b1
        assert int(out["y0"][e]) == F.gate_round2(kind, bw, S, 0, int(out["xh"][e]), o, k0)
        assert int(out["y1"][e]) == F.gate_round2(kind, bw, S, 1, int(out["xh"][e]), o, k1)
    y = (out["y0"] + out["y1"] - out["rout"]).astype(dt)
    assert np.array_equal(y, plain(kind, x, bw))


@pytest.mark.gpu
@pytest.mark.parametrize("bw", [32, 64])
@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("n", [1, 33, 1 << 20])
def test_gate_reconstruction_sizes(ddg, cuda, bw, kind, n):
    x, r = make_inputs(bw, kind, n, seed=n + kind)
    out = run_gate(ddg, kind, bw, n, x, r, seed=99, op=7)
    y = (out["y0"] + out["y1"] - out["rout"]).astype(ring_dt(bw))
    assert np.array_equal(y, plain(kind, x, bw))


@pytest.mark.gpu
def test_gate_empty_is_noop(ddg, cuda):
    for kind in KINDS:
        ddg.gate_round1(kind, 32, S, 0, None, None, None, None)
        ddg.gate_round2(kind, 32, S, 0, 0, None, None, None, None, None, None, None)


@pytest.mark.gpu
@pytest.mark.parametrize("bw", [32, 64])
def test_aes_engines_agree(ddg, cuda, bw):
    """The two AES engines (two staged round tables + rotation, four staged
    tables) give identical keys, round-1 bits and shares, and identical hash
    chains in the throughput probe."""
    import torch

    kind, n = F.GATE_RELU_ARS_SPLIT, 5000
    x, r = make_inputs(bw, kind, n, seed=bw + 1)
    outs = []
    try:
        for nt in (2, 4):
            ddg.aes_tables(nt)
            outs.append(run_gate(ddg, kind, bw, n, x, r, seed=77, op=9))
            chain = torch.zeros(4096, dtype=torch.int32, device="cuda")
            ddg.check(ddg.lib().ddg_aes_chain_variant(4096, 16, nt, chain.data_ptr(), None))
            torch.cuda.synchronize()
            outs[-1]["chain"] = chain.cpu().numpy()
    finally:
        ddg.aes_tables(4)
    a, b = outs
    for k in ("k0", "k1", "rout", "y0", "y1", "chain"):
        assert np.array_equal(a[k], b[k]), k
    for kk in a["bits"]:
        assert np.array_equal(a["bits"][kk], b["bits"][kk])
