"""The CPU oracle, pinned against the reference's golden vectors (no GPU)."""
import os

import numpy as np
import pytest

from oracle import fss_ref as F
from oracle import ring_forward as RF

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = os.path.join(HERE, "golden", "ff_golden.npz")


def test_aes_fips197_kat():
    # FIPS-197 appendix C.1; the same vector pins the reference's AES (gpu_mpc/lss/lss_test.cpp:52-70)
    ct = F.aes128(bytes(range(16)), bytes.fromhex("00112233445566778899aabbccddeeff"))
    assert ct.hex() == "69c4e0d86a7b0430d8cdb78070b4c55a"


@pytest.mark.parametrize("d", [5, 7, 8, 12, 31, 63])
def test_dcf_compares(d):
    rng = np.random.default_rng(d)
    for _ in range(25):
        alpha = int(rng.integers(0, 1 << d, dtype=np.uint64)) if d < 64 else 0
        k = F.dcf_keygen(d, alpha, rng.bytes(16), rng.bytes(16))
        xs = [int(v) for v in rng.integers(0, 1 << d, size=6, dtype=np.uint64)]
        xs += [alpha, max(alpha - 1, 0), min(alpha + 1, (1 << d) - 1), 0, (1 << d) - 1]
        for x in xs:
            c = F.dcf_eval(d, x, k[0], k[2], k[3]) ^ F.dcf_eval(d, x, k[1], k[2], k[3])
            assert c == int(x < alpha)


@pytest.mark.parametrize("d", [1, 5, 6, 7, 12, 19, 51])
def test_dcfeq_compares_and_equals(d):
    rng = np.random.default_rng(d + 100)
    for _ in range(25):
        alpha = int(rng.integers(0, 1 << d, dtype=np.uint64))
        k = F.dcfeq_keygen(d, alpha, rng.bytes(16), rng.bytes(16))
        xs = [int(v) for v in rng.integers(0, 1 << d, size=6, dtype=np.uint64)]
        xs += [alpha, max(alpha - 1, 0), min(alpha + 1, (1 << d) - 1), alpha ^ 1, alpha ^ 64, 0, (1 << d) - 1]
        for x in (v & ((1 << d) - 1) for v in xs):
            b = F.dcfeq_eval(d, x, k[0], k[2], k[3]) ^ F.dcfeq_eval(d, x, k[1], k[2], k[3])
            assert b & 1 == int(x < alpha) and (b >> 1) & 1 == int(x == alpha)


@pytest.mark.parametrize("bw", [32, 64])
@pytest.mark.parametrize("kind", [0, 1, 2, 3, 4, 5, 6, 7, 8])
def test_gate_functionality(bw, kind):
    M = (1 << bw) - 1
    rng = np.random.default_rng(bw + kind)
    R = RF.Ring(bw)
    for i in range(200):
        x = int(rng.integers(0, M, dtype=np.uint64, endpoint=True)) & M
        r = int(rng.integers(0, M, dtype=np.uint64, endpoint=True)) & M
        if i % 4 == 1:  # x_hat agrees with r on the upper bits: exercises the equality branch
            x = ((r & ~((1 << 12) - 1)) + int(rng.integers(0, 1 << 12)) - r) & M
        if i % 4 == 2:
            x = [0, 1, M, 1 << (bw - 1), (1 << (bw - 1)) - 1, (1 << 12) - 1, M - 4095][i % 7]
        if i % 4 == 3:  # x_hat agrees with r on carry bits 5..11: the split LRS equality branch
            x = ((r & ~31) + int(rng.integers(0, 32)) - r + (int(rng.integers(0, 1 << 20)) << 12)) & M
        if i % 8 == 5:  # x_hat agrees with r on bits 18..30 (three-part split: U1 equal, U2/V decide)
            x = ((r & ~((1 << 18) - 1)) + int(rng.integers(0, 1 << 18)) - r) & M
            x ^= int(rng.integers(0, 2)) << (bw - 1)
        if kind in (3, 6):
            x &= M >> 1
        k0, k1, ry = F.gate_keygen(kind, bw, 12, 3, 1, i, r)
        y = (F.gate_eval_pair(kind, bw, 12, (x + r) & M, k0, k1) - ry) & M
        xa = np.array([x], dtype=np.uint64)
        lrs = R.red(R.signed(xa) >> 12)
        want = [R.relu(xa), R.relu_ars(xa, 12), R.ars(xa, 12), lrs, R.relu(xa), R.relu_ars(xa, 12), lrs,
                R.relu(xa), R.relu_ars(xa, 12)][kind]
        assert y == int(want[0])


@pytest.mark.parametrize("bw", [32, 64])
def test_lut(bw):
    T = F.invsqrt_table(12, 138)
    assert np.array_equal(T, RF.invsqrt_table(12, 138))
    assert T[0] == 0 and T[1] == 4096 and T[4] == 2048 and T[139] == 0
    rng = np.random.default_rng(bw)
    M = (1 << bw) - 1
    for i, deg in enumerate([0, 1, 2, 137, 138] + [int(v) for v in rng.integers(0, 139, size=10)]):
        r = int(rng.integers(0, M, dtype=np.uint64, endpoint=True)) & M
        ro = int(rng.integers(0, M, dtype=np.uint64, endpoint=True)) & M
        k0, k1 = F.lut_keygen(bw, 5, 9, i, r & 255, ro)
        xh = (deg + r) & M
        v = (F.lut_eval(bw, 0, xh, T, k0) + F.lut_eval(bw, 1, xh, T, k1) - ro) & M
        assert v == int(T[deg])


def _golden(bw, synth):
    g = np.load(GOLD)
    seed = int(g[f"bw{bw}_seed"])
    return (g[f"bw{bw}_X"], g[f"bw{bw}_A_raw"].astype(np.float32), g[f"bw{bw}_mask"].astype(np.float32),
            g[f"bw{bw}_pvec"], synth.affinity_weights(seed), g[f"bw{bw}_pmvo"], g[f"bw{bw}_out"])


@pytest.mark.parametrize("bw", [32, 64])
def test_ff_restatement_bit_exact_vs_reference_golden(bw, synth):
    X, A, m, pv, layers, pmvo, out = _golden(bw, synth)
    Ah = synth.normalized_adjacency(A)
    for b in range(X.shape[0]):
        p, o, _ = RF.ff_forward(X[b], Ah[b], m[b], pv[b], layers, 12, bw)
        assert np.array_equal(p, pmvo[b])
        assert int(o[0]) == int(out[b])


# measured gap |protocol_forward - fixed_forward| on the 16 golden samples per
# ring (affinity units): bw 32 max 0.0076, mean 0.0030; bw 64 max 0.0132, mean
# 0.0044.  Pinned just above, so that a change of either function shows.
BRIDGE = {32: (0.0080, 0.0032), 64: (0.0135, 0.0046)}


@pytest.mark.parametrize("bw", [32, 64])
def test_protocol_forward_bridge_to_reference_fixed_forward(bw, synth):
    """The 2PC graph computes a different integer function from fixed_forward.py
    (aggregate-first truncation, LUT-derived A_hat, mask-multiply pool); the
    reference itself gates their agreement at 0.005 affinity units
    (scripts/dev_tools/validate_batch_fixed.py:33), on trained weights.  On
    these random-weight models (N(0,1) * 0.1 init, larger pre-activations than
    trained ones) the gap is pinned at its measured maximum and mean over 16
    samples per ring (BRIDGE)."""
    X, A, m, pv, layers, pmvo, out = _golden(bw, synth)
    B = X.shape[0]
    assert B >= 16
    q = synth.quantize_weights(layers, 12)
    xr, ar = synth.to_ring(X, 12, bw), synth.to_ring(A, 0, bw)
    mr = synth.to_ring(np.broadcast_to(m[:, :, None], (B, 138, 376)), 12, bw)
    pr = synth.to_ring(pv, 12, bw)
    _, aff = RF.protocol_forward(xr, ar, mr, pr, q, bw, 12)
    d = np.abs(aff - out / 4096.0)
    top, mean = BRIDGE[bw]
    assert d.max() <= top and d.mean() <= mean, d


def test_weight_blob_roundtrip(synth, tmp_path):
    q = synth.quantize_weights(synth.affinity_weights(3), 12)
    man = synth.write_weights(str(tmp_path / "weights.bin"), q)
    assert man["total_elements"] == sum(W.size + b.size for W, b in q)
    back = synth.read_weights(str(tmp_path / "weights.bin"))
    for (W, b), (W2, b2) in zip(q, back):
        assert np.array_equal(W, W2) and np.array_equal(b, b2)


def test_shares_reconstruct(synth):
    inp = synth.Inputs(2, 32, seed=4, with_protein_cnn=False)
    for name in ("x", "adj", "mask"):
        s0, s1 = getattr(inp, name + "_sh")
        assert np.array_equal((s0 + s1).astype(np.uint32), getattr(inp, name + "_ring"))


@pytest.mark.parametrize("bw", [32, 64])
def test_tt_and_ot_gates_match_plaintext_and_dcf_bits(bw):
    """The AND-tree gates of the C oracle reconstruct the plaintext function
    and open the same masked comparison bits as the DCF split gate of the same
    dealer seed (random inputs plus the equality branches of the split)."""
    import numpy as np

    R = RF.Ring(bw)
    M = (1 << bw) - 1
    rng = np.random.default_rng(bw)
    for kind in F.TT_KINDS + F.OT_KINDS:
        tt = kind in F.TT_KINDS
        wk = (F.TT_WORD_KIND if tt else F.OT_WORD_KIND)[kind]
        for i in range(60):
            r = int(rng.integers(0, 1 << 62)) * 4 + int(rng.integers(0, 4)) & M
            x = int(rng.integers(0, 1 << 62)) * 4 & M
            if i % 3 == 1:
                x = ((r & ~((1 << 12) - 1)) | int(rng.integers(0, 1 << 12))) - r & M
            if i % 3 == 2:
                x = ((r & ~63) | int(rng.integers(0, 64))) - r & M
            if wk == F.GATE_LRS:
                x &= M >> 1
            xh = (x + r) & M
            if tt:
                k0, k1, ro = F.tt_keygen(kind, bw, 12, 9, 4, i, r)
                y = F.tt_gate_pair(kind, bw, 12, xh, k0, k1)
                b0, b1 = F.tt_eval_pair(kind, bw, 12, xh, k0, k1)
            else:
                k0, k1, ro = F.ot_keygen(kind, bw, 12, 9, 4, i, r)
                y = F.ot_gate_pair(kind, bw, 12, xh, i, k0, k1)
                b0, b1, _, _ = F.ot_eval_pair(kind, bw, 12, xh, i, k0, k1)
            want = {F.GATE_RELU_SPLIT: R.relu(x), F.GATE_RELU_ARS_SPLIT: R.relu_ars(x, 12), F.GATE_RELU: R.relu(x),
                    F.GATE_RELU_ARS: R.relu_ars(x, 12), F.GATE_LRS: R.red(R.signed(x) >> 12)}[wk]
            assert (y - ro) & M == int(want)
            g0, g1, _ = F.gate_keygen(wk, bw, 12, 9, 4, i, r)
            d = F.gate_round1(wk, bw, 12, xh, g0) ^ F.gate_round1(wk, bw, 12, xh, g1)
            # the bits each word kind's round 2 reads: LRS the carry, RELU the full compare,
            # RELU_ARS full compare and carry, the SPLIT kinds hi compare, carry and hi equality
            m = {F.GATE_LRS: 2, F.GATE_RELU: 1, F.GATE_RELU_ARS: 3}.get(wk, 7)
            assert (b0 ^ b1) & m == d & m
