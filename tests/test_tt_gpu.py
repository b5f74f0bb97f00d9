"""Truth-table comparison gates (GATE_RELU_TT, GATE_RELU_ARS_TT, GATE_LRS_TT) against the C oracle.

Same bar as the other gate tests (the reference's primitive tests,
gpu_mpc/lss/lss_test.cpp:330-389: bit-exact on random and boundary inputs,
both parties, openings in the test): every party's key bytes (digit table
rows, triple words, dealer words), its masked comparison bits after the AND
tree and its round-2 share equal oracle/fss_ref.c's element by element; the
reconstructed outputs equal the plaintext function; and the opened bits equal
those of the DCF gate of the same dealer seed.
"""
import numpy as np
import pytest

from oracle import fss_ref as F
from oracle.ring_forward import Ring
from tests.gpu_util import dev_bytes, from_dev, ptr, ring_dt, to_dev
from tests.test_gates_gpu import make_inputs, plain

S = 12
TT_KINDS = [F.GATE_RELU_TT, F.GATE_RELU_ARS_TT, F.GATE_LRS_TT, F.GATE_RELU_TTF, F.GATE_RELU_ARS_TTF]
FULL_KINDS = (F.GATE_RELU_TTF, F.GATE_RELU_ARS_TTF)


def run_tt(ddg, kind, bw, n, x, r, seed=5, op=3, s=S):
    dt = ring_dt(bw)
    kb = ddg.gate_key_bytes(kind, bw, s, n)
    k0, k1 = dev_bytes(kb), dev_bytes(kb)
    d_r, d_ro = to_dev(r), dev_bytes(n * (bw // 8))
    ddg.gate_keygen(kind, bw, s, n, seed, op, ptr(d_r), ptr(d_ro), ptr(k0), ptr(k1))
    xh = (x + r).astype(dt)
    d_x = to_dev(xh)
    words = (n + 31) // 32
    nb = ddg.gate_round1_arrays(kind, bw, s)
    bits = [dev_bytes(4 * nb * words) for _ in range(2)]
    shares = [dev_bytes(n * (bw // 8)) for _ in range(2)]
    ddg.gate_eval_pair(kind, bw, s, n, ptr(d_x), ptr(k0), ptr(k1), ptr(bits[0]), ptr(bits[1]), ptr(shares[0]),
                       ptr(shares[1]))
    import torch

    torch.cuda.synchronize()
    return dict(k0=k0.cpu().numpy(), k1=k1.cpu().numpy(), rout=from_dev(d_ro, dt, n),
                bits=[from_dev(b, np.uint32, nb * words) for b in bits], y0=from_dev(shares[0], dt, n),
                y1=from_dev(shares[1], dt, n), xh=xh)


def bit(arr, word0, e):
    return (int(arr[word0 + e // 32]) >> (e % 32)) & 1


@pytest.mark.gpu
@pytest.mark.parametrize("bw", [32, 64])
@pytest.mark.parametrize("kind", TT_KINDS)
def test_tt_keys_bits_shares_match_oracle(ddg, cuda, bw, kind):
    n = 300
    wk = F.TT_WORD_KIND[kind]
    x, r = make_inputs(bw, wk, n, seed=kind * 10 + bw)
    out = run_tt(ddg, kind, bw, n, x, r)
    lay = ddg.tt_key_layout(kind, bw, S, n)
    dt = ring_dt(bw)
    words = (n + 31) // 32
    rows = [out["k0"][lay["tables"]:lay["tables"] + 4 * lay["rows"] * n].view(np.uint32),
            out["k1"][lay["tables"]:lay["tables"] + 4 * lay["rows"] * n].view(np.uint32)]
    tri = [out["k0"][lay["tri"]:lay["tri"] + 4 * lay["tri_words"] * n].view(np.uint32),
           out["k1"][lay["tri"]:lay["tri"] + 4 * lay["tri_words"] * n].view(np.uint32)]
    w = [out["k0"][lay["words"]:].view(dt), out["k1"][lay["words"]:].view(dt)]
    carry = kind == F.GATE_LRS_TT
    full = kind in FULL_KINDS
    for e in range(n):
        k0, k1, ry = F.tt_keygen(kind, bw, S, 5, 3, e, int(r[e]))
        assert int(out["rout"][e]) == ry
        for p, ref in ((0, k0), (1, k1)):
            for j in range(lay["rows"]):
                assert int(rows[p][j * n + e]) == ref.tab[j], (p, j)
            for j in range(lay["tri_words"]):
                assert int(tri[p][j * n + e]) == ref.tri[j], (p, j)
            for wi in range(F.GATE_NWORDS[kind]):
                assert int(w[p][wi * n + e]) == ref.w[wi]
        b0, b1 = F.tt_eval_pair(kind, bw, S, int(out["xh"][e]), k0, k1)
        for p, bb in ((0, b0), (1, b1)):
            if carry:
                assert bit(out["bits"][p], 0, e) == (bb >> 1) & 1
            elif full:  # [full compare | lo compare]
                assert bit(out["bits"][p], 0, e) == bb & 1
                assert bit(out["bits"][p], words, e) == (bb >> 1) & 1
            else:
                assert bit(out["bits"][p], 0, e) == bb & 1
                assert bit(out["bits"][p], words, e) == (bb >> 2) & 1
                assert bit(out["bits"][p], 2 * words, e) == (bb >> 1) & 1
        o = b0 ^ b1
        assert int(out["y0"][e]) == F.tt_round2(kind, bw, S, 0, int(out["xh"][e]), o, k0)
        assert int(out["y1"][e]) == F.tt_round2(kind, bw, S, 1, int(out["xh"][e]), o, k1)
        g0, g1, _ = F.gate_keygen(wk, bw, S, 5, 3, e, int(r[e]))
        d = F.gate_round1(wk, bw, S, int(out["xh"][e]), g0) ^ F.gate_round1(wk, bw, S, int(out["xh"][e]), g1)
        m = {F.GATE_LRS: 2, F.GATE_RELU: 1, F.GATE_RELU_ARS: 3}.get(wk, 7)
        assert o & m == d & m
    y = (out["y0"] + out["y1"] - out["rout"]).astype(dt)
    assert np.array_equal(y, plain(wk, x, bw))


@pytest.mark.gpu
@pytest.mark.parametrize("bw", [32, 64])
@pytest.mark.parametrize("kind", TT_KINDS)
@pytest.mark.parametrize("n", [1, 33, 1 << 20])
def test_tt_reconstruction_sizes(ddg, cuda, bw, kind, n):
    wk = F.TT_WORD_KIND[kind]
    x, r = make_inputs(bw, wk, n, seed=n + kind)
    out = run_tt(ddg, kind, bw, n, x, r, seed=99, op=7)
    y = (out["y0"] + out["y1"] - out["rout"]).astype(ring_dt(bw))
    assert np.array_equal(y, plain(wk, x, bw))


@pytest.mark.gpu
def test_tt_empty_is_noop(ddg, cuda):
    for kind in TT_KINDS:
        ddg.gate_eval_pair(kind, 32, S, 0, None, None, None, None, None, None, None)


@pytest.mark.gpu
@pytest.mark.parametrize("kind", [F.GATE_RELU_TTF, F.GATE_RELU_TT])
def test_tt_relu_with_a_digit_state_wider_than_32_bits(ddg, cuda, kind):
    """bw=64 at scale 13 has 17 digits (a 34-bit digit state): the runtime-plan
    level kernel runs and the triple bits keep 5 per AND, since the grouped
    layout needs the state in 32 bits.  Every key's triple words equal the
    oracle's and the reconstructed ReLU equals the plaintext one."""
    bw, sc, n = 64, 13, 3000
    dt = ring_dt(bw)
    rng = np.random.default_rng(13 + kind)
    x = rng.integers(0, np.iinfo(dt).max, size=n, dtype=dt, endpoint=True)
    r = rng.integers(0, np.iinfo(dt).max, size=n, dtype=dt, endpoint=True)
    out = run_tt(ddg, kind, bw, n, x, r, s=sc)
    lay = ddg.tt_key_layout(kind, bw, sc, n)
    tri = [out[k][lay["tri"]:lay["tri"] + 4 * lay["tri_words"] * n].view(np.uint32) for k in ("k0", "k1")]
    for e in range(0, n, 97):
        k0, k1, _ = F.tt_keygen(kind, bw, sc, 5, 3, e, int(r[e]))
        for p, ref in ((0, k0), (1, k1)):
            for j in range(lay["tri_words"]):
                assert int(tri[p][j * n + e]) == ref.tri[j], (p, j, e)
    y = (out["y0"] + out["y1"] - out["rout"]).astype(dt)
    assert np.array_equal(y, Ring(bw).relu(x))
