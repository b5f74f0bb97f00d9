"""OT-leaf ReLU gates (GATE_RELU_OT, GATE_RELU_ARS_OT) against the C oracle, through the C ABI.

Mirrors the reference's LSS primitive tests (gpu_mpc/lss/lss_test.cpp:330-389:
ReLU / compare / MSB bit-exact on random and boundary inputs, both parties,
openings in the test): every party's key bytes (AES round keys, receiver
records, triple c bits, words), its masked comparison bits after the AND tree
and its round-2 share are compared with oracle/fss_ref.c element by element;
the reconstructed outputs with the plaintext function; and the opened bits
with those of the DCF gate (GATE_RELU*_SPLIT) that the same dealer seed
defines, which the OT protocol must reproduce.
"""
import numpy as np
import pytest

from oracle import fss_ref as F
from tests.gpu_util import dev_bytes, from_dev, ptr, ring_dt, to_dev
from tests.test_gates_gpu import make_inputs, plain

S = 12
OT_KINDS = [F.GATE_RELU_OT, F.GATE_RELU_ARS_OT]


def plain_ot(kind, x, bw):
    return plain(F.OT_WORD_KIND[kind], x, bw)


def run_ot(ddg, kind, bw, n, x, r, seed=5, op=3):
    dt = ring_dt(bw)
    kb = ddg.gate_key_bytes(kind, bw, S, n)
    k0, k1 = dev_bytes(kb), dev_bytes(kb)
    d_r, d_ro = to_dev(r), dev_bytes(n * (bw // 8))
    ddg.gate_keygen(kind, bw, S, n, seed, op, ptr(d_r), ptr(d_ro), ptr(k0), ptr(k1))
    xh = (x + r).astype(dt)
    d_x = to_dev(xh)
    words = (n + 31) // 32
    nb = ddg.gate_round1_arrays(kind, bw, S)
    bits = [dev_bytes(4 * nb * words) for _ in range(2)]
    shares = [dev_bytes(n * (bw // 8)) for _ in range(2)]
    ddg.gate_eval_pair(kind, bw, S, n, ptr(d_x), ptr(k0), ptr(k1), ptr(bits[0]), ptr(bits[1]), ptr(shares[0]),
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
@pytest.mark.parametrize("kind", OT_KINDS)
def test_ot_keys_bits_shares_match_oracle(ddg, cuda, bw, kind):
    n = 300
    x, r = make_inputs(bw, F.OT_WORD_KIND[kind], n, seed=kind * 10 + bw)
    out = run_ot(ddg, kind, bw, n, x, r)
    lay = ddg.ot_key_layout(kind, bw, S, n)
    dt = ring_dt(bw)
    nwords = F.GATE_NWORDS[kind]
    words = (n + 31) // 32
    w = [out["k0"][lay["words"]:].view(dt), out["k1"][lay["words"]:].view(dt)]
    c0 = [out["k0"][lay["c0"]:lay["c0"] + 4 * n].view(np.uint32), out["k1"][lay["c0"]:lay["c0"] + 4 * n].view(np.uint32)]
    for e in range(n):
        k0, k1, ry = F.ot_keygen(kind, bw, S, 5, 3, e, int(r[e]))
        assert int(out["rout"][e]) == ry
        for p, (blob, ref) in enumerate(((out["k0"], k0), (out["k1"], k1))):
            if e == 0:
                assert blob[lay["ks"]:lay["ks"] + 176].tobytes() == bytes(ref.ks)
            for t in range(lay["slots"]):
                assert int(blob[lay["recv"] + t * n + e]) == ref.recv[t], (p, t)
            assert int(c0[p][e]) == ref.c0
            for wi in range(nwords):
                assert int(w[p][wi * n + e]) == ref.w[wi]
        b0, b1, _, _ = F.ot_eval_pair(kind, bw, S, int(out["xh"][e]), e, k0, k1)
        for p, bb in ((0, b0), (1, b1)):
            assert bit(out["bits"][p], 0, e) == bb & 1
            assert bit(out["bits"][p], words, e) == (bb >> 2) & 1
            assert bit(out["bits"][p], 2 * words, e) == (bb >> 1) & 1
        o = b0 ^ b1
        assert int(out["y0"][e]) == F.ot_round2(kind, bw, S, 0, int(out["xh"][e]), o, k0)
        assert int(out["y1"][e]) == F.ot_round2(kind, bw, S, 1, int(out["xh"][e]), o, k1)
        # the opened bits are those of the DCF split gate of the same dealer seed
        wk = F.OT_WORD_KIND[kind]
        g0, g1, _ = F.gate_keygen(wk, bw, S, 5, 3, e, int(r[e]))
        assert o == (F.gate_round1(wk, bw, S, int(out["xh"][e]), g0) ^ F.gate_round1(wk, bw, S, int(out["xh"][e]), g1))
    y = (out["y0"] + out["y1"] - out["rout"]).astype(dt)
    assert np.array_equal(y, plain_ot(kind, x, bw))


@pytest.mark.gpu
@pytest.mark.parametrize("bw", [32, 64])
@pytest.mark.parametrize("kind", OT_KINDS)
@pytest.mark.parametrize("n", [1, 33, 1 << 20])
def test_ot_reconstruction_sizes(ddg, cuda, bw, kind, n):
    x, r = make_inputs(bw, F.OT_WORD_KIND[kind], n, seed=n + kind)
    out = run_ot(ddg, kind, bw, n, x, r, seed=99, op=7)
    y = (out["y0"] + out["y1"] - out["rout"]).astype(ring_dt(bw))
    assert np.array_equal(y, plain_ot(kind, x, bw))


@pytest.mark.gpu
def test_ot_empty_is_noop(ddg, cuda):
    for kind in OT_KINDS:
        ddg.gate_eval_pair(kind, 32, S, 0, None, None, None, None, None, None, None)
