"""The forward driven layer by layer through the per-layer C ABI.

The reference's graph calls its backend one layer or op at a time over a
caller-held key cursor and the backend's GpuPeer: ddgSecureAdjNorm{Keygen,Eval}
(gpu_mpc/secure_adj_norm.h:204-213, 394-405), GCNLayer::forward
(gcn_layer.h:99-103), MaskedMaxPoolLayer::_forward (masked_maxpool_layer.h:
23-47), and mul / relu / FC / output of Backend<T> (ddg_orca_base.h:170-323).
Here the dealer writes both parties' keys call by call, and the two parties
(two host threads) evaluate call by call with the same cursor discipline:
  * the dealer's keys equal ddg_dealer_forward's byte for byte;
  * the revealed outputs equal the fused forward's (ddg_forward_eval_pair) and
    the plaintext integer forward's (oracle protocol_forward) bit for bit,
    over the in-process zero-copy channel and over a transport the caller
    supplies (ddg_comm: stream sync, device->host copy, a host queue to the
    peer, host->device copy, as the reference's GpuPeer does over TCP);
  * the fused forward runs over the caller's transport too.
"""
import ctypes
import os
import queue
import threading

import numpy as np
import pytest

from oracle import ring_forward as RF
from tests.gpu_util import dev_bytes, ptr, to_dev

S = 12
NMAX, FEAT, POOL, PROT = 138, 94, 376, 128
LAYER_IN = [94, 188, 282, 376, 1024, 256, 1024, 512, 256]
LAYER_OUT = [188, 282, 376, 1024, 128, 1024, 512, 256, 1]


def _cudart():
    import nvidia.cuda_runtime as cr

    L = ctypes.CDLL(os.path.join(list(cr.__path__)[0], "lib", "libcudart.so.12"))
    L.cudaMemcpy.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int]
    L.cudaStreamSynchronize.argtypes = [ctypes.c_void_p]
    return L


def host_transport(party, queues, cudart):
    """The caller's transport of one party: its share goes device -> host ->
    the peer's queue, the peer's share host -> device."""

    def exchange(p, d_send, d_recv, nbytes, stream):
        assert p == party
        if cudart.cudaStreamSynchronize(stream) != 0:
            return 1
        buf = ctypes.create_string_buffer(nbytes)
        if cudart.cudaMemcpy(buf, d_send, nbytes, 2) != 0:  # device to host
            return 1
        queues[1 - party].put(buf.raw)
        peer = queues[party].get(timeout=120)
        if len(peer) != nbytes:
            return 1
        return cudart.cudaMemcpy(d_recv, peer, nbytes, 1)  # host to device

    return exchange


class Bufs:
    """device buffers of wires, kept alive for the test"""

    def __init__(self, es):
        self.es, self.keep = es, []

    def _buf(self, n):
        import torch

        t = dev_bytes(n * self.es)
        torch.cuda.synchronize()  # torch zero-fills on its own stream; the library writes on the party's
        self.keep.append(t)
        return t

    def wire(self, ddg, n):
        return ddg.Wire(ptr(self._buf(n)), n, None)

    def mask_wire(self, ddg, n):
        return ddg.MaskWire(ptr(self._buf(n)), n, None, None)


def layered_keygen(ddg, bw, B, seed, blob, k0, k1, kb, masks=None, ops=False):
    """The dealer, layer by layer, in the order of the fused forward.  masks
    (dict, optional) receives the dealer's mask of every named wire."""
    L = ddg.lib()
    d = ddg.Dealer(bw, S, 0, seed, blob)
    d.bind_keys(ptr(k0), ptr(k1), kb)
    c = ddg.Cursor()
    bufs = Bufs(bw // 8)
    if masks is not None:
        masks["_bufs"] = bufs
    mw = lambda n: bufs.mask_wire(ddg, n)  # noqa: E731
    chk = ddg.check
    try:
        Ah = mw(B * NMAX * NMAX)
        chk(L.ddg_adjnorm_keygen(d.h, c, B, Ah))
        H = mw(B * NMAX * FEAT)
        chk(L.ddg_op_input_keygen(d.h, c, H.n, H))
        for l in range(3):
            Hn = mw(B * NMAX * LAYER_OUT[l])
            if ops:  # GCNLayer::forward from Backend<T> ops: matmul 3-arg, truncation, FC + ReLU
                Pm, AX = mw(B * NMAX * LAYER_IN[l]), mw(B * NMAX * LAYER_IN[l])
                chk(L.ddg_op_matmul_keygen(d.h, c, B, LAYER_IN[l], Ah, H, Pm))
                chk(L.ddg_op_gate_keygen(d.h, c, ddg.GATE_LRS_TT, Pm, AX))
                chk(L.ddg_op_fc_keygen(d.h, c, l, B * NMAX, ddg.ACT_RELU, AX, Hn))
            else:
                chk(L.ddg_gcn_layer_keygen(d.h, c, l, B, Ah, H, Hn))
            H = Hn
            if masks is not None:
                masks[f"gcn{l}.H"] = H
        M = mw(B * NMAX * POOL)
        chk(L.ddg_op_input_keygen(d.h, c, M.n, M))
        Pm = mw(B * NMAX * POOL)
        chk(L.ddg_op_mul_keygen(d.h, c, 0, 0, 0, H, M, 1, Pm))
        pooled = mw(B * POOL)
        chk(L.ddg_maxpool_keygen(d.h, c, B, Pm, pooled))
        d1 = mw(B * 1024)
        chk(L.ddg_op_fc_keygen(d.h, c, 3, B, ddg.ACT_RELU, pooled, d1))
        d2 = mw(B * PROT)
        chk(L.ddg_op_fc_keygen(d.h, c, 4, B, ddg.ACT_TRUNC, d1, d2))
        f = mw(B * 256)
        chk(L.ddg_op_concat_protein_keygen(d.h, c, B, d2, f))
        f_cat = f
        for l in (5, 6, 7):
            fn = mw(B * LAYER_OUT[l])
            chk(L.ddg_op_fc_keygen(d.h, c, l, B, ddg.ACT_RELU, f, fn))
            f = fn
        o = mw(B)
        chk(L.ddg_op_fc_keygen(d.h, c, 8, B, ddg.ACT_NONE, f, o))
        chk(L.ddg_op_output_keygen(d.h, c, o))
        if masks is not None:
            masks.update({"A_hat": Ah, "gcn2.H": H, "masked": Pm, "pooled": pooled, "d1": d1, "d2": d2,
                          "fused": f_cat, "f3": f, "out2s": o})
        return c.offset
    finally:
        d.close()


def layered_eval(ddg, party, bw, B, shares, out, ops=False):
    """One evaluator, layer by layer; shares = device (x, adj, mask, protein)."""
    L = ddg.lib()
    c = ddg.Cursor()
    bufs = Bufs(bw // 8)
    w = lambda n: bufs.wire(ddg, n)  # noqa: E731
    chk = ddg.check
    h = party.h
    out["_bufs"] = bufs
    Ah = w(B * NMAX * NMAX)
    chk(L.ddg_adjnorm_eval(h, c, B, ptr(shares[1]), Ah))
    H = w(B * NMAX * FEAT)
    chk(L.ddg_op_input_eval(h, c, H.n, ptr(shares[0]), H))
    for l in range(3):
        Hn = w(B * NMAX * LAYER_OUT[l])
        if ops:
            Pm, AX = w(B * NMAX * LAYER_IN[l]), w(B * NMAX * LAYER_IN[l])
            chk(L.ddg_op_matmul_eval(h, c, B, LAYER_IN[l], Ah, H, Pm))
            chk(L.ddg_op_gate_eval(h, c, ddg.GATE_LRS_TT, Pm, AX))
            chk(L.ddg_op_fc_eval(h, c, l, B * NMAX, ddg.ACT_RELU, AX, Hn))
        else:
            chk(L.ddg_gcn_layer_eval(h, c, l, B, Ah, H, Hn))
        H = Hn
        out[f"gcn{l}.H"] = H
    M = w(B * NMAX * POOL)
    chk(L.ddg_op_input_eval(h, c, M.n, ptr(shares[2]), M))
    Pm = w(B * NMAX * POOL)
    chk(L.ddg_op_mul_eval(h, c, 0, 0, 0, H, M, 1, Pm))
    pooled = w(B * POOL)
    chk(L.ddg_maxpool_eval(h, c, B, Pm, pooled))
    d1 = w(B * 1024)
    chk(L.ddg_op_fc_eval(h, c, 3, B, ddg.ACT_RELU, pooled, d1))
    d2 = w(B * PROT)
    chk(L.ddg_op_fc_eval(h, c, 4, B, ddg.ACT_TRUNC, d1, d2))
    f = w(B * 256)
    chk(L.ddg_op_concat_protein_eval(h, c, B, d2, ptr(shares[3]), f))
    f_cat = f
    for l in (5, 6, 7):
        fn = w(B * LAYER_OUT[l])
        chk(L.ddg_op_fc_eval(h, c, l, B, ddg.ACT_RELU, f, fn))
        f = fn
    o = w(B)
    chk(L.ddg_op_fc_eval(h, c, 8, B, ddg.ACT_NONE, f, o))
    raw = np.zeros(B, dtype=np.int64)
    aff = np.zeros(B, dtype=np.float64)
    chk(L.ddg_op_output_eval(h, c, B, o, raw.ctypes.data, aff.ctypes.data))
    out["raw"], out["aff"], out["offset"] = raw, aff, c.offset
    out.update({"A_hat": Ah, "masked": Pm, "pooled": pooled, "d1": d1, "d2": d2, "fused": f_cat, "f3": f,
                "out2s": o})


def wire_host(d_ptr, n, dt):
    """n ring elements at a device address, copied to the host"""
    import torch

    torch.cuda.synchronize()
    buf = np.empty(n, dtype=dt)
    cr = _cudart()
    assert cr.cudaMemcpy(buf.ctypes.data, d_ptr, buf.nbytes, 2) == 0
    return buf


def run_both(fn0, fn1):
    errs = [None, None]

    def run(i, fn):
        try:
            fn()
        except Exception as e:  # re-raised below
            errs[i] = e

    ts = [threading.Thread(target=run, args=(i, f)) for i, f in enumerate((fn0, fn1))]
    for t in ts:
        t.start()
    for t in ts:
        t.join(timeout=600)
    for e in errs:
        if e is not None:
            raise e


def setup(ddg, synth, bw, B, seed):
    q = synth.quantize_weights(synth.affinity_weights(5), S)
    blob = synth.weights_blob(q)
    inp = synth.Inputs(B, bw, seed=seed, with_protein_cnn=False)
    shares = [[to_dev(np.asarray(a[p])) for a in (inp.x_sh, inp.adj_sh, inp.mask_sh, inp.protein_sh)] for p in (0, 1)]
    return q, blob, inp, shares


def parties(ddg, bw, blob, keys, kb):
    ps = [ddg.Party(p, bw, S, 0) for p in (0, 1)]
    for p, k in zip(ps, keys):
        p.set_weights(blob)
        p.bind_keys(ptr(k), kb)
    return ps


@pytest.mark.gpu
@pytest.mark.parametrize("bw", [32, 64])
@pytest.mark.parametrize("gcn", ["layer", "ops"])
def test_layered_keygen_and_eval_match_fused_forward(ddg, synth, cuda, bw, gcn):
    import torch

    B = 3
    q, blob, inp, shares = setup(ddg, synth, bw, B, seed=61)
    kb = ddg.forward_key_bytes(bw, S, B)
    fused = [dev_bytes(kb) for _ in range(2)]
    ddg.dealer_forward(bw, S, B, 555, blob, 0, ptr(fused[0]), ptr(fused[1]))
    layered = [dev_bytes(kb) for _ in range(2)]
    masks = {}
    ops = gcn == "ops"
    end = layered_keygen(ddg, bw, B, 555, blob, layered[0], layered[1], kb, masks, ops=ops)
    torch.cuda.synchronize()
    assert 0 < end <= kb
    for p in (0, 1):
        assert torch.equal(layered[p], fused[p]), f"party {p}: layered dealer keys differ from ddg_dealer_forward's"

    trace = {}
    want_raw, want_aff = RF.protocol_forward(inp.x_ring, inp.adj_ring, inp.mask_ring, inp.protein_ring, q, bw, S,
                                             trace=trace)
    want_raw = RF.Ring(bw).signed(want_raw)
    ps = parties(ddg, bw, blob, layered, kb)
    ddg.pair_local(ps[0], ps[1])
    raw_f, aff_f = ddg.forward_pair(ps[0], ps[1], B, [ptr(t) for t in shares[0]], [ptr(t) for t in shares[1]])
    assert np.array_equal(raw_f, want_raw)
    outs = [{}, {}]
    run_both(lambda: layered_eval(ddg, ps[0], bw, B, shares[0], outs[0], ops=ops),
             lambda: layered_eval(ddg, ps[1], bw, B, shares[1], outs[1], ops=ops))
    # every intermediate wire, unmasked with the dealer's mask, is the oracle's value
    dt = np.uint32 if bw == 32 else np.uint64
    for name in ("A_hat", "gcn0.H", "gcn1.H", "gcn2.H", "masked", "pooled", "d1", "d2", "fused", "f3", "out2s"):
        n = masks[name].n
        mask = wire_host(masks[name].d_mask, n, dt)
        for p in (0, 1):
            val = wire_host(outs[p][name].d_value, n, dt)
            got = (val - mask).astype(dt)
            want = np.asarray(trace[name], dtype=np.uint64).astype(dt).reshape(-1)
            bad = np.flatnonzero(got != want)
            assert bad.size == 0, f"party {p}, wire {name}: {bad.size} of {n} values differ (first {bad[:5]})"
    for p in (0, 1):
        assert np.array_equal(outs[p]["raw"], raw_f) and np.array_equal(outs[p]["aff"], aff_f)
        assert outs[p]["offset"] == end  # the evaluators consumed exactly what the dealer wrote
    for p in ps:
        p.close()


@pytest.mark.gpu
def test_layered_and_fused_forward_over_caller_transport(ddg, synth, cuda):
    """Openings through a ddg_comm callback that moves every share through host
    memory and a queue to the peer (the reference's D2H -> TCP -> H2D)."""
    bw, B = 32, 2
    q, blob, inp, shares = setup(ddg, synth, bw, B, seed=62)
    kb = ddg.forward_key_bytes(bw, S, B)
    keys = [dev_bytes(kb) for _ in range(2)]
    ddg.dealer_forward(bw, S, B, 777, blob, 0, ptr(keys[0]), ptr(keys[1]))
    want_raw, want_aff = RF.protocol_forward(inp.x_ring, inp.adj_ring, inp.mask_ring, inp.protein_ring, q, bw, S)
    want_raw = RF.Ring(bw).signed(want_raw)
    cudart = _cudart()
    qs = [queue.Queue(), queue.Queue()]
    ps = parties(ddg, bw, blob, keys, kb)
    for i, p in enumerate(ps):
        p.connect_callback(host_transport(i, qs, cudart))
    outs = [{}, {}]
    run_both(lambda: layered_eval(ddg, ps[0], bw, B, shares[0], outs[0]),
             lambda: layered_eval(ddg, ps[1], bw, B, shares[1], outs[1]))
    for p in (0, 1):
        assert np.array_equal(outs[p]["raw"], want_raw) and np.array_equal(outs[p]["aff"], want_aff)
    # the fused forward over the same transport
    res = [None, None]

    def fused(i):
        res[i] = ps[i].forward(B, *[ptr(t) for t in shares[i]])

    run_both(lambda: fused(0), lambda: fused(1))
    assert np.array_equal(res[0][0], want_raw) and np.array_equal(res[0][1], want_aff)
    st = ps[0].stats()
    assert st["rounds"] > 50 and st["bytes_sent"] > 0
    for p in ps:
        p.close()


@pytest.mark.gpu
def test_layered_gate_per_op_and_cursor_errors(ddg, cuda):
    """Backend<T>::relu one op at a time with the default truth-table kind (the
    per-op round 1 of ddg_gate_round1 refuses the interactive kinds): both
    parties' ddg_op_gate_eval reveal ReLU(x) + r_out for the dealer's
    ddg_op_gate_keygen keys; a cursor past the bound key region is refused."""
    import torch

    bw, n = 32, 5000
    synth_w = np.zeros(sum(i * o + o for i, o in zip(LAYER_IN, LAYER_OUT)), dtype=np.int64)
    L = ddg.lib()
    kind = ddg.GATE_RELU_TTF
    kb = ddg.gate_key_bytes(kind, bw, S, n) + 4096
    keys = [dev_bytes(kb) for _ in range(2)]
    d = ddg.Dealer(bw, S, 0, 99, synth_w)
    d.bind_keys(ptr(keys[0]), ptr(keys[1]), kb)
    rng = np.random.default_rng(3)
    x = rng.integers(0, 2**32, size=n, dtype=np.uint64).astype(np.uint32)
    r = rng.integers(0, 2**32, size=n, dtype=np.uint64).astype(np.uint32)
    d_r, d_ro = to_dev(r), dev_bytes(4 * n)
    xin = ddg.MaskWire(ptr(d_r), n, None, None)
    xout = ddg.MaskWire(ptr(d_ro), 0, None, None)
    c = ddg.Cursor()
    ddg.check(L.ddg_op_gate_keygen(d.h, c, kind, xin, xout))
    assert xout.n == n and c.ops > 0
    d.close()
    ps = parties(ddg, bw, synth_w, keys, kb)
    ddg.pair_local(ps[0], ps[1])
    d_x = to_dev((x + r).astype(np.uint32))
    ys = [dev_bytes(4 * n) for _ in range(2)]
    curs = [ddg.Cursor(), ddg.Cursor()]

    def one(p):
        ddg.check(L.ddg_op_gate_eval(ps[p].h, curs[p], kind, ddg.Wire(ptr(d_x), n, None), ddg.Wire(ptr(ys[p]), 0, None)))

    run_both(lambda: one(0), lambda: one(1))
    torch.cuda.synchronize()
    y = ys[0].cpu().numpy().view(np.uint32)
    assert np.array_equal(y, ys[1].cpu().numpy().view(np.uint32))  # both parties reveal the same y_hat
    ro = d_ro.cpu().numpy().view(np.uint32)
    want = np.maximum(x.view(np.int32).astype(np.int64), 0).astype(np.uint32)
    assert np.array_equal((y - ro).astype(np.uint32), want)
    assert curs[0].offset == curs[1].offset == c.offset
    # the next call would read beyond the bound region: refused, cursor unchanged
    far = ddg.Cursor(kb - 256, 0, 0)
    with pytest.raises(ddg.DdgError) as e:
        one_far = L.ddg_op_gate_eval(ps[0].h, far, kind, ddg.Wire(ptr(d_x), n, None), ddg.Wire(ptr(ys[0]), 0, None))
        ddg.check(one_far)
    assert e.value.code == 3 and far.offset == kb - 256
    for p in ps:
        p.close()
