"""End-to-end online forward (dealer + two parties on one GPU) against the oracle.

The reference's integration gate (tests/test_mpc_online_gate.py:91-151) runs
dealer + 2 evaluators and compares the revealed AFFINITY[i] with a plaintext
model; here the two parties run as two host threads on cuda:0 with the GPU
dealer's keys, and the revealed 2s->s outputs must equal
oracle.ring_forward.protocol_forward bit for bit.
"""
import numpy as np
import pytest

from oracle import ring_forward as RF
from tests.gpu_util import dev_bytes, ptr, to_dev

S = 12


def setup_pair(ddg, synth, bw, B, seed=123, wseed=5):
    q = synth.quantize_weights(synth.affinity_weights(wseed), S)
    blob = synth.weights_blob(q)
    kb = ddg.forward_key_bytes(bw, S, B)
    k0, k1 = dev_bytes(kb), dev_bytes(kb)
    ddg.dealer_forward(bw, S, B, seed, blob, 0, ptr(k0), ptr(k1))
    p0, p1 = ddg.Party(0, bw, S, 0), ddg.Party(1, bw, S, 0)
    for p, k in ((p0, k0), (p1, k1)):
        p.set_weights(blob)
        p.bind_keys(ptr(k), kb)
    ddg.pair_local(p0, p1)
    return q, p0, p1, (k0, k1)


def dev_inputs(inp):
    keep = []
    ins = []
    for p in (0, 1):
        arrs = [to_dev(np.asarray(inp.x_sh[p])), to_dev(np.asarray(inp.adj_sh[p])), to_dev(np.asarray(inp.mask_sh[p])),
                to_dev(np.asarray(inp.protein_sh[p]))]
        keep += arrs
        ins.append([ptr(a) for a in arrs])
    return ins, keep


def expected(inp, q, bw):
    return RF.protocol_forward(inp.x_ring, inp.adj_ring, inp.mask_ring, inp.protein_ring, q, bw, S)


@pytest.mark.gpu
@pytest.mark.parametrize("bw", [32, 64])
def test_forward_bit_exact(ddg, synth, cuda, bw):
    B = 3
    inp = synth.Inputs(B, bw, seed=21, with_protein_cnn=False)
    q, p0, p1, keep_k = setup_pair(ddg, synth, bw, B)
    ins, keep = dev_inputs(inp)
    raw, aff = ddg.forward_pair(p0, p1, B, ins[0], ins[1])
    want_raw, want_aff = expected(inp, q, bw)
    assert np.array_equal(raw, RF.Ring(bw).signed(want_raw)), (raw, want_raw)
    assert np.array_equal(aff, want_aff)
    st = p0.stats()
    assert st["rounds"] > 50 and st["key_bytes_used"] <= ddg.forward_key_bytes(bw, S, B)


@pytest.mark.gpu
@pytest.mark.parametrize("bw", [32, 64])
@pytest.mark.parametrize("mode", ["split2", "split3", "ot"])
def test_forward_bit_exact_other_relu_forms(ddg, synth, cuda, bw, mode):
    """The other comparison backends give the same revealed outputs as the
    default truth-table backend: DCF keys (two- and three-part splits,
    one-shot round 1) and the OT-leaf gates (garbled digit tables), each with
    its own key layout."""
    B = 3
    try:
        if mode == "ot":
            ddg.relu_backend(ddg.RELU_OT)
        else:
            ddg.relu_backend(ddg.RELU_DCF)
            ddg.relu_split(2 if mode == "split2" else 3)
        inp = synth.Inputs(B, bw, seed=22, with_protein_cnn=False)
        q, p0, p1, keep_k = setup_pair(ddg, synth, bw, B, seed=321)
        ins, keep = dev_inputs(inp)
        for _ in range(2):
            raw, aff = ddg.forward_pair(p0, p1, B, ins[0], ins[1])
            want_raw, want_aff = expected(inp, q, bw)
            assert np.array_equal(raw, RF.Ring(bw).signed(want_raw)), (raw, want_raw)
            assert np.array_equal(aff, want_aff)
        st = p0.stats()
        assert st["key_bytes_used"] <= ddg.forward_key_bytes(bw, S, B)
    finally:
        ddg.relu_backend(ddg.RELU_TT)
        ddg.relu_split(3)


@pytest.mark.gpu
def test_forward_host_inputs_and_repeat(ddg, synth, cuda):
    """Host (pinned or pageable) share buffers; keys re-used for a second forward
    (timing-only key reuse, as the reference's benchmark loop rewinds keyBuf)."""
    bw, B = 32, 4
    inp = synth.Inputs(B, bw, seed=5, with_protein_cnn=False)
    q, p0, p1, keep_k = setup_pair(ddg, synth, bw, B, seed=9)
    host = []
    for p in (0, 1):
        arrs = [np.ascontiguousarray(inp.x_sh[p]), np.ascontiguousarray(inp.adj_sh[p]),
                np.ascontiguousarray(inp.mask_sh[p]), np.ascontiguousarray(inp.protein_sh[p])]
        host.append(arrs)
    want_raw, want_aff = expected(inp, q, bw)
    for _ in range(2):
        raw, aff = ddg.forward_pair(p0, p1, B, [a.ctypes.data for a in host[0]], [a.ctypes.data for a in host[1]],
                                    on_host=True)
        assert np.array_equal(aff, want_aff)


@pytest.mark.gpu
def test_forward_comparison_timing(ddg, synth, cuda):
    """Comparison-kernel timing of an in-process pair: launch events are read
    back after the forwards, counted once per launch, and the pair union lies
    between the larger party union and their sum."""
    bw, B = 32, 3
    inp = synth.Inputs(B, bw, seed=21, with_protein_cnn=False)
    q, p0, p1, keep_k = setup_pair(ddg, synth, bw, B)
    ins, keep = dev_inputs(inp)
    want_raw, want_aff = expected(inp, q, bw)
    ddg.forward_pair(p0, p1, B, ins[0], ins[1])  # untimed
    counts = []
    for nfwd in (1, 3):
        for p in (p0, p1):
            p.enable_dcf_timing(True)
        for _ in range(nfwd):
            raw, aff = ddg.forward_pair(p0, p1, B, ins[0], ins[1])
            assert np.array_equal(aff, want_aff)
        ddg.parties_dcf_union([p0, p1])
        t = [p0.dcf_timing(), p1.dcf_timing()]
        counts.append(t[0]["launches"])
        assert t[0]["launches"] == t[1]["launches"] > 0
        assert t[0]["bytes"] > 0 and t[0]["sum_ms"] > 0
        for x in t:
            assert 0 < x["union_ms"] <= x["sum_ms"] + 1e-6
        assert max(t[0]["union_ms"], t[1]["union_ms"]) - 1e-6 <= t[0]["pair_union_ms"]
        assert t[0]["pair_union_ms"] <= t[0]["union_ms"] + t[1]["union_ms"] + 1e-6
        # a second read-back adds nothing
        assert p0.dcf_timing()["launches"] == t[0]["launches"]
        for p in (p0, p1):
            p.enable_dcf_timing(False)
    assert counts[1] == 3 * counts[0]


@pytest.mark.gpu
@pytest.mark.parametrize("bw", [32, 64])
def test_forward_cuda_graph_replays_bit_exact(ddg, synth, cuda, bw):
    """The pair forward captured into a CUDA graph and replayed twice gives the
    ordinary forward's outputs bit for bit; each replay counts its kernels, and
    the comparison-kernel timing sees the launches of one replay."""
    B = 3
    inp = synth.Inputs(B, bw, seed=31, with_protein_cnn=False)
    q, p0, p1, keep_k = setup_pair(ddg, synth, bw, B, seed=77)
    ins, keep = dev_inputs(inp)
    raw0, aff0 = ddg.forward_pair(p0, p1, B, ins[0], ins[1])
    want_raw, want_aff = expected(inp, q, bw)
    assert np.array_equal(raw0, RF.Ring(bw).signed(want_raw))
    n_plain = ddg.launch_count()
    ddg.forward_pair(p0, p1, B, ins[0], ins[1])
    n_plain = ddg.launch_count() - n_plain
    for p in (p0, p1):
        p.enable_dcf_timing(True)
    g = ddg.ForwardGraph(p0, p1, B, ins[0], ins[1])
    try:
        for _ in range(2):
            n = ddg.launch_count()
            raw, aff = g.launch()
            assert ddg.launch_count() - n == n_plain
            assert np.array_equal(raw, raw0) and np.array_equal(aff, aff0)
        ddg.parties_dcf_union([p0, p1])
        t = [p0.dcf_timing(), p1.dcf_timing()]
        assert t[0]["launches"] == t[1]["launches"] > 0
        assert 0 < t[0]["pair_union_ms"] <= t[0]["union_ms"] + t[1]["union_ms"] + 1e-6
    finally:
        g.close()
        for p in (p0, p1):
            p.enable_dcf_timing(False)
    # the parties still run ordinary forwards afterwards
    raw2, aff2 = ddg.forward_pair(p0, p1, B, ins[0], ins[1])
    assert np.array_equal(raw2, raw0)


@pytest.mark.gpu
def test_forward_edge_graphs(ddg, synth, cuda):
    """kiba-shaped graphs (up to 100 atoms), a 138-atom graph, and an all-zero
    padding sample (degree 0 -> table[0] = 0; deepdtagen_inference.cu:72-79)."""
    bw, B = 64, 3
    inp = synth.Inputs(B, bw, seed=8, atoms=(10, 100), with_protein_cnn=False)
    rng = np.random.default_rng(1)
    X, A, m = synth.gen_graph(rng, 138, 138)
    inp.X_float[1], inp.A_raw[1], inp.mask[1] = X, A, m
    inp.X_float[2] = 0
    inp.A_raw[2] = 0
    inp.mask[2] = 0
    mask_tiled = np.broadcast_to(inp.mask[:, :, None], (B, 138, 376))
    inp.x_ring = synth.to_ring(inp.X_float, S, bw)
    inp.adj_ring = synth.to_ring(inp.A_raw, 0, bw)
    inp.mask_ring = synth.to_ring(mask_tiled, S, bw)
    inp.x_sh = synth.split_shares(inp.x_ring, 1, bw)
    inp.adj_sh = synth.split_shares(inp.adj_ring, 2, bw)
    inp.mask_sh = synth.split_shares(inp.mask_ring, 3, bw)
    q, p0, p1, keep_k = setup_pair(ddg, synth, bw, B, seed=77)
    ins, keep = dev_inputs(inp)
    raw, aff = ddg.forward_pair(p0, p1, B, ins[0], ins[1])
    want_raw, want_aff = expected(inp, q, bw)
    assert np.array_equal(aff, want_aff)


@pytest.mark.gpu
def test_forward_rejects_short_key_region(ddg, synth, cuda):
    bw, B = 32, 2
    inp = synth.Inputs(B, bw, seed=3, with_protein_cnn=False)
    q, p0, p1, keep_k = setup_pair(ddg, synth, bw, B)
    p0.bind_keys(ptr(keep_k[0]), 1024)
    ins, keep = dev_inputs(inp)
    with pytest.raises(ddg.DdgError) as e:
        ddg.forward_pair(p0, p1, B, ins[0], ins[1])
    assert e.value.code == 3


def _cfg_inputs(synth, bw, B, atoms, seed):
    return synth.Inputs(B, bw, seed=seed, atoms=atoms, with_protein_cnn=False)


@pytest.mark.gpu
@pytest.mark.parametrize("bw,B,atoms", [(32, 16, (10, 60)), (32, 256, (10, 60)), (64, 256, (10, 100))],
                         ids=["pr1-bw32-B16", "bench-bw32-B256", "kiba-bw64-B256"])
def test_forward_bit_exact_at_benched_configs(ddg, synth, cuda, bw, B, atoms):
    """The forward at the sizes it is run and benchmarked at: the PR1 reference
    case (bw=32, B=16, davis-shaped graphs), the bench workload (bw=32, B=256:
    one party's key region is beyond 2^32 bytes and the largest gate covers
    11 M elements on a full grid) and the kiba-shaped bw=64 workload at B=256.
    Every revealed output equals protocol_forward bit for bit, on the host
    launches and, at B=256, on a replay of the CUDA-graph capture too."""
    inp = _cfg_inputs(synth, bw, B, atoms, seed=400 + B + bw)
    q, p0, p1, keep_k = setup_pair(ddg, synth, bw, B, seed=4000 + B + bw)
    kb = ddg.forward_key_bytes(bw, S, B)
    if B == 256:
        assert kb > 2**32, kb  # 64-bit key offsets are exercised
    ins, keep = dev_inputs(inp)
    raw, aff = ddg.forward_pair(p0, p1, B, ins[0], ins[1])
    want_raw, want_aff = expected(inp, q, bw)
    want_signed = RF.Ring(bw).signed(want_raw)
    bad = np.flatnonzero(raw != want_signed)
    assert bad.size == 0, f"{bad.size} of {B} samples differ, first {bad[:8]}"
    assert np.array_equal(aff, want_aff)
    assert p0.stats()["key_bytes_used"] <= kb
    if B == 256:
        g = ddg.ForwardGraph(p0, p1, B, ins[0], ins[1])
        try:
            graw, gaff = g.launch()
        finally:
            g.close()
        assert np.array_equal(graw, want_signed) and np.array_equal(gaff, want_aff)


@pytest.mark.gpu
def test_forward_graph_timing_readouts_follow_replays(ddg, synth, cuda):
    """Comparison-kernel timing with a CUDA graph: every read-out adds the
    launches of the replay that ran since the previous one (replay, read,
    replay, read), a host-launched forward in between adds its own launches
    with events of its own (the graph's events are not handed out again), and
    the replays keep giving the oracle's outputs."""
    bw, B = 32, 3
    inp = synth.Inputs(B, bw, seed=41, with_protein_cnn=False)
    q, p0, p1, keep_k = setup_pair(ddg, synth, bw, B, seed=78)
    ins, keep = dev_inputs(inp)
    want_raw, want_aff = expected(inp, q, bw)
    ddg.forward_pair(p0, p1, B, ins[0], ins[1])  # one-time set-up outside the capture
    for p in (p0, p1):
        p.enable_dcf_timing(True)
    g = ddg.ForwardGraph(p0, p1, B, ins[0], ins[1])
    try:
        seen = []

        def read():
            ddg.parties_dcf_union([p0, p1])
            t = [p0.dcf_timing(), p1.dcf_timing()]
            assert t[0]["launches"] == t[1]["launches"]
            seen.append(t[0])

        raw, aff = g.launch()
        assert np.array_equal(aff, want_aff)
        read()
        n1 = seen[0]["launches"]
        assert n1 > 0
        read()  # no replay since: nothing added
        assert seen[1]["launches"] == n1
        g.launch()
        read()
        assert seen[2]["launches"] == 2 * n1
        # the second replay ran after the first: its intervals extend the union
        assert seen[2]["union_ms"] > 1.5 * seen[0]["union_ms"]
        assert seen[2]["pair_union_ms"] > 1.5 * seen[0]["pair_union_ms"]
        raw, aff = ddg.forward_pair(p0, p1, B, ins[0], ins[1])  # host launches with pool events
        assert np.array_equal(aff, want_aff)
        read()
        assert seen[3]["launches"] == 3 * n1
        assert seen[3]["union_ms"] > seen[2]["union_ms"]
        raw, aff = g.launch()
        assert np.array_equal(raw, RF.Ring(bw).signed(want_raw)) and np.array_equal(aff, want_aff)
        read()
        assert seen[4]["launches"] == 4 * n1
        assert seen[4]["union_ms"] > seen[3]["union_ms"]
    finally:
        g.close()
        for p in (p0, p1):
            p.enable_dcf_timing(False)


@pytest.mark.gpu
def test_forward_graph_with_pinned_host_inputs(ddg, synth, cuda):
    """A graph captured with host inputs (ddg_forward_graph_create_ex, on_host):
    every replay copies the pinned input shares in and reveals the oracle's
    outputs; new values written into the same pinned buffers between replays
    are picked up (the copies are part of the replay)."""
    import torch

    bw, B = 32, 3
    q, p0, p1, keep_k = setup_pair(ddg, synth, bw, B, seed=91)
    inps = [synth.Inputs(B, bw, seed=sd, with_protein_cnn=False) for sd in (51, 52)]

    def pinned(inp):
        return [[torch.from_numpy(np.ascontiguousarray(a[p]).view(np.uint8).copy()).pin_memory()
                 for a in (inp.x_sh, inp.adj_sh, inp.mask_sh, inp.protein_sh)] for p in (0, 1)]

    bufs = pinned(inps[0])
    ptrs = [[t.data_ptr() for t in bufs[p]] for p in (0, 1)]
    raw, aff = ddg.forward_pair(p0, p1, B, ptrs[0], ptrs[1], on_host=True)  # one-time set-up
    g = ddg.ForwardGraph(p0, p1, B, ptrs[0], ptrs[1], on_host=True)
    try:
        for k, inp in enumerate(inps):
            if k:
                new = pinned(inp)
                for p in (0, 1):
                    for dst, src in zip(bufs[p], new[p]):
                        dst.copy_(src)
            want_raw, want_aff = expected(inp, q, bw)
            for _ in range(2):
                raw, aff = g.launch()
                assert np.array_equal(raw, RF.Ring(bw).signed(want_raw)) and np.array_equal(aff, want_aff)
    finally:
        g.close()


@pytest.mark.gpu
def test_forward_pipeline_on_pinned_host_inputs(ddg, synth, cuda):
    """Pipelined forwards (ddg_forward_pipeline_*): steps alternate between two
    pinned input sets, each step's copies overlap the previous step's forward,
    and every step reveals the oracle's outputs of its own inputs, delivered
    by a later submit (two steps in flight) or by wait()."""
    import torch

    bw, B = 32, 3
    q, p0, p1, keep_k = setup_pair(ddg, synth, bw, B, seed=93)
    inps = [synth.Inputs(B, bw, seed=sd, with_protein_cnn=False) for sd in (61, 62)]
    bufs = [[[torch.from_numpy(np.ascontiguousarray(a[p]).view(np.uint8).copy()).pin_memory()
              for a in (inp.x_sh, inp.adj_sh, inp.mask_sh, inp.protein_sh)] for p in (0, 1)] for inp in inps]
    ptrs = [[[t.data_ptr() for t in b[p]] for p in (0, 1)] for b in bufs]
    ddg.forward_pair(p0, p1, B, ptrs[0][0], ptrs[0][1], on_host=True)  # one-time set-up
    want = [expected(inp, q, bw) for inp in inps]
    pipe = ddg.ForwardPipeline(p0, p1, B)
    try:
        outs = []
        for k in range(5):
            outs.append((k % 2, pipe.submit(ptrs[k % 2][0], ptrs[k % 2][1])))
        pipe.wait()
        for which, (raw, aff) in outs:
            want_raw, want_aff = want[which]
            assert np.array_equal(raw, RF.Ring(bw).signed(want_raw)) and np.array_equal(aff, want_aff)
        # a second round after wait() starts from an idle pipeline
        raw, aff = pipe.submit(ptrs[1][0], ptrs[1][1])
        pipe.wait()
        assert np.array_equal(raw, RF.Ring(bw).signed(want[1][0])) and np.array_equal(aff, want[1][1])
    finally:
        pipe.close()


@pytest.mark.gpu
def test_forward_graph_enqueue_then_sync(ddg, synth, cuda):
    """Replays queued back to back (ddg_forward_graph_enqueue) and one sync:
    the last replay's output is the oracle's, and a launch after the sync
    still is."""
    bw, B = 32, 3
    inp = synth.Inputs(B, bw, seed=47, with_protein_cnn=False)
    q, p0, p1, keep_k = setup_pair(ddg, synth, bw, B, seed=79)
    ins, keep = dev_inputs(inp)
    want_raw, want_aff = expected(inp, q, bw)
    ddg.forward_pair(p0, p1, B, ins[0], ins[1])  # one-time set-up outside the capture
    g = ddg.ForwardGraph(p0, p1, B, ins[0], ins[1])
    try:
        for _ in range(4):
            g.enqueue()
        raw, aff = g.sync()
        assert np.array_equal(raw, RF.Ring(bw).signed(want_raw)) and np.array_equal(aff, want_aff)
        raw, aff = g.launch()
        assert np.array_equal(raw, RF.Ring(bw).signed(want_raw)) and np.array_equal(aff, want_aff)
    finally:
        g.close()
