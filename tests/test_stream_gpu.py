"""Key chunks and the double-buffered key stream (dealer -> sealed chunks ->
pinned host ring / key file -> HBM slots), plus the failure paths the
reference handles with asserts (deepdtagen_inference.cu:387-390, 644): a
corrupted or truncated chunk, a key file that is too short, a peer that never
arrives."""
import os

import numpy as np
import pytest

from oracle import ring_forward as RF
from tests.gpu_util import ptr, to_dev

S = 12


def setup(ddg, synth, bw, B, nchunks):
    q = synth.quantize_weights(synth.affinity_weights(5), S)
    blob = synth.weights_blob(q)
    chunks = ddg.dealer_chunks(bw, S, B, [100 + i for i in range(nchunks)], blob, 0)
    p0, p1 = ddg.Party(0, bw, S, 0), ddg.Party(1, bw, S, 0)
    for p in (p0, p1):
        p.set_weights(blob)
    ddg.pair_local(p0, p1)
    inp = synth.Inputs(B, bw, seed=17, with_protein_cnn=False)
    keep, ins = [], []
    for p in (0, 1):
        arrs = [to_dev(np.asarray(a[p])) for a in (inp.x_sh, inp.adj_sh, inp.mask_sh, inp.protein_sh)]
        keep += arrs
        ins.append([ptr(a) for a in arrs])
    _, want = RF.protocol_forward(inp.x_ring, inp.adj_ring, inp.mask_ring, inp.protein_ring, q, bw, S)
    return chunks, p0, p1, ins, keep, want


@pytest.mark.gpu
@pytest.mark.parametrize("bw", [32, 64])
def test_stream_from_pinned_host_ring(ddg, synth, cuda, bw):
    B = 2
    chunks, p0, p1, ins, keep, want = setup(ddg, synth, bw, B, 3)
    ks0, ks1 = ddg.KeyStream(p0, B), ddg.KeyStream(p1, B)
    for c0, c1 in chunks:
        ks0.add_host_chunk(c0.data_ptr())
        ks1.add_host_chunk(c1.data_ptr())
    ks0.set_verify(True)
    ks1.set_verify(True)
    for step in range(5):  # chunks 0,1,2,0,1: every chunk's masks differ, the output must not
        raw, aff = ddg.forward_pair_streamed(ks0, ks1, ins[0], ins[1])
        assert np.array_equal(aff, want), step
    st = ks0.stats()
    assert st["chunks"] == 5 and st["bytes"] >= 5 * ddg.forward_key_bytes(bw, S, B)


@pytest.mark.gpu
def test_stream_from_key_file(ddg, synth, cuda, tmp_path):
    bw, B = 32, 2
    chunks, p0, p1, ins, keep, want = setup(ddg, synth, bw, B, 2)
    paths = []
    for p in (0, 1):
        path = str(tmp_path / f"DeepDTAGen_{bw}_{S}_party{p}_inference_key{p}.dat")
        ddg.write_key_file(path, [c[p] for c in chunks])
        paths.append(path)
    ks0, ks1 = ddg.KeyStream(p0, B), ddg.KeyStream(p1, B)
    ks0.open_file(paths[0], 2)
    ks1.open_file(paths[1], 2)
    for step in range(3):
        raw, aff = ddg.forward_pair_streamed(ks0, ks1, ins[0], ins[1])
        assert np.array_equal(aff, want), step
    assert ks0.stats()["read_ms"] > 0


@pytest.mark.gpu
def test_corrupted_and_truncated_chunks_are_rejected(ddg, synth, cuda, tmp_path):
    import torch

    bw, B = 32, 1
    q = synth.quantize_weights(synth.affinity_weights(5), S)
    chunks = ddg.dealer_chunks(bw, S, B, [7], synth.weights_blob(q), 0)
    d = chunks[0][0].to("cuda")
    assert ddg.key_chunk_verify(d.data_ptr(), bw, S, B) == 0
    d[12345] ^= 1
    with pytest.raises(ddg.DdgError) as e:
        ddg.key_chunk_verify(d.data_ptr(), bw, S, B)
    assert e.value.code == 3 and "checksum" in str(e.value)
    with pytest.raises(ddg.DdgError):  # wrong batch for this chunk
        ddg.key_chunk_verify(d.data_ptr(), bw, S, 2) if d.numel() >= ddg.key_chunk_bytes(bw, S, 2) else \
            ddg.check(3)
    p = ddg.Party(0, bw, S, 0)
    ks = ddg.KeyStream(p, B)
    path = str(tmp_path / "short.dat")
    with open(path, "wb") as f:
        f.write(chunks[0][0].numpy().tobytes()[:-4096])
    with pytest.raises(ddg.DdgError) as e:
        ks.open_file(path, 1)
    assert e.value.code == 3
    torch.cuda.synchronize()


@pytest.mark.gpu
def test_peer_that_never_arrives_times_out(ddg, synth, cuda):
    """Party 1 never runs: party 0's first opening gives up with DDG_ERR_PEER
    after the channel timeout instead of hanging."""
    import time

    bw, B = 32, 1
    q = synth.quantize_weights(synth.affinity_weights(5), S)
    blob = synth.weights_blob(q)
    kb = ddg.forward_key_bytes(bw, S, B)
    import torch

    k0 = torch.zeros(kb, dtype=torch.uint8, device="cuda")
    p0, p1 = ddg.Party(0, bw, S, 0), ddg.Party(1, bw, S, 0)
    p0.set_weights(blob)
    p0.bind_keys(k0.data_ptr(), kb)
    ddg.pair_local(p0, p1)
    p0.set_timeout(300)
    inp = synth.Inputs(B, bw, seed=1, with_protein_cnn=False)
    arrs = [to_dev(np.asarray(a[0])) for a in (inp.x_sh, inp.adj_sh, inp.mask_sh, inp.protein_sh)]
    t0 = time.time()
    with pytest.raises(ddg.DdgError) as e:
        p0.forward(B, *[ptr(a) for a in arrs])
    assert e.value.code == 4 and time.time() - t0 < 30
