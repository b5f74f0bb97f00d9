"""The command-line drop-in ddg_inference against the oracle.

Mirrors the reference's integration gate (tests/test_mpc_online_gate.py:91-151:
dealer, then two evaluators, then AFFINITY[i] compared with a plaintext model)
on the reference's CLI (deepdtagen_inference <bw> <scale> <role> <party>
<keydir> <sampledir> <B> [peer_ip]): the dealer writes both parties' chunked
key files and meta.json, the evaluators stream the chunks and party 0 prints
AFFINITY[i]=%.6f, which must equal oracle.ring_forward.protocol_forward's
affinity for every sample, including a partial last chunk.
"""
import json
import os
import re
import subprocess

import numpy as np
import pytest

from oracle import ring_forward as RF

S = 12
HERE = os.path.dirname(os.path.abspath(__file__))
BIN = os.path.join(os.path.dirname(HERE), "idash26-track3_b200", "ddg_inference")


def run(args, env=None, timeout=600):
    e = dict(os.environ)
    e.update(env or {})
    return subprocess.run([BIN] + [str(a) for a in args], capture_output=True, text=True, env=e, timeout=timeout)


def affinities(stdout):
    got = {}
    for line in stdout.splitlines():
        m = re.match(r"AFFINITY\[(\d+)\]=(-?[0-9.]+)$", line)
        if m:
            got[int(m.group(1))] = m.group(2)
    return got


def dataset(synth, tmp_path, bw, N, seed):
    sampledir = tmp_path / "samples"
    inp = synth.Inputs(N, bw, seed=seed, with_protein_cnn=False)
    inp.write(str(sampledir))
    q = synth.quantize_weights(synth.affinity_weights(5), S)
    synth.write_weights(str(sampledir / "weights.bin"), q)
    _, aff = RF.protocol_forward(inp.x_ring, inp.adj_ring, inp.mask_ring, inp.protein_ring, q, bw, S)
    return sampledir, {i: f"{a:.6f}" for i, a in enumerate(aff)}


def test_usage_errors_exit_1():
    if not os.path.exists(BIN):
        pytest.skip("ddg_inference not built")
    r = run([])
    assert r.returncode == 1 and "usage" in r.stderr
    r = run([48, 12, 1, 0, "/tmp/k", "/tmp/s", 4])
    assert r.returncode == 1


@pytest.mark.gpu
@pytest.mark.parametrize("backend", ["tt", "ot", "dcf"])
@pytest.mark.parametrize("bw", [32, 64])
def test_dealer_then_both_parties_in_one_process(synth, cuda, tmp_path, bw, backend):
    N, B = 5, 2  # three chunks, the last one partial
    sampledir, want = dataset(synth, tmp_path, bw, N, seed=31 + bw)
    keydir = tmp_path / "keys"
    env = {"DDG_RELU_BACKEND": backend}
    r = run([bw, S, 0, 2, keydir, sampledir, B], env=env)
    assert r.returncode == 0, r.stderr
    meta = json.loads((keydir / "meta.json").read_text())
    assert (meta["B"], meta["NC"], meta["N"], meta["bw"], meta["relu_backend"]) == (B, 3, N, bw, backend)
    for p in (0, 1):
        assert (keydir / f"DeepDTAGen_{bw}_{S}_party{p}_inference_key{p}.dat").stat().st_size > 0
    r = run([bw, S, 1, 2, keydir, sampledir, B], env=env)
    assert r.returncode == 0, r.stderr
    assert affinities(r.stdout) == want
    # evaluators with another backend expect another key layout and refuse the file
    other = {"DDG_RELU_BACKEND": "dcf" if backend != "dcf" else "tt"}
    r = run([bw, S, 1, 2, keydir, sampledir, B], env=other)
    assert r.returncode == 2


@pytest.mark.gpu
def test_key_file_of_another_batch_size_is_refused(synth, cuda, tmp_path):
    sampledir, _ = dataset(synth, tmp_path, 32, 4, seed=3)
    keydir = tmp_path / "keys"
    assert run([32, S, 0, 2, keydir, sampledir, 2]).returncode == 0
    r = run([32, S, 1, 2, keydir, sampledir, 4])  # keys were made for B=2
    assert r.returncode == 2 and "key" in r.stderr.lower()


@pytest.mark.gpu
def test_two_processes_over_nccl(synth, cuda, tmp_path):
    """Party 1 and party 0 as separate processes on GPUs 0 and 1 (party 1
    starts first and listens, as in the reference's run order)."""
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs (NCCL cannot put both ranks on one GPU)")
    N, B = 3, 2
    sampledir, want = dataset(synth, tmp_path, 32, N, seed=7)
    keydir = tmp_path / "keys"
    assert run([32, S, 0, 2, keydir, sampledir, B]).returncode == 0
    port = str(29650 + os.getpid() % 500)
    env1 = {"DDG_DEVICE": "1", "DDG_PEER_PORT": port, "NCCL_NVLS_ENABLE": "0"}
    env0 = {"DDG_DEVICE": "0", "DDG_PEER_PORT": port, "NCCL_NVLS_ENABLE": "0"}
    e = dict(os.environ)
    e.update(env1)
    p1 = subprocess.Popen([BIN, "32", str(S), "1", "1", str(keydir), str(sampledir), str(B)], stdout=subprocess.PIPE,
                          stderr=subprocess.PIPE, text=True, env=e)
    try:
        r0 = run([32, S, 1, 0, keydir, sampledir, B, "127.0.0.1"], env=env0, timeout=300)
        out1, err1 = p1.communicate(timeout=300)
    finally:
        if p1.poll() is None:
            p1.kill()
    assert r0.returncode == 0, r0.stderr
    assert p1.returncode == 0, err1
    assert affinities(r0.stdout) == want
    assert affinities(out1) == {}  # only party 0 reveals
