"""Openings over NCCL and over CUDA IPC (host handoffs, and device-side handoffs with peer stores)
between two processes on two GPUs (skipped with fewer GPUs)."""
import os
import subprocess
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.gpu
@pytest.mark.parametrize("comm", ["nccl", "ipc", "ipc-push"])
@pytest.mark.parametrize("bw", ["32", "64"])
def test_pair_forward_bit_exact(cuda, bw, comm):
    if cuda.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    env = dict(os.environ, DDG_CHECK_BW=bw, DDG_CHECK_COMM=comm, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
                        "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", "29531",
                        os.path.join(REPO, "tests", "pair_check.py")], env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert f"{comm} pair OK" in r.stdout


@pytest.mark.gpu
@pytest.mark.parametrize("comm", ["ipc", "ipc-push"])
def test_two_lanes_per_rank_bit_exact(cuda, comm):
    """Two parties per process (lanes), each paired with the other rank's lane
    over its own channel, forwards run concurrently from two host threads: the
    device-side waits of one lane never wait on a launch that the peer's host
    has still to make, so a context-wide synchronisation taken by the other
    lane (a first launch, an allocation) drains."""
    if cuda.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    env = dict(os.environ, DDG_CHECK_BW="32", DDG_CHECK_COMM=comm, DDG_CHECK_LANES="2", NCCL_NVLS_ENABLE="0")
    r = subprocess.run(["timeout", "-k", "30", "400", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
                        "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", "29532",
                        os.path.join(REPO, "tests", "pair_check.py")], env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert f"{comm} pair x2 lanes OK" in r.stdout


@pytest.mark.gpu
@pytest.mark.parametrize("comm", ["ipc", "ipc-push"])
def test_single_party_graph_replays_bit_exact(cuda, comm):
    """Each rank captures its own party's forward over a push-mode channel and
    replays it three times, then runs one host-launched forward: every output
    matches the oracle (the device-side generation base keeps graph replays
    and host launches in step).  Then rank 0 replays once more while rank 1
    stays on the host: its bounded device-side waits give up and the replay
    reports DDG_ERR_PEER.  A host-handoff channel refuses the capture."""
    if cuda.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    env = dict(os.environ, DDG_CHECK_BW="32", DDG_CHECK_COMM=comm, DDG_CHECK_GRAPH="1", DDG_CHECK_ABSENT="1",
               NCCL_NVLS_ENABLE="0")
    r = subprocess.run(["timeout", "-k", "30", "400", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
                        "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", "29533",
                        os.path.join(REPO, "tests", "pair_check.py")], env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    if comm == "ipc-push":
        assert "ipc-push pair graph absent peer detected in" in r.stdout and " OK" in r.stdout, r.stdout[-2000:]
    else:
        assert "ipc pair graph refused OK" in r.stdout
