"""Host-side logic of the multi-GPU path on CPU ranks (gloo, world size 2).

Covers what bench.py's torchrun path does outside the library: the party
layout (pair i = ranks (i, k+i)), broadcasting the per-pair NCCL unique ids,
the max-over-ranks reduction of the timed region, and failure detection: a
rank that dies before a collective makes the survivor's collective fail within
the process-group timeout instead of hanging (the reference has no failure
handling beyond asserts).
"""
import datetime
import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

import bench


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _init(rank, world, port, timeout_s=30):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))


def _put_and_exit(q, msg, code):
    """os._exit skips the queue's feeder thread: flush the message first."""
    q.put(msg)
    q.close()
    q.join_thread()
    os._exit(code)


def _worker_layout(rank, world, port, q):
    import torch

    try:
        _init(rank, world, port)
    except Exception as e:  # noqa: BLE001 -- reported, so the test retries on another port
        _put_and_exit(q, ("setup failed", rank, type(e).__name__), 1)
    pairs, pair, party, peer = bench.roles(rank, world)
    # one id per party pair (and lane), as bench.py broadcasts them
    uids = [[[os.urandom(128) for _ in range(1)] for _ in range(pairs)] if rank == 0 else None]
    dist.broadcast_object_list(uids, src=0)
    t = torch.tensor([10.0 + rank])
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    q.put((rank, pairs, pair, party, peer, uids[0][pair][0][:8], float(t.item())))
    dist.barrier()
    dist.destroy_process_group()


def test_roles_layout():
    assert bench.roles(0, 1) == (1, 0, None, None)
    for world in (2, 4, 8):
        seen = set()
        for r in range(world):
            pairs, pair, party, peer = bench.roles(r, world)
            assert pairs == world // 2 and bench.roles(peer, world)[3] == r
            assert bench.roles(peer, world)[1] == pair and bench.roles(peer, world)[2] == 1 - party
            seen.add((pair, party))
        assert len(seen) == world
    with pytest.raises(ValueError):
        bench.roles(0, 3)


def _spawn_world2(target, nmsg, tries=3):
    """Start the two ranks on a fresh port; a rank that cannot set up the
    process group (the port was taken meanwhile) reports it, and the pair is
    started again on another port.  Returns the ranks' messages."""
    ctx = mp.get_context("spawn")
    for attempt in range(tries):
        q = ctx.Queue()
        port = _free_port()
        ps = [ctx.Process(target=target, args=(r, 2, port, q)) for r in range(2)]
        for p in ps:
            p.start()
        got = [q.get(timeout=120) for _ in range(nmsg)]
        for p in ps:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
        failed = [m for m in got if isinstance(m, tuple) and m and m[0] == "setup failed"]
        if not failed or attempt == tries - 1:
            return got, ps
    return got, ps


def test_gloo_world2_layout_broadcast_and_max():
    got, ps = _spawn_world2(_worker_layout, 2)
    assert not any(m[0] == "setup failed" for m in got), got
    for p in ps:
        assert p.exitcode == 0
    got = sorted(got)
    (r0, pairs0, pair0, party0, peer0, u0, m0), (r1, pairs1, pair1, party1, peer1, u1, m1) = got
    assert (party0, party1) == (0, 1) and (peer0, peer1) == (1, 0) and pair0 == pair1 == 0
    assert u0 == u1 and m0 == m1 == 11.0


def _worker_dies(rank, world, port, q):
    try:
        _init(rank, world, port, timeout_s=5)
        dist.barrier()  # both ranks are connected before one of them dies
    except Exception as e:  # noqa: BLE001
        _put_and_exit(q, ("setup failed", rank, type(e).__name__), 1)
    if rank == 1:
        os._exit(3)  # the peer dies before the next collective
    try:
        dist.broadcast_object_list([None], src=1)
        msg = "no error"
    except Exception as e:  # noqa: BLE001 -- any collective failure is the expected outcome
        msg = "error: " + type(e).__name__
    _put_and_exit(q, msg, 0)


def test_dead_peer_is_detected_not_hung():
    got, ps = _spawn_world2(_worker_dies, 1)
    msg = got[0]
    assert isinstance(msg, str) and msg.startswith("error"), msg
