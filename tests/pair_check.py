"""Two-rank check of the inter-process channels: party 0 on rank 0, party 1 on rank 1.

Launched with torchrun (see tests/test_multigpu_gpu.py).  Both ranks run the
GPU dealer with the same seed (so they hold matching keys), take their own
party's shares of the same seeded inputs, open every value over the channel
named by DDG_CHECK_COMM (nccl: ncclSend/ncclRecv; ipc: CUDA-IPC send slots
read in place; ipc-push: peer stores into the consumer's receive slots and
device-side flags), and rank 0 compares the revealed outputs of several forwards
with the integer oracle.  With DDG_CHECK_LANES=L > 1 every rank holds L
parties (lanes), each with its own keys, inputs and channel to the matching
lane of the other rank, and runs their forwards concurrently from L host
threads, as the split bench layout with --lanes does.  With DDG_CHECK_GRAPH=1
(ipc-push, one lane) every rank then captures its own party's forward into a
CUDA graph and replays it, a host-launched forward follows the replays, and
all of them are compared; over host-handoff IPC the capture must be refused.
With DDG_CHECK_ABSENT=1 as well, rank 0 then replays its graph once more with
a 2 s limit while rank 1 stays on the host (a flag that nothing sets): the
replay must end with DDG_ERR_PEER, and rank 0's context must stay usable.
Exits non-zero on any mismatch.
"""
import datetime
import importlib
import os
import sys
import uuid

import numpy as np
import torch
import torch.distributed as dist

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, REPO)


def absent_peer(ddg, P, B, ins, rank, dev):
    """Rank 0 replays its forward while rank 1 never runs its own: the first
    device-side wait for rank 1 gives up after 2 s, the rest give up at once."""
    import time

    dist.barrier()
    note = ""
    if rank == 0:
        P.set_timeout(2000)
        g = ddg.ForwardGraph(P, None, B, ins)
        t0 = time.time()
        try:
            g.launch()
            note = " absent peer NOT detected"
        except ddg.DdgError as e:
            note = " absent peer detected" if e.code == 4 else f" absent peer error {e}"  # DDG_ERR_PEER
        dt = time.time() - t0
        g.close()
        assert float(torch.ones(4, device=dev).sum().item()) == 4.0  # the context still works
        note += f" in {dt:.1f} s"
        if dt > 30:
            note += " (too slow: error)"
    dist.barrier()
    return note


def main():
    from oracle import ring_forward as RF

    ddg = importlib.import_module("idash26-track3_b200")
    synth = importlib.import_module("idash26-track3_b200.synth")
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    assert world == 2
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
    bw, B, s = int(os.environ.get("DDG_CHECK_BW", "32")), 3, 12
    comm = os.environ.get("DDG_CHECK_COMM", "nccl")
    lanes = int(os.environ.get("DDG_CHECK_LANES", "1"))
    q = synth.quantize_weights(synth.affinity_weights(5), s)
    blob = synth.weights_blob(q)
    kb = ddg.forward_key_bytes(bw, s, B)
    if comm in ("ipc", "ipc-push"):
        uid = [[f"ddg_check_{uuid.uuid4().hex[:16]}_{l}" for l in range(lanes)] if rank == 0 else None]
    else:
        uid = [[ddg.nccl_unique_id() for _ in range(lanes)] if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    parties, inps, keep = [], [], []
    for lane in range(lanes):
        k0 = torch.empty(kb, dtype=torch.uint8, device=dev)
        k1 = torch.empty(kb, dtype=torch.uint8, device=dev)
        ddg.dealer_forward(bw, s, B, 31 + lane, blob, local, k0.data_ptr(), k1.data_ptr())
        inp = synth.Inputs(B, bw, seed=44 + lane, with_protein_cnn=False)
        P = ddg.Party(rank, bw, s, local)
        P.set_weights(blob)
        P.bind_keys((k0 if rank == 0 else k1).data_ptr(), kb)
        P.set_timeout(120_000)
        if comm in ("ipc", "ipc-push"):
            P.connect_ipc(uid[0][lane], ddg.forward_max_exchange_bytes(bw, s, B), push=comm == "ipc-push")
        else:
            P.connect_nccl(uid[0][lane], 2, rank, 1 - rank)
        bufs = [torch.from_numpy(np.ascontiguousarray(a[rank]).view(np.uint8).copy()).to(dev)
                for a in (inp.x_sh, inp.adj_sh, inp.mask_sh, inp.protein_sh)]
        parties.append(P)
        inps.append(inp)
        keep.append((k0, k1, bufs))
    ins = [[b.data_ptr() for b in k[2]] for k in keep]
    # every forward reuses the IPC send slots many times over (dozens of
    # openings, four slots) and starts where the previous one left them; the
    # same keys and shares give the same outputs every time
    if lanes == 1:
        outs = [[parties[0].forward(B, *ins[0])[1]] for _ in range(3)]
    else:
        outs = [[o[1] for o in ddg.forward_lanes(parties, B, ins)] for _ in range(3)]
    graph_note = ""
    if os.environ.get("DDG_CHECK_GRAPH") == "1" and lanes == 1:
        if comm == "ipc-push":
            g = ddg.ForwardGraph(parties[0], None, B, ins[0])
            outs += [[g.launch()[1]] for _ in range(3)]
            g.close()
            outs.append([parties[0].forward(B, *ins[0])[1]])  # host-launched after the replays
            graph_note = " graph"
            if os.environ.get("DDG_CHECK_ABSENT") == "1":
                graph_note += absent_peer(ddg, parties[0], B, ins[0], rank, dev)
        else:
            try:
                ddg.ForwardGraph(parties[0], None, B, ins[0]).close()
                graph_note = " graph NOT refused"
            except ddg.DdgError as e:
                graph_note = " graph refused" if e.code == 5 else f" graph error {e}"  # DDG_ERR_STATE
    ok = 1
    if rank == 0:
        want = [RF.protocol_forward(i.x_ring, i.adj_ring, i.mask_ring, i.protein_ring, q, bw, s)[1] for i in inps]
        ok = int(all(np.array_equal(o[l], want[l]) for o in outs for l in range(lanes)))
        tag = f"{comm} pair" + (f" x{lanes} lanes" if lanes > 1 else "") + graph_note
        ok = ok and "NOT" not in graph_note and "error" not in graph_note
        print(tag, "OK" if ok else f"MISMATCH {outs} vs {want}", parties[0].stats(), flush=True)
    flag = torch.tensor([ok])
    dist.broadcast(flag, src=0)
    for P in parties:
        P.close()
    dist.destroy_process_group()
    sys.exit(0 if int(flag.item()) else 1)


if __name__ == "__main__":
    main()
