#!/usr/bin/env python
"""Online 2PC throughput of the DeepDTAGen affinity branch on B200.

Workload: the full affinity branch -- secure
adjacency normalisation, GCN x3, masked max-pool, FC head -- at bw=32,
scale 12, micro-batch B=256 of davis-shaped synthetic graphs, keys resident
in HBM.  A step is one online forward of B samples by both parties.

  N = 1      : both parties on cuda:0 (two host threads, zero-copy openings)
  N = 2,4,8  : torchrun, one process per GPU, every pair on its own
               micro-batch (weak scaling, no collective on the data path).
               --layout colocated (default): every GPU runs both parties of its
               own pair, as at N = 1.  --layout split: one party per process,
               ranks 0..k-1 party 0, ranks k..2k-1 party 1, pair i = (i, k+i)
               exchanging its openings over CUDA IPC (--comm ipc: send slots
               read in place over NVLink) or NCCL send/recv (--comm nccl).

value    : samples/s of the whole job, inputs (shares) and keys already in HBM.
e2e      : the same through the C ABI with host (pinned) share buffers: every
           step copies both parties' input shares host->device and the
           revealed affinities device->host.
roofline : the comparison kernels of the selected backend (default: the
           truth-table gates' ot_level_kernel), their algorithmic bytes (key
           bytes, inputs, state and openings) over the union of their launch
           intervals, measured with CUDA events on the party streams during
           the timed region, against the measured HBM copy bandwidth; plus
           e2e_key_frac, both parties' key bytes per step over the step time.
cpu_baseline / --impl reference : the reference's own CPU LSS ReLU backend
           (gpu_mpc/lss, compiled by oracle/Makefile into oracle/_ref) over
           loopback, plus the plaintext integer forward of the same graph.
parity   : (N = 1, with the CPU baseline) the revealed outputs of the
           warm-up forward, of the CUDA-graph replay and of the e2e forward
           against the plaintext integer forward of the same inputs, weights
           and graph, all B samples, bit for bit; the run fails on a mismatch.
"""
from __future__ import annotations

import argparse
import datetime
import importlib
import json
import os
import statistics
import subprocess
import sys
import time
import uuid

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)
_JSON_OUT = None


def stdout_for_json_only():
    """stdout carries exactly one JSON line.  Everything else that a library
    may write to file descriptor 1 (NCCL prints its version banner there) goes
    to stderr: fd 1 is pointed at stderr and the JSON line is written to a
    duplicate of the original stdout."""
    global _JSON_OUT
    _JSON_OUT = os.fdopen(os.dup(1), "w", buffering=1)
    os.dup2(2, 1)
    sys.stdout = sys.stderr


def emit(line: dict):
    out = _JSON_OUT or sys.stdout
    out.write(json.dumps(line) + "\n")
    out.flush()

NMAX, FEAT, POOL, PROT = 138, 94, 376, 128
RELUS_PER_SAMPLE = 171_076           # 138*(188+282+376) + 376*137 + 2816
A10_SAMPLES_PER_S = 16 / 0.136       # reference README.md:99-101, A10, B=16, bw=32

# DRAM bytes (read + write) per algorithmic byte of each backend's comparison
# kernel, from ncu captures (dram__bytes_read.sum + dram__bytes_write.sum over
# the kernel's algorithmic bytes):
#   tt : ot_level_kernel, all four levels of both parties of one full-compare
#        ReLU gate at 2^23 elements (microbench.py tt): 162.4 MB of DRAM
#        traffic for 183.0 MB of algorithmic bytes per launch on average (the
#        level-1 key reads reach DRAM once; part of the openings and state
#        written stays in L2 for the next level);
#   dcf: gate_round1_kernel, three-part ReLU(ARS) at B=16: 300.0 MB for 295.9 MB.
NCU_DRAM_BYTES_PER_ALG_BYTE = {"tt": 162.4 / 183.0, "dcf": 300.0 / 295.9, "ot": None}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--bw", type=int, default=32, choices=[32, 64])
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--scale", type=int, default=12)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--lanes", type=int, default=1,
                    help="N>1 with --comm ipc: batch lanes per rank, each its own party with its own IPC channel, "
                         "stream and host thread, so one lane computes while another waits for an opening.  "
                         "With --comm nccl only 1: two lanes (two communicators used concurrently from two threads "
                         "per GPU) stalled for 900 s on the first 2-GPU run, cause not established")
    ap.add_argument("--layout", default="colocated", choices=["colocated", "split"],
                    help="N>1: colocated = every GPU runs both parties of its own pair on its own micro-batch "
                         "(openings stay on the device; weak scaling with the per-GPU work of N=1); split = party 0 "
                         "on ranks 0..N/2-1, party 1 on the others, pair i = (i, N/2+i), openings over NVLink "
                         "(--comm)")
    ap.add_argument("--peer-timeout", type=int, default=120,
                    help="N>1: seconds a party waits for its peer at one opening before giving up")
    ap.add_argument("--comm", default="ipc-push", choices=["ipc-push", "ipc", "nccl"],
                    help="N>1, split layout: openings between the two parties of a pair over CUDA IPC with the "
                         "handoff on the device (default: peer stores into the consumer's HBM and a flag), over CUDA "
                         "IPC with host handoffs (the consumer reads the producer's slot over NVLink), or NCCL "
                         "send/recv")
    ap.add_argument("--aes-tables", type=int, default=4, choices=[2, 4],
                    help="AES engine: 4 staged round tables (default) or 2 tables + rotation")
    ap.add_argument("--relu-split", type=int, default=0, choices=[0, 2, 3],
                    help="comparison split of the ReLU gates: 3 parts (fewest AES) or 2 (smaller keys); "
                         "0 = 3 with resident keys, 2 with --stream")
    ap.add_argument("--relu-backend", default="tt", choices=["tt", "ot", "dcf"],
                    help="comparison backend of the ReLU and truncation gates: dealer digit truth tables with a "
                         "Beaver AND tree (default), OT-leaf digit tables with the same tree (ReLU only), or DCF "
                         "keys (split per --relu-split)")
    ap.add_argument("--gemm", default="tensor", choices=["tensor", "cuda-cores"],
                    help="ring GEMM engine: tcgen05 limb products (default) or the CUDA-core kernel")
    ap.add_argument("--graph", default="on", choices=["on", "off"],
                    help="colocated pairs with resident keys: replay the timed forwards from one CUDA-graph "
                         "capture of both parties (default) or launch them from the host every step")
    ap.add_argument("--no-subrecords", action="store_true",
                    help="skip the sub-records of the line: at N=1 (bw=32) the bw=64 kiba-shaped workload "
                         "(BASELINE configs[3]), at N>1 (colocated) the split layout (party 0 and party 1 on different "
                         "GPUs, openings over CUDA IPC)")
    ap.add_argument("--sub-steps", type=int, default=10, help="timed steps of each sub-record")
    ap.add_argument("--stream", type=int, default=0, metavar="NCHUNKS",
                    help="streaming regime (BASELINE configs[4]): keys of NCHUNKS forwards per party live in pinned "
                         "host memory and are streamed into HBM through the double-buffered key stream, cyclically")
    a = ap.parse_args()
    if a.relu_split == 0:
        a.relu_split = 2 if a.stream else 3
    if a.lanes < 1 or (a.lanes != 1 and a.comm == "nccl"):
        raise SystemExit("--lanes: more than 1 lane per rank needs --comm ipc or ipc-push (see --help)")
    if a.stream and a.batch == 256:
        a.batch = 64  # one chunk per party is ~6.4 GB at bw=32
    return a


def roles(rank: int, world: int):
    """Party layout of a run on `world` GPUs: (pairs, pair index, party, peer rank).
    Ranks 0..k-1 are party 0, ranks k..2k-1 party 1; pair i = (i, k+i)."""
    if world == 1:
        return 1, 0, None, None
    if world % 2:
        raise ValueError("multi-GPU runs need an even number of GPUs (one party per GPU)")
    pairs = world // 2
    pair, party = rank % pairs, rank // pairs
    return pairs, pair, party, rank + pairs if party == 0 else rank - pairs


def measured_peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def atoms_of(bw):
    """Atom-count range of the synthetic graphs: davis-shaped U[10,60] for the
    bw=32 config, kiba-shaped U[10,100] for the bw=64 config ([3])."""
    return (10, 60) if bw == 32 else (10, 100)


def colocated(a, n_gpus):
    return n_gpus == 1 or a.layout == "colocated"


def parallelism(a, n_gpus):
    if n_gpus == 1:
        return "1 GPU, both parties"
    if colocated(a, n_gpus):
        return f"{n_gpus} party pairs, both parties of a pair on one GPU (openings on the device), " \
               "independent micro-batches per GPU"
    over = {"ipc": "CUDA IPC (peer slots read over NVLink, host handoffs)",
            "ipc-push": "CUDA IPC with device-side handoffs (peer stores into the consumer's HBM, flags)",
            "nccl": "NCCL send/recv"}[a.comm]
    return f"{n_gpus // 2} party pairs over {over}, one party per GPU"


def config_of(a, n_gpus):
    pairs = n_gpus if colocated(a, n_gpus) else n_gpus // 2
    if a.stream:
        return {
            "workload": f"streaming regime (BASELINE configs[4]): full affinity branch, bw={a.bw}, scale={a.scale}, "
                        f"B={a.batch} per pair per step, keys streamed host->HBM every step from a ring of "
                        f"{a.stream} pinned chunks per party (timing-only key reuse)",
            "bw": a.bw, "scale": a.scale, "batch_per_pair": a.batch, "pairs": pairs, "stream_chunks": a.stream,
            "relu_split": a.relu_split,
            "parallelism": parallelism(a, n_gpus),
            "l2": "inputs larger than L2: every step copies and streams a full key chunk per party"}
    return {
        "workload": f"full affinity branch (adj-norm, GCNx3, masked max-pool, FC head), bw={a.bw}, scale={a.scale}, "
                    f"B={a.batch} {'davis' if a.bw == 32 else 'kiba'}-shaped synthetic graphs (atoms "
                    f"U{list(atoms_of(a.bw))}) per pair, keys resident in HBM "
                    f"(BASELINE configs[{2 if a.bw == 32 else 3}])",
        "bw": a.bw, "scale": a.scale, "batch_per_pair": a.batch, "pairs": pairs,
        "parallelism": parallelism(a, n_gpus),
        "truncation": "exact (floor) at every site",
        "gemm": "tcgen05 kind::i8 limb products" if a.gemm == "tensor" else "CUDA-core integer multiply-add",
        "aes": f"T-table AES, {a.aes_tables} round tables staged in shared memory",
        "relu_split": a.relu_split,
        "relu_backend": a.relu_backend,
        "launch": (("CUDA graph: both parties' forward captured once, replayed every timed step"
                    if a.layout == "colocated" or n_gpus == 1 else
                    "CUDA graph: each rank's own party forward captured once, replayed every timed step "
                    "(handoffs on the device)") if uses_graph(a) else "host launches every step"),
        "l2": "inputs larger than L2: every step streams each party's full key region (GBs; "
              "key_bytes_per_party_per_step in the line)",
    }


def uses_graph(a):
    """The timed forwards replay a CUDA graph: colocated pairs, or split parties
    over push-mode IPC with one lane per rank, resident keys only."""
    if a.graph != "on" or a.stream:
        return False
    return a.layout == "colocated" or (a.comm == "ipc-push" and a.lanes == 1)


# ------------------------------------------------------------------ clocks

class Clocks:
    """nvidia-smi samples of the job's GPUs (every 50 ms) with host timestamps,
    taken by one process (rank 0) for all of them.  The sampler starts before
    the warm-up steps and has produced a sample before the timed region opens;
    `window(t0, t1)` keeps the samples taken inside the timed region (the
    nearest one on each side when the region is shorter than the sampling
    period) and reports their median SM clock and every active reason."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, indices):
        self.indices = {str(i) for i in indices}
        self.p, self.samples, self.thread = None, [], None

    def start(self):
        import threading

        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                       "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.p = None
            return

        def reader():
            for line in self.p.stdout:
                f = [x.strip() for x in line.split(",")]
                if len(f) < 9 or f[0] not in self.indices:
                    continue
                try:
                    rec = (time.time(), float(f[1]), float(f[2]),
                           [nm for nm, v in zip(self.NAMES, f[5:9]) if v.lower().startswith("active")])
                except ValueError:
                    continue
                self.samples.append(rec)

        self.thread = threading.Thread(target=reader, daemon=True)
        self.thread.start()
        t = time.time()
        while not self.samples and time.time() - t < 10 and self.p.poll() is None:
            time.sleep(0.02)

    def stop(self):
        if self.p:
            self.p.terminate()
            try:
                self.p.wait(timeout=5)
            except Exception:
                self.p.kill()
            if self.thread:
                self.thread.join(timeout=5)

    def window(self, t0, t1):
        if not self.samples:
            return None
        inside = [r for r in self.samples if t0 <= r[0] <= t1]
        if not inside:  # region shorter than the sampling period: one period of margin on both sides
            inside = [r for r in self.samples if t0 - 0.06 <= r[0] <= t1 + 0.06]
        if not inside:
            return None
        reasons = sorted({nm for r in inside for nm in r[3]})
        return {"sm_mhz": statistics.median(r[1] for r in inside), "sm_max_mhz": inside[-1][2], "reasons": reasons,
                "samples": len(inside)}


# ------------------------------------------------------------------ CPU baseline

def physical_cores():
    """Physical cores of this host (distinct (core, socket) pairs of lscpu -p),
    or None when lscpu is unavailable."""
    try:
        out = subprocess.run(["lscpu", "-p=core,socket"], capture_output=True, text=True, timeout=10).stdout
        pairs = {ln.strip() for ln in out.splitlines() if ln and not ln.startswith("#")}
        return len(pairs) or None
    except Exception:
        return None


def check_outputs(bw, inp, q, outs):
    """Parity of the GPU's revealed outputs: the plaintext integer forward of
    the same graph (oracle/ring_forward.py protocol_forward, the function the
    two-party forward must reproduce bit for bit) on all samples of the
    bench's inputs.  outs: {name: (raw, affinity)} of forwards of those inputs.
    Returns (seconds per sample of the plaintext forward, parity record)."""
    import numpy as np

    from oracle import ring_forward as RF

    B = inp.x_ring.shape[0]
    t0 = time.perf_counter()
    want_raw, want_aff = RF.protocol_forward(inp.x_ring, inp.adj_ring, inp.mask_ring, inp.protein_ring, q, bw, 12)
    fwd_s = (time.perf_counter() - t0) / B
    want = RF.Ring(bw).signed(want_raw)
    rec = {"oracle": "plaintext integer forward of the same graph, inputs and weights (protocol_forward)",
           "samples": int(B)}
    ok = True
    for name, (raw, aff) in outs.items():
        bad = int(np.count_nonzero(np.asarray(raw) != want)) + int(np.count_nonzero(np.asarray(aff) != want_aff))
        rec[name] = "bit-exact" if bad == 0 else f"MISMATCH: {bad} values differ"
        ok = ok and bad == 0
    rec["result"] = "bit-exact" if ok else "MISMATCH"
    return fwd_s, rec


def cpu_baseline(bw, relu_n=8_000_000, fwd_samples=2, check=None):
    """Reference LSS ReLU over loopback (all host cores) + plaintext integer
    forward.  With check = (inputs, quantised weights, {name: GPU outputs}) the
    plaintext forward runs on the bench's own B samples and doubles as the
    parity check of the GPU outputs."""
    cores = os.cpu_count() or 2
    exe = os.path.join(REPO, "oracle", "_ref", "lss_bench")
    kind, relu_s_per_sample, detail = "port", None, {}
    if os.path.exists(exe):
        r = subprocess.run([exe, str(relu_n), str(bw), str(max(cores // 2, 1))], capture_output=True, text=True,
                           timeout=600)
        d = json.loads(r.stdout.strip().splitlines()[-1])
        if "seconds" in d:
            kind = "reference"
            relu_s_per_sample = d["seconds"] * RELUS_PER_SAMPLE / relu_n
            detail = d
    parity = None
    if check is not None:
        inp, q, outs = check
        fwd_samples = int(inp.x_ring.shape[0])
        fwd_s, parity = check_outputs(bw, inp, q, outs)
    else:
        from oracle import ring_forward as RF

        synth = importlib.import_module("idash26-track3_b200.synth")
        inp = synth.Inputs(fwd_samples, bw, seed=3, with_protein_cnn=False)
        q = synth.quantize_weights(synth.affinity_weights(5), 12)
        t0 = time.perf_counter()
        RF.protocol_forward(inp.x_ring, inp.adj_ring, inp.mask_ring, inp.protein_ring, q, bw, 12)
        fwd_s = (time.perf_counter() - t0) / fwd_samples
    per_sample = fwd_s + (relu_s_per_sample or 0.0)
    sample = (f"reference LSS ReLU (gpu_mpc/lss compiled unmodified, 2 processes over loopback TCP, "
              f"{max(cores // 2, 1)} OpenMP threads each) timed on {relu_n} elements at bw={bw} and extrapolated "
              f"linearly to the {RELUS_PER_SAMPLE} ReLUs of a sample; plus the plaintext integer forward "
              f"(numpy, oracle/ring_forward.py, one thread) timed on {fwd_samples} samples for the linear layers"
              if kind == "reference" else
              f"plaintext integer forward only (oracle/ring_forward.py, {fwd_samples} samples); LSS binary absent")
    out = {"value": 1.0 / per_sample, "unit": "samples/s", "cores": cores, "physical_cores": physical_cores(),
           "kind": kind, "sample": sample, "relu_s_per_sample": relu_s_per_sample,
           "relu_extrapolated_from_elements": relu_n if kind == "reference" else None,
           "linear_s_per_sample": fwd_s, "lss": detail}
    if parity is not None:
        out["parity"] = parity
    return out


def np_equal(a, b):
    import numpy as np

    return all(np.array_equal(np.asarray(x), np.asarray(y)) for x, y in zip(a, b))


def run_reference(a, rank, world):
    if rank != 0:
        return
    t_steps = []
    for i in range(a.warmup + a.steps):
        t0 = time.perf_counter()
        cb = cpu_baseline(a.bw, relu_n=2_000_000, fwd_samples=1)
        if i >= a.warmup:
            t_steps.append((time.perf_counter() - t0, cb))
    vals = [cb["value"] for _, cb in t_steps]
    v = statistics.median(vals)
    cb = t_steps[-1][1]
    cb = dict(cb, value=v)
    line = {"impl": "reference", "metric": "online 2PC samples/sec (full affinity branch)", "value": v,
            "unit": "samples/s", "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": 1e3 * statistics.median([t for t, _ in t_steps]), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": f"u{a.bw}", "data": "synthetic",
            "config": config_of(a, world), "cpu_baseline": cb,
            "e2e": {"value": v, "unit": "samples/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    emit(line)


# ------------------------------------------------------------------ our arm

class _StreamLane:
    """adapts a KeyStream to the forward(batch, x, adj, mask, prot, on_host) call of a lane"""

    def __init__(self, ks):
        self.ks = ks

    def forward(self, batch, x, adj, mask, prot, on_host=False):
        return self.ks.forward(x, adj, mask, prot, on_host=on_host)


def make_keys(ddg, torch, bw, s, B, seed, blob, device):
    kb = ddg.forward_key_bytes(bw, s, B)
    k0 = torch.empty(kb, dtype=torch.uint8, device=device)
    k1 = torch.empty(kb, dtype=torch.uint8, device=device)
    ddg.dealer_forward(bw, s, B, seed, blob, device.index, k0.data_ptr(), k1.data_ptr())
    torch.cuda.synchronize(device)
    return kb, k0, k1


def share_buffers(torch, inp, party, device, rows=None):
    import numpy as np

    sl = slice(None) if rows is None else slice(*rows)
    arrs = [np.ascontiguousarray(x[party][sl]) for x in (inp.x_sh, inp.adj_sh, inp.mask_sh, inp.protein_sh)]
    dev = [torch.from_numpy(a.view(np.uint8).copy()).to(device) for a in arrs]
    host = [torch.from_numpy(a.view(np.uint8).copy()).pin_memory() for a in arrs]
    return dev, host


def h2d_probe(torch, bufs, device):
    """Host->device bandwidth of this box for the e2e inputs: the same pinned
    buffers copied once into fresh device tensors (GB/s), outside any timed
    region; the e2e step's copies run at about this rate."""
    srcs = [t for b in bufs for t in b[1]]
    dsts = [torch.empty_like(t, device=device) for t in srcs]
    st = torch.cuda.Stream(device=device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(st):
        e0.record(st)
        for d, h in zip(dsts, srcs):
            d.copy_(h, non_blocking=True)
        e1.record(st)
    e1.synchronize()
    nbytes = sum(int(t.numel()) for t in srcs)
    return nbytes / (e0.elapsed_time(e1) / 1e3) / 1e9


def _timed_steps(torch, stream, device, fn, k):
    """k calls of fn() between CUDA events on `stream`, synchronised on both sides; ms"""
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(k):
        fn()
    e1.record(stream)
    torch.cuda.synchronize(device)
    return e0.elapsed_time(e1)


def subrecord_bw64(a, ddg, synth, torch, device, local):
    """BASELINE configs[3] on the same GPU after the main measurement: bw=64,
    kiba-shaped graphs (atoms U[10,100]), B = --batch, both parties on the GPU,
    CUDA-graph replay.  Returns (record, (inputs, outputs)) for the parity check."""
    bw, s, B = 64, a.scale, a.batch
    blob = synth.weights_blob(synth.quantize_weights(synth.affinity_weights(5), s))
    inp = synth.Inputs(B, bw, seed=2000, atoms=atoms_of(bw))
    kb, k0, k1 = make_keys(ddg, torch, bw, s, B, 2097, blob, device)
    parties = [ddg.Party(0, bw, s, local), ddg.Party(1, bw, s, local)]
    for p, k in zip(parties, (k0, k1)):
        p.set_weights(blob)
        p.bind_keys(k.data_ptr(), kb)
    ddg.pair_local(parties[0], parties[1])
    bufs = [share_buffers(torch, inp, p, device) for p in (0, 1)]
    ins = [[t.data_ptr() for t in bufs[p][0]] for p in (0, 1)]
    outs = {}
    for _ in range(a.warmup):
        outs["warmup_forward"] = ddg.forward_pair(parties[0], parties[1], B, ins[0], ins[1])
    g = ddg.ForwardGraph(parties[0], parties[1], B, ins[0], ins[1])
    try:
        outs["graph_replay"] = g.launch()
        stream = torch.cuda.ExternalStream(parties[0].stream, device=device)
        ms = _timed_steps(torch, stream, device, g.launch, a.sub_steps)
    finally:
        g.close()
    for p in parties:
        p.close()
    del k0, k1, bufs
    torch.cuda.empty_cache()
    rec = {"workload": f"full affinity branch, bw=64, scale={s}, B={B} kiba-shaped synthetic graphs (atoms "
                       f"U[10, 100]), keys resident, both parties on the GPU, CUDA-graph replay (BASELINE configs[3])",
           "value": B * a.sub_steps / (ms / 1e3), "unit": "samples/s", "ms_per_step": ms / a.sub_steps,
           "steps": a.sub_steps, "warmup": a.warmup, "dtype": "u64", "key_bytes_per_party_per_step": kb,
           "e2e_key_frac": 2 * kb / (ms / a.sub_steps / 1e3) / 1e9 / measured_peaks()[0]}
    return rec, (inp, outs)


def subrecord_split(a, ddg, synth, torch, dist, rank, world, local, device, push=True):
    """The split layout on the same GPUs after the colocated measurement: ranks
    0..k-1 party 0, ranks k..2k-1 party 1, pair i = (i, k+i), each pair on its
    own micro-batch of B, openings over CUDA IPC (NVLink).  Time max over ranks."""
    bw, s, B = a.bw, a.scale, a.batch
    pairs, pair, party, peer = roles(rank, world)
    blob = synth.weights_blob(synth.quantize_weights(synth.affinity_weights(5), s))
    inp = synth.Inputs(B, bw, seed=3000 + pair, atoms=atoms_of(bw))
    tag = uuid.uuid4().hex[:16]
    names = [[f"ddg_{tag}_s{i}" for i in range(pairs)] if rank == 0 else None]
    dist.broadcast_object_list(names, src=0)
    P = ddg.Party(party, bw, s, local)
    P.set_weights(blob)
    kb, k0, k1 = make_keys(ddg, torch, bw, s, B, 3000 + 97 * pair, blob, device)
    mine = k0 if party == 0 else k1
    del k0, k1
    torch.cuda.empty_cache()
    P.bind_keys(mine.data_ptr(), kb)
    P.set_timeout(1000 * a.peer_timeout)
    P.connect_ipc(names[0][pair], ddg.forward_max_exchange_bytes(bw, s, B), push=push)
    buf = share_buffers(torch, inp, party, device)
    ins = [t.data_ptr() for t in buf[0]]
    o = None
    for _ in range(a.warmup):
        o = P.forward(B, *ins)
    # push mode: every handoff happens on the device, so each rank replays its
    # own party's forward from a CUDA graph (both ranks alike)
    g, agree = None, None
    if push and a.graph == "on":
        g = ddg.ForwardGraph(P, None, B, ins)
        og = g.launch()  # untimed: the first replay uploads the graph
        agree = bool(o is not None and (o[0] == og[0]).all())
    dist.barrier()
    stream = torch.cuda.ExternalStream(P.stream, device=device)
    ms = _timed_steps(torch, stream, device, (lambda: g.enqueue()) if g else (lambda: P.forward(B, *ins)),
                      a.sub_steps)
    if g is not None:
        og2 = g.sync()  # status of the timed replays (a device-side wait that gave up raises)
        agree = bool(agree and (og2[0] == o[0]).all())
    t = torch.tensor([ms], device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    st = P.stats()
    if g is not None:
        g.close()
    dist.barrier()
    P.close()
    del mine, buf
    torch.cuda.empty_cache()
    value = pairs * B * a.sub_steps / (ms / 1e3)
    return {"layout": "split: ranks 0..k-1 party 0, ranks k..2k-1 party 1, pair i = (i, k+i), one micro-batch per "
                      "pair, openings over CUDA IPC " + ("with device-side handoffs (peer stores into the consumer's "
                      "HBM, flags)" if push else "with host handoffs (send slots read in place over NVLink)"),
            "pairs": pairs, "value": value, "unit": "samples/s", "ms_per_step": ms / a.sub_steps,
            "steps": a.sub_steps, "warmup": a.warmup, "samples_per_s_per_gpu": value / world,
            "nvlink_bytes_per_step": 2 * pairs * st["bytes_sent"], "openings_per_step": st["rounds"],
            "launch": ("CUDA graph of each rank's own party forward, replayed every step" if g is not None
                       else "host-launched forward on each rank"),
            "graph_output_equals_host_forward": agree}


def main():
    a = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != a.gpus:
        a.gpus = world if world > 1 else a.gpus
    if a.impl == "reference":
        run_reference(a, rank, world)
        return
    import numpy as np
    import torch

    ddg = importlib.import_module("idash26-track3_b200")
    synth = importlib.import_module("idash26-track3_b200.synth")
    ddg.gemm_path(ddg.GEMM_TENSOR if a.gemm == "tensor" else ddg.GEMM_CUDA_CORES)
    ddg.aes_tables(a.aes_tables)
    ddg.relu_split(a.relu_split)
    ddg.relu_backend({"tt": ddg.RELU_TT, "ot": ddg.RELU_OT, "dcf": ddg.RELU_DCF}[a.relu_backend])
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist = None
    if world > 1:
        import torch.distributed as dist

        if world % 2 and a.layout == "split":
            raise SystemExit("the split layout needs an even number of GPUs (one party per GPU)")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=900), device_id=device)
    B, bw, s = a.batch, a.bw, a.scale
    blob = synth.weights_blob(synth.quantize_weights(synth.affinity_weights(5), s))

    # -------- parties, keys, inputs
    streams = []
    colo = colocated(a, world)
    if colo:
        pairs, pair = world, rank
        inp = synth.Inputs(B, bw, seed=1000 + pair, atoms=atoms_of(bw))
        parties = [ddg.Party(0, bw, s, local), ddg.Party(1, bw, s, local)]
        if a.stream:
            kb = ddg.forward_key_bytes(bw, s, B)
            chunks = ddg.dealer_chunks(bw, s, B, [1000 + 97 * pair + i for i in range(a.stream)], blob, local)
            for p in parties:
                p.set_weights(blob)
            streams = [ddg.KeyStream(p, B) for p in parties]
            for c in chunks:
                for ks, h in zip(streams, c):
                    ks.add_host_chunk(h.data_ptr())
        else:
            kb, k0, k1 = make_keys(ddg, torch, bw, s, B, 1000 + 97 * pair, blob, device)
            for p, k in zip(parties, (k0, k1)):
                p.set_weights(blob)
                p.bind_keys(k.data_ptr(), kb)
        ddg.pair_local(parties[0], parties[1])
        bufs = [share_buffers(torch, inp, p, device) for p in (0, 1)]
    else:
        pairs, pair, party, peer = roles(rank, world)
        lanes = a.lanes
        if B % lanes:
            raise SystemExit(f"--batch {B} not divisible by --lanes {lanes}")
        Bl = B // lanes
        inp = synth.Inputs(B, bw, seed=1000 + pair, atoms=atoms_of(bw))
        # one channel per party pair (and lane): a pair's openings never
        # involve the other ranks
        if a.comm != "nccl":
            tag = uuid.uuid4().hex[:16]
            uids = [[[f"ddg_{tag}_{i}_{l}" for l in range(lanes)] for i in range(pairs)] if rank == 0 else None]
        else:
            uids = [[[ddg.nccl_unique_id() for _ in range(lanes)] for _ in range(pairs)] if rank == 0 else None]
        dist.broadcast_object_list(uids, src=0)
        parties, keep_keys = [], []
        for lane in range(lanes):
            P = ddg.Party(party, bw, s, local)
            P.set_weights(blob)
            seed = 1000 + 97 * pair + 7 * lane
            if a.stream:
                kb = ddg.forward_key_bytes(bw, s, Bl)
                chunks = ddg.dealer_chunks(bw, s, Bl, [seed + i for i in range(a.stream)], blob, local)
                ks = ddg.KeyStream(P, Bl)
                for c in chunks:
                    ks.add_host_chunk(c[party].data_ptr())
                keep_keys.append([c[party] for c in chunks])
                del chunks
                streams.append(ks)
            else:
                kb, k0, k1 = make_keys(ddg, torch, bw, s, Bl, seed, blob, device)
                mine = k0 if party == 0 else k1
                del k0, k1
                torch.cuda.empty_cache()
                P.bind_keys(mine.data_ptr(), kb)
                keep_keys.append(mine)
            P.set_timeout(1000 * a.peer_timeout)
            if a.comm != "nccl":
                P.connect_ipc(uids[0][pair][lane], ddg.forward_max_exchange_bytes(bw, s, Bl), push=a.comm == "ipc-push")
            else:
                P.connect_nccl(uids[0][pair][lane], 2, party, 1 - party)
            parties.append(P)
        bufs = [share_buffers(torch, inp, party, device, (lane * Bl, (lane + 1) * Bl)) for lane in range(lanes)]

    graph = [None]

    def step(on_host):
        if graph[0] is not None and not on_host:
            # a forward graph's replays follow each other with no host round trip
            # (read back after the timed steps); the e2e pipeline submits
            return graph[0].enqueue() if hasattr(graph[0], "enqueue") else graph[0].launch()
        if colo:
            ins = [[t.data_ptr() for t in (bufs[p][1] if on_host else bufs[p][0])] for p in (0, 1)]
            if streams:
                return ddg.forward_pair_streamed(streams[0], streams[1], ins[0], ins[1], on_host=on_host)
            return ddg.forward_pair(parties[0], parties[1], B, ins[0], ins[1], on_host=on_host)
        ins = [[t.data_ptr() for t in (b[1] if on_host else b[0])] for b in bufs]
        if streams:
            out = ddg.forward_lanes([_StreamLane(ks) for ks in streams], B // len(parties), ins, on_host)
        else:
            out = ddg.forward_lanes(parties, B // len(parties), ins, on_host)
        return out

    stream = torch.cuda.ExternalStream(parties[0].stream, device=device)

    def timed(on_host, k, wall=None):
        if dist:
            dist.barrier()
        torch.cuda.synchronize(device)
        if wall is not None:
            wall[0] = time.time()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(k):
            step(on_host)
        e1.record(stream)
        torch.cuda.synchronize(device)
        if wall is not None:
            wall[1] = time.time()
        ms = e0.elapsed_time(e1)
        if dist:
            t = torch.tensor([ms], device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
            dist.barrier()
        return ms

    clocks = Clocks(range(world) if world > 1 else [local])
    if rank == 0:
        clocks.start()
    outs = {}  # revealed outputs of untimed forwards of the timed inputs (colocated, resident keys)
    o = None
    for _ in range(a.warmup):
        o = step(False)
    if colo and not streams and o is not None:
        outs["warmup_forward"] = o
    ks_before = [ks.stats() for ks in streams]
    for p in parties:
        p.enable_dcf_timing(True)
    graph_ok = False
    if colo and uses_graph(a):
        # capture after the warm-up forwards (one-time set-up done), with the
        # comparison-kernel timing on, so that every replay records its launches
        try:
            graph[0] = ddg.ForwardGraph(parties[0], parties[1], B, [t.data_ptr() for t in bufs[0][0]],
                                        [t.data_ptr() for t in bufs[1][0]])
            outs["graph_replay"] = graph[0].launch()  # untimed: the first replay uploads the graph
            graph_ok = True
        except Exception as ex:  # noqa: BLE001 -- any capture failure falls back to host launches
            # a failed capture may leave the pair's channel marked failed: pair the
            # parties again and launch from the host, and say so in config.launch
            print(f"bench: CUDA-graph capture failed ({ex}); timing host launches instead", file=sys.stderr)
            if graph[0] is not None:
                graph[0].close()
            graph[0] = None
            a.graph = "off"
            ddg.pair_local(parties[0], parties[1])
            step(False)
            for p in parties:
                p.enable_dcf_timing(True)
    elif uses_graph(a):
        # split, push-mode IPC: every rank captures its own party's forward (all
        # handoffs on the device) after the warm-up forwards; a failed capture
        # ends the run (the peer's replays then give up at --peer-timeout)
        graph[0] = ddg.ForwardGraph(parties[0], None, B, [t.data_ptr() for t in bufs[0][0]])
        graph[0].launch()  # untimed: the first replay uploads the graph
        graph_ok = True
    n0 = ddg.launch_count()
    tw = [0.0, 0.0]
    ms = timed(False, a.steps, tw)
    launches = ddg.launch_count() - n0
    if graph[0] is not None:
        # the last timed replay's output (checked against the oracle with the others), and
        # the GEMM and channel status words of the timed replays
        last = graph[0].sync()
        if colo and not streams:
            outs["graph_timed_last"] = last
    clocks.stop()
    clk = clocks.window(*tw)
    stats = parties[0].stats()
    if not colo:
        lane_stats = [p.stats() for p in parties]
        stats = {"bytes_sent": sum(x["bytes_sent"] for x in lane_stats), "rounds": lane_stats[0]["rounds"],
                 "key_bytes_used": sum(x["key_bytes_used"] for x in lane_stats)}
        kb = sum(ddg.forward_key_bytes(bw, s, B // len(parties)) for _ in parties)
    # the launch events of the timed steps are read back here, after the timed region
    if len(parties) > 1:
        ddg.parties_dcf_union(parties)
    dcf = [p.dcf_timing() for p in parties]
    stream_info = None
    if streams:
        after = [ks.stats() for ks in streams]
        copied = sum(x["bytes"] - y["bytes"] for x, y in zip(after, ks_before))
        copy_ms = sum(x["copy_ms"] - y["copy_ms"] for x, y in zip(after, ks_before))
        stream_info = {"chunk_bytes": ddg.key_chunk_bytes(bw, s, B), "chunks_per_party": a.stream,
                       "h2d_bytes_per_step_per_gpu": copied / a.steps,
                       "h2d_gbs_during_copies": copied / (copy_ms / 1e3) / 1e9 if copy_ms else None,
                       "h2d_gbs_over_step": copied / (ms / 1e3) / 1e9}
    # with a graph the launch events hold the last replay: one forward's launches
    fwd_timed = 1 if graph[0] is not None else a.steps
    if graph[0] is not None:
        graph[0].close()
        graph[0] = None
    for p in parties:
        p.enable_dcf_timing(False)

    e2e = None
    if not a.no_e2e:
        o = step(True)
        if colo and not streams:
            outs["e2e_forward"] = o
        e2e_graph, pipe, e2e_how = None, None, "host launches every step"
        if colo and uses_graph(a) and graph_ok:
            # pipelined forwards on the pinned host input shares: two graphs of the
            # forward on alternating device staging sets, each step's host->device
            # copies overlapping the previous step's forward
            try:
                pipe = ddg.ForwardPipeline(parties[0], parties[1], B)
                hp = [[t.data_ptr() for t in bufs[p][1]] for p in (0, 1)]
                first = pipe.submit(hp[0], hp[1])
                pipe.wait()
                outs["e2e_pipeline"] = first

                class _PipelineStep:
                    def launch(self):
                        return pipe.submit(hp[0], hp[1])

                e2e_graph = _PipelineStep()
                graph[0] = e2e_graph
                e2e_how = ("pipelined CUDA graphs of both parties' forward (ddg_forward_pipeline): every step copies "
                           "its pinned input shares host->device on a copy stream, overlapping the previous step's "
                           "forward, and reads its output back")
            except Exception as ex:  # noqa: BLE001 -- fall back to the host-input graph
                print(f"bench: forward pipeline failed ({ex}); e2e with a host-input graph", file=sys.stderr)
                if pipe is not None:
                    pipe.close()
                pipe, e2e_graph = None, None
                ddg.pair_local(parties[0], parties[1])
                step(True)
        if colo and uses_graph(a) and graph_ok and e2e_graph is None:
            # the same forward with the pinned host inputs captured too: every
            # replay copies both parties' input shares host -> device
            try:
                e2e_graph = ddg.ForwardGraph(parties[0], parties[1], B, [t.data_ptr() for t in bufs[0][1]],
                                             [t.data_ptr() for t in bufs[1][1]], on_host=True)
                outs["e2e_graph_replay"] = e2e_graph.launch()
                graph[0] = e2e_graph
                e2e_how = ("CUDA graph of both parties' forward with the host->device copies of their pinned input "
                           "shares and the output read-back, replayed every step")
            except Exception as ex:  # noqa: BLE001 -- fall back to host launches for the e2e steps
                print(f"bench: host-input graph capture failed ({ex}); e2e with host launches", file=sys.stderr)
                if e2e_graph is not None:
                    e2e_graph.close()
                e2e_graph = None
                ddg.pair_local(parties[0], parties[1])
                step(True)
        ms_e2e = timed(True, a.steps) if e2e_graph is None else timed(False, a.steps)
        if pipe is not None:
            pipe.wait()  # hands the timed steps' outputs over (their read-backs ran inside the timed region)
            pipe.close()
            graph[0] = None
        elif e2e_graph is not None:
            e2e_graph.close()
            graph[0] = None
        # both parties' input shares of every pair cross host->device each step
        own = [sum(int(t.numel()) for t in b[1]) for b in bufs]
        h2d = sum(own) if colo else 2 * sum(own)
        e2e = {"value": pairs * B * a.steps / (ms_e2e / 1e3), "unit": "samples/s",
               "h2d_bytes_per_step": h2d * pairs, "d2h_bytes_per_step": B * (bw // 8) * pairs,
               "ms_per_step": ms_e2e / a.steps, "h2d_probe_gbs": h2d_probe(torch, bufs, device),
               "launch": e2e_how}
        if pipe is not None:
            e2e["note"] = ("the timed forwards of `value` carry the comparison-kernel event records of the live "
                           "roofline (about 140 per forward); the pipeline's graphs carry none, and its input copies "
                           "run beside the forwards, so e2e can read slightly above value")

    value = pairs * B * a.steps / (ms / 1e3)
    peak, peak_kind = measured_peaks()
    if colo:
        union = dcf[0]["pair_union_ms"]
        alg = dcf[0]["bytes"] + dcf[1]["bytes"]
        aes = dcf[0]["aes_blocks"] + dcf[1]["aes_blocks"]
        nl = dcf[0]["launches"] + dcf[1]["launches"]
    else:
        union = dcf[0]["pair_union_ms"] if len(parties) > 1 else dcf[0]["union_ms"]
        alg = sum(d["bytes"] for d in dcf)
        aes = sum(d["aes_blocks"] for d in dcf)
        nl = sum(d["launches"] for d in dcf)
    achieved = alg / (union / 1e3) / 1e9 if union > 0 else 0.0
    ratio = NCU_DRAM_BYTES_PER_ALG_BYTE.get(a.relu_backend)
    # both parties' key regions stream from HBM once per step (colocated: on this GPU)
    key_bytes_per_gpu_step = (2 if colo else 1) * kb
    roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                "frac": achieved / peak, "peak_source": peak_kind,
                "traffic": (alg / nl * ratio) if (nl and ratio) else None,
                "traffic_note": "DRAM bytes per launch = algorithmic bytes per launch x the DRAM/algorithmic "
                                "ratio of an ncu capture of the same kernel",
                "e2e_key_frac": key_bytes_per_gpu_step / (ms / a.steps / 1e3) / 1e9 / peak,
                "e2e_key_note": "key bytes of both parties of a pair streamed per step on one GPU, over the "
                                "step time, against the measured HBM copy bandwidth (the key-bytes-over-HBM "
                                "roofline of the whole forward)",
                "kernel": {"tt": "comparison kernels: ot_level_kernel (truth tables + AND-tree levels of the "
                                 "ReLU and truncation gates)",
                           "ot": "comparison kernels: ot_garble_kernel + ot_level_kernel (ReLU gates) and "
                                 "gate_round1_kernel (DCF, truncation gates)",
                           "dcf": "gate_round1_kernel (DCF evaluation)"}[a.relu_backend], "launches": nl,
                "dcf_share_of_step": union / (ms * fwd_timed / a.steps) if ms > 0 else None,
                "aes_gblocks_per_s": aes / (union / 1e3) / 1e9 if union > 0 else 0.0}
    # AES ceiling on this GPU (the binding roofline of the DCF): fixed-key hash chains
    out = torch.zeros(148 * 3 * 256 * 8, dtype=torch.int32, device=device)
    ddg.check(ddg.lib().ddg_aes_chain(out.numel(), 64, out.data_ptr(), None))
    torch.cuda.synchronize(device)
    ea, eb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ea.record()
    for _ in range(3):
        ddg.check(ddg.lib().ddg_aes_chain(out.numel(), 64, out.data_ptr(), torch.cuda.current_stream().cuda_stream))
    eb.record()
    torch.cuda.synchronize(device)
    aes_peak = out.numel() * 64 * 3 / (ea.elapsed_time(eb) / 1e3) / 1e9
    roofline["aes_peak_gblocks_per_s"] = aes_peak
    roofline["aes_frac"] = roofline["aes_gblocks_per_s"] / aes_peak if aes_peak else None

    # sub-records, after the main run's parties and keys are released
    for ks in streams:
        ks.close()
    for p in parties:
        p.close()
    streams, parties, bufs, k0, k1, keep_keys = [], [], None, None, None, None
    torch.cuda.empty_cache()
    sub, chk64 = {}, None
    if not a.no_subrecords and not a.stream and colo:
        if world == 1 and bw == 32:
            sub["bw64"], chk64 = subrecord_bw64(a, ddg, synth, torch, device, local)
        elif world > 1:
            sub["split"] = subrecord_split(a, ddg, synth, torch, dist, rank, world, local, device, push=True)
            sub["split_host_handoff"] = subrecord_split(a, ddg, synth, torch, dist, rank, world, local, device,
                                                        push=False)

    cb = None
    parity = None
    # the GPU outputs agree among themselves (graph replay, host launches, host buffers)
    names = list(outs)
    same = all(np_equal(outs[n], outs[names[0]]) for n in names[1:]) if names else None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        q = synth.quantize_weights(synth.affinity_weights(5), s)
        cb = cpu_baseline(bw, check=(inp, q, outs) if outs else None)
        parity = cb.pop("parity", None)
        if chk64 is not None:
            _, sub["bw64"]["parity"] = check_outputs(64, chk64[0], q, chk64[1])
    if parity is None:
        parity = {"result": "not checked against the oracle (N > 1, streaming or --no-cpu-baseline)",
                  "gpu_paths_agree": same}
    else:
        parity["gpu_paths_agree"] = same
    if rank == 0:
        line = {"metric": "online 2PC samples/sec (full affinity branch)", "value": value, "unit": "samples/s",
                "n_gpus": world, "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms / a.steps,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": value / A10_SAMPLES_PER_S,
                "vs_baseline_note": "reference's published 136 ms per batch of 16 on one A10 (README.md:99-101)",
                "dtype": f"u{bw}", "data": "synthetic", "config": config_of(a, world), "roofline": roofline,
                "cpu_baseline": cb, "e2e": e2e, "gpu_launches": launches, "clocks": clk,
                "comm": {"bytes_sent_per_party_per_step": stats["bytes_sent"], "rounds_per_step": stats["rounds"],
                         "bytes_per_sample": 2 * stats["bytes_sent"] / B,
                         # emulated LAN, full duplex: each party's bytes at 1 Gbps + one 1 ms RTT per opening
                         "lan_1gbps_1ms_rtt_s_per_step": stats["bytes_sent"] * 8 / 1e9 + stats["rounds"] * 1e-3},
                "key_bytes_per_party_per_step": kb, "stream": stream_info, "parity": parity,
                "subrecords": sub or None}
        emit(line)
        bad64 = sub.get("bw64", {}).get("parity", {}).get("result") == "MISMATCH"
        if parity.get("result") == "MISMATCH" or same is False or bad64:
            raise SystemExit("bench: the GPU forward's outputs do not match (see parity in the JSON line)")
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    stdout_for_json_only()
    main()
