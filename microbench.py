"""Kernel microbenchmarks of the online path (BASELINE configs[1] and the GEMM rows).

    python microbench.py dcf  [--sizes 20 22 24 26] [--bw 32 64]
    python microbench.py lut  [--n 1048576]
    python microbench.py gemm [--batch 256]
    python microbench.py aes
    python microbench.py tt   [--sizes 23] [--bw 32]

Prints one JSON object.  Everything goes through libddg.so's C ABI on cuda:0:

* dcf  -- 2^k independent comparisons 1{x < r} with 1-bit output (the round-1
  kernel of the DReLU gate: a (bw-1)-bit DCF, GATE_RELU) and, beside it, the
  split form the forward uses (GATE_RELU_SPLIT: 19/51-bit DCF with equality
  + 12-bit DCF) and the split-carry truncation (GATE_LRS_SPLIT).  Keys come
  from the GPU dealer with a fixed seed; inputs are uniform in Z_2^bw.
  Reported: evals/s, key GB/s against the measured HBM copy bandwidth, and
  AES blocks/s against the AES probe.  Key arrays are larger than L2 from
  2^20 elements on, and each timed launch reads its whole key once.
* lut  -- 2^20 DPF look-ups into the 139-entry 2^12/sqrt(k) table.
* gemm -- the GCN layer-3 ring GEMMs at B samples: the FC (B*138 x 282) .
  (282 x 376) and the per-sample Beaver product (138 x 138) . (138 x 282),
  on the tensor cores (tcgen05 kind::i8 limb products; default and wide
  column tiles) and on the CUDA cores.
* aes  -- the fixed-key AES ceiling of both AES engines.
* tt   -- both parties of one truth-table gate (full-compare ReLU, ReLU-ARS,
  truncation carry) through ddg_gate_eval_pair: all AND-tree levels, the
  openings in place on the device, and round 2.

Timing: CUDA events on the launching stream after warm-up launches; the
median of the timed repetitions.
"""
from __future__ import annotations

import argparse
import importlib
import json
import os
import sys

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)


def peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def timeit(torch, fn, warm=2, reps=5):
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b))
    ts.sort()
    return ts[len(ts) // 2] / 1e3


def aes_ceiling(ddg, torch, tables=0):
    n, iters = 148 * 768 * 8, 64
    out = torch.zeros(n, dtype=torch.int32, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    t = timeit(torch, lambda: ddg.check(ddg.lib().ddg_aes_chain_variant(n, iters, tables, out.data_ptr(), st)))
    return n * iters / t / 1e9


def run_dcf(ddg, torch, a):
    hbm, _, src = peaks()
    res = {"hbm_peak_gbs": hbm, "peak_source": src, "aes_ceiling_gblocks": aes_ceiling(ddg, torch)}
    st = torch.cuda.current_stream().cuda_stream
    for bw in a.bw:
        dt = torch.int32 if bw == 32 else torch.int64
        for kind, name in ((ddg.GATE_RELU, "dcf"), (ddg.GATE_RELU_SPLIT, "split"), (ddg.GATE_LRS_SPLIT, "lrs_split")):
            for lg in a.sizes:
                N = 1 << lg
                kb = ddg.gate_key_bytes(kind, bw, 12, N)
                # two key regions + inputs must fit next to what torch already holds
                if 2 * kb + 64 * N > 0.8 * torch.cuda.mem_get_info()[0]:
                    res[f"bw{bw}_{name}_2^{lg}"] = "skipped: keys do not fit"
                    continue
                k0 = torch.empty(kb, dtype=torch.uint8, device="cuda")
                k1 = torch.empty(kb, dtype=torch.uint8, device="cuda")
                g = torch.Generator(device="cuda").manual_seed(lg + bw)
                info = torch.iinfo(dt)
                r = torch.randint(info.min, info.max, (N,), dtype=dt, device="cuda", generator=g)
                x = torch.randint(info.min, info.max, (N,), dtype=dt, device="cuda", generator=g)
                if kind == ddg.GATE_LRS_SPLIT:
                    x = x & info.max  # LRS precondition: x in [0, 2^(bw-1))
                ro = torch.empty_like(r)
                ddg.gate_keygen(kind, bw, 12, N, 1, 1, r.data_ptr(), ro.data_ptr(), k0.data_ptr(), k1.data_ptr(), st)
                xh = x + r
                words = (N + 31) // 32
                bh = torch.empty(2 * words, dtype=torch.int32, device="cuda")
                bl = torch.empty(words, dtype=torch.int32, device="cuda")
                t = timeit(torch, lambda: ddg.gate_round1(kind, bw, 12, N, xh.data_ptr(), k0.data_ptr(), bh.data_ptr(),
                                                          bl.data_ptr(), st))
                lay = ddg.gate_key_layout(kind, bw, 12, N)
                # algorithmic bytes: every DCF key byte once, the input, the output bits
                nbits = 1 if kind == ddg.GATE_RELU else 3
                alg = lay["words"] + N * bw // 8 + nbits * N / 8
                aes = lay["hi_levels"] + 1 + (lay["lo_levels"] + 1 if kind != ddg.GATE_RELU else 0)
                res[f"bw{bw}_{name}_2^{lg}"] = {
                    "evals_per_s": N / t, "ms": t * 1e3, "key_bytes_per_eval": lay["words"] / N,
                    "aes_per_eval": aes, "gbs": alg / t / 1e9, "hbm_frac": alg / t / 1e9 / hbm,
                    "aes_gblocks_per_s": N * aes / t / 1e9}
                del k0, k1, r, x, xh, ro, bh, bl
                torch.cuda.empty_cache()
    return res


def run_lut(ddg, torch, a):
    import numpy as np

    hbm, _, src = peaks()
    L = ddg.lib()
    res = {"hbm_peak_gbs": hbm, "peak_source": src}
    st = torch.cuda.current_stream().cuda_stream
    for bw in (32, 64):
        dt = torch.int32 if bw == 32 else torch.int64
        n = a.n
        kb = int(L.ddg_lut_key_bytes(bw, n))
        k0 = torch.empty(kb, dtype=torch.uint8, device="cuda")
        k1 = torch.empty(kb, dtype=torch.uint8, device="cuda")
        g = torch.Generator(device="cuda").manual_seed(bw)
        info = torch.iinfo(dt)
        r = torch.randint(info.min, info.max, (n,), dtype=dt, device="cuda", generator=g)
        ro = torch.randint(info.min, info.max, (n,), dtype=dt, device="cuda", generator=g)
        deg = torch.randint(0, 139, (n,), dtype=dt, device="cuda", generator=g)
        tab = np.zeros(256, dtype=np.int64)
        tab[1:139] = np.floor(4096 / np.sqrt(np.arange(1, 139)) + 0.5)
        d_tab = torch.from_numpy(tab.astype(np.int32 if bw == 32 else np.int64)).cuda()
        ddg.check(L.ddg_lut_keygen(bw, n, 3, 5, r.data_ptr(), ro.data_ptr(), k0.data_ptr(), k1.data_ptr(), st))
        xh = deg + r
        out = torch.empty_like(r)
        t = timeit(torch, lambda: ddg.check(L.ddg_lut_eval(bw, n, 0, xh.data_ptr(), d_tab.data_ptr(), k0.data_ptr(),
                                                           out.data_ptr(), st)))
        alg = kb + 2 * n * bw // 8
        res[f"bw{bw}_lut_{n}"] = {"lookups_per_s": n / t, "ms": t * 1e3, "key_bytes_per_lookup": kb / n,
                                  "gbs": alg / t / 1e9, "hbm_frac": alg / t / 1e9 / hbm}
    return res


def run_tt(ddg, torch, a):
    """Both parties of one truth-table gate on cuda:0 (ddg_gate_eval_pair: every
    AND-tree level, the openings in place, round 2): the full-compare ReLU and
    ReLU-ARS gates and the truncation carry, n = 2^k elements."""
    hbm, _, src = peaks()
    res = {"hbm_peak_gbs": hbm, "peak_source": src}
    st = torch.cuda.current_stream().cuda_stream
    for bw in a.bw:
        dt = torch.int32 if bw == 32 else torch.int64
        for kind, name in ((ddg.GATE_RELU_TTF, "relu_ttf"), (ddg.GATE_RELU_ARS_TTF, "relu_ars_ttf"),
                           (ddg.GATE_LRS_TT, "lrs_tt")):
            for lg in a.sizes:
                N = 1 << lg
                kb = ddg.gate_key_bytes(kind, bw, 12, N)
                if 2 * kb + 64 * N > 0.8 * torch.cuda.mem_get_info()[0]:
                    res[f"bw{bw}_{name}_2^{lg}"] = "skipped: keys do not fit"
                    continue
                k0 = torch.empty(kb, dtype=torch.uint8, device="cuda")
                k1 = torch.empty(kb, dtype=torch.uint8, device="cuda")
                g = torch.Generator(device="cuda").manual_seed(lg + bw)
                info = torch.iinfo(dt)
                r = torch.randint(info.min, info.max, (N,), dtype=dt, device="cuda", generator=g)
                x = torch.randint(info.min, info.max, (N,), dtype=dt, device="cuda", generator=g)
                if kind == ddg.GATE_LRS_TT:
                    x = x & info.max  # LRS precondition: x in [0, 2^(bw-1))
                ro = torch.empty_like(r)
                ddg.gate_keygen(kind, bw, 12, N, 1, 1, r.data_ptr(), ro.data_ptr(), k0.data_ptr(), k1.data_ptr(), st)
                xh = x + r
                words = (N + 31) // 32
                nb = ddg.gate_round1_arrays(kind, bw, 12)
                bits = [torch.empty(nb * words, dtype=torch.int32, device="cuda") for _ in range(2)]
                sh = [torch.empty_like(r) for _ in range(2)]
                t = timeit(torch, lambda: ddg.gate_eval_pair(kind, bw, 12, N, xh.data_ptr(), k0.data_ptr(),
                                                             k1.data_ptr(), bits[0].data_ptr(), bits[1].data_ptr(),
                                                             sh[0].data_ptr(), sh[1].data_ptr(), st))
                lay = ddg.tt_key_layout(kind, bw, 12, N)
                res[f"bw{bw}_{name}_2^{lg}"] = {
                    "elements_per_s": N / t, "ms": t * 1e3, "key_bytes_per_element_per_party": kb / N,
                    "levels": lay["levels"], "key_gbs_both_parties": 2 * kb / t / 1e9,
                    "key_hbm_frac": 2 * kb / t / 1e9 / hbm}
                del k0, k1, r, x, xh, ro, bits, sh
                torch.cuda.empty_cache()
    return res


def run_gemm(ddg, torch, a):
    hbm, bf16, src = peaks()
    L = ddg.lib()
    B = a.batch
    res = {"hbm_peak_gbs": hbm, "bf16_peak_tflops": bf16, "peak_source": src, "batch": B}
    st = torch.cuda.current_stream().cuda_stream
    for bw in (32, 64):
        dt = torch.int32 if bw == 32 else torch.int64
        info = torch.iinfo(dt)
        g = torch.Generator(device="cuda").manual_seed(bw)

        def rnd(*shape):
            return torch.randint(info.min, info.max, shape, dtype=dt, device="cuda", generator=g)

        P = bw // 8
        limb_products = P * (P + 1) // 2
        # FC: (B*138 x 282) . (282 x 376) + bias + key words (party 0)
        M, K, N = B * 138, 282, 376
        x, W, b2s, c, out = rnd(M, K), rnd(K, N), rnd(N), rnd(M, N), rnd(M, N)
        # Beaver: per sample (138 x 138) . (138 x 282), both products
        Ah, Hh, mA, mH, Z, s = rnd(B, 138, 138), rnd(B, 138, 282), rnd(B, 138, 138), rnd(B, 138, 282), \
            rnd(B, 138, 282), rnd(B, 138, 282)
        for path, pname in ((ddg.GEMM_TENSOR, "tensor"), (ddg.GEMM_TENSOR_WIDE, "tensor_wide"),
                            (ddg.GEMM_CUDA_CORES, "cuda_cores")):
            ddg.gemm_path(path)
            t = timeit(torch, lambda: ddg.check(L.ddg_fc_share(bw, 0, M, K, N, x.data_ptr(), W.data_ptr(),
                                                               b2s.data_ptr(), c.data_ptr(), out.data_ptr(), st)))
            mac = M * K * N
            alg = (M * K + K * N + N + 2 * M * N) * P
            res[f"bw{bw}_fc_{pname}"] = {"ms": t * 1e3, "ring_tmac_per_s": mac / t / 1e12,
                                         "int8_tops": 2 * mac * limb_products / t / 1e12, "gbs": alg / t / 1e9,
                                         "hbm_frac": alg / t / 1e9 / hbm}
            t = timeit(torch, lambda: ddg.check(L.ddg_matmul_share(bw, 0, B, 138, 138, 282, Ah.data_ptr(),
                                                                   Hh.data_ptr(), mA.data_ptr(), mH.data_ptr(),
                                                                   Z.data_ptr(), s.data_ptr(), st)))
            mac = 2 * B * 138 * 138 * 282
            alg = (2 * B * 138 * 138 + 4 * B * 138 * 282) * P
            res[f"bw{bw}_beaver_{pname}"] = {"ms": t * 1e3, "ring_tmac_per_s": mac / t / 1e12,
                                             "int8_tops": 2 * mac * limb_products / t / 1e12, "gbs": alg / t / 1e9,
                                             "hbm_frac": alg / t / 1e9 / hbm}
        ddg.gemm_path(ddg.GEMM_TENSOR)
        ddg.gemm_status()
    return res


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("what", choices=["dcf", "lut", "gemm", "aes", "tt"])
    ap.add_argument("--sizes", type=int, nargs="+", default=[20, 22, 24, 26])
    ap.add_argument("--bw", type=int, nargs="+", default=[32, 64])
    ap.add_argument("--n", type=int, default=1 << 20)
    ap.add_argument("--batch", type=int, default=256)
    a = ap.parse_args()
    import torch

    ddg = importlib.import_module("idash26-track3_b200")
    torch.cuda.set_device(0)
    if a.what == "dcf":
        res = run_dcf(ddg, torch, a)
    elif a.what == "lut":
        res = run_lut(ddg, torch, a)
    elif a.what == "tt":
        res = run_tt(ddg, torch, a)
    elif a.what == "gemm":
        res = run_gemm(ddg, torch, a)
    else:
        res = {"aes_2tables_gblocks": aes_ceiling(ddg, torch, 2), "aes_4tables_gblocks": aes_ceiling(ddg, torch, 4)}
    print(json.dumps({"microbench": a.what, **res}))


if __name__ == "__main__":
    main()
