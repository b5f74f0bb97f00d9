"""The word-parallel AND-tree levels of the truth-table gates, on the CPU.

The level kernel compiled for (bw, scale) = (32, 12) and (64, 12) closes and
opens every AND of a level with word-wide operations on a lane layout
(idash26-track3_b200/csrc/tt_lanes.cuh).  tests/tt_lanes_check.cpp plays the
whole tree for both parties on random shared digit bits and dealer triples and
compares the reconstructed roots with the plaintext radix comparison; this test
compiles it with the host C++ compiler and runs it.  The GPU tests
(tests/test_tt_gpu.py) then check the kernels against the oracle's keys.
"""
import os
import shutil
import subprocess

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "..", "idash26-track3_b200", "csrc")


def _cuda_include():
    for d in (os.environ.get("CUDA_HOME", ""), "/usr/local/cuda"):
        if d and os.path.exists(os.path.join(d, "include", "cuda_runtime.h")):
            return os.path.join(d, "include")
    return None


def test_lane_levels_reconstruct_the_plaintext_comparison(tmp_path):
    cxx = shutil.which("g++") or shutil.which("c++")
    inc = _cuda_include()
    if cxx is None or inc is None:
        pytest.skip("needs a host C++ compiler and the CUDA headers")
    exe = tmp_path / "tt_lanes_check"
    subprocess.run([cxx, "-std=c++17", "-O2", "-I", CSRC, "-I", inc, os.path.join(HERE, "tt_lanes_check.cpp"), "-o",
                    str(exe)], check=True, capture_output=True, text=True)
    r = subprocess.run([str(exe), "5000"], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout + r.stderr
    # the CUDA plan places every triple bit where the C oracle's keygen puts it
    from oracle import fss_ref as F

    mode_kind = {1: F.GATE_RELU_TT, 2: F.GATE_LRS_TT, 3: F.GATE_RELU_TTF}
    seen = 0
    for line in r.stdout.splitlines():
        if not line.startswith("positions"):
            continue
        head, vals = line.split(":")
        _, _, mode, _, bw, _, packed = head.split()
        v = [int(x) for x in vals.split()]
        want = F.tt_tri_positions(mode_kind[int(mode)], int(bw), 12)
        got_pairs = v[:-1]
        assert got_pairs[0::2] == want["tpa"] and got_pairs[1::2] == want["tpc"], (line, want)
        if int(mode) == 3:
            assert v[-1] == want["mu"], (line, want)
        if int(bw) == 32:
            assert packed == "1", line  # the benchmarked plans group their triple bits by level
        seen += 1
    assert seen == 6
    # every scale of both ring widths: the same plans exist on both sides and
    # every triple bit sits where the oracle's keygen puts it (the runtime-plan
    # kernel and the keygen of other scales follow the same placement)
    checked = 0
    for line in r.stdout.splitlines():
        if not line.startswith("allpos"):
            continue
        head, vals = line.split(":")
        _, mode, bw, sc, ok, packed = head.split()
        mode, bw, sc, ok = int(mode), int(bw), int(sc), int(ok)
        try:
            want = F.tt_tri_positions(mode_kind[mode], bw, sc)
        except ValueError:
            want = None
        assert (want is not None) == bool(ok), line
        if want is None:
            continue
        v = [int(x) for x in vals.split()]
        assert v[:-1][0::2] == want["tpa"] and v[:-1][1::2] == want["tpc"], (line, want)
        if mode == 3:
            assert v[-1] == want["mu"], (line, want)
        checked += 1
    assert checked > 200, checked
