"""The offline tools in C++ (idash26-track3_b200/cli): ddg_export_weights
writes the weights.bin blob and JSON manifest byte for byte as the Python
writer (restating reference/export_weights.py:38-75), and ddg_share writes
share files whose pairs reconstruct exactly the fixed-point values of the
Python sharer (reference/share_data.py:39-79, 135-159), with the protein
vectors byte-identical.  No GPU needed."""
import os
import subprocess

import numpy as np
import pytest

S = 12


@pytest.fixture(scope="module")
def tools(ddg):
    b = __import__("importlib").import_module("idash26-track3_b200.build")
    return dict(zip(b.TOOLS, b.build_tools()))


def test_export_weights_matches_python_writer(tools, synth, tmp_path):
    layers = synth.affinity_weights(5)
    raw = np.concatenate([np.concatenate([np.asarray(W, "<f4").ravel(), np.asarray(b, "<f4").ravel()])
                          for W, b in layers])
    raw.tofile(tmp_path / "w.f32")
    r = subprocess.run([tools["ddg_export_weights"], str(S), str(tmp_path / "w.f32"), str(tmp_path / "c.bin")],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    synth.write_weights(str(tmp_path / "py.bin"), synth.quantize_weights(layers, S), S)
    assert (tmp_path / "c.bin").read_bytes() == (tmp_path / "py.bin").read_bytes()
    assert (tmp_path / "c.bin.json").read_text() == (tmp_path / "py.bin.json").read_text()
    # a wrong-size input is refused
    (tmp_path / "short.f32").write_bytes(raw.tobytes()[:-4])
    r = subprocess.run([tools["ddg_export_weights"], str(S), str(tmp_path / "short.f32"), str(tmp_path / "x.bin")],
                       capture_output=True, text=True)
    assert r.returncode == 2


@pytest.mark.parametrize("bw", [32, 64])
def test_share_reconstructs_python_fixed_point(tools, synth, tmp_path, bw):
    B = 3
    inp = synth.Inputs(B, bw, seed=44, with_protein_cnn=False)
    src = tmp_path / "plain"
    src.mkdir()
    for name, a in (("x", inp.X_float), ("adj", inp.A_raw), ("mask", inp.mask), ("protein", inp.protein_float)):
        np.asarray(a, "<f8").tofile(src / f"{name}.f64")
    out = tmp_path / "shares"
    r = subprocess.run([tools["ddg_share"], str(bw), str(S), "77", str(src), str(out)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    dt = "<u4" if bw == 32 else "<u8"
    for name, want in (("x", inp.x_ring), ("adj", inp.adj_ring), ("mask", inp.mask_ring)):
        s0 = np.fromfile(out / f"{name}_share0.dat", dt)
        s1 = np.fromfile(out / f"{name}_share1.dat", dt)
        assert s0.size == s1.size == np.asarray(want).size
        assert np.array_equal((s0 + s1).astype(dt), np.asarray(want, dt).ravel()), name
        assert np.count_nonzero(s0) > 0.99 * s0.size  # pads, not the values
    inp.write(str(tmp_path / "py"))
    assert (out / "protein_emb.dat").read_bytes() == (tmp_path / "py" / "protein_emb.dat").read_bytes()
    # a different seed gives different pads, the same sums
    out2 = tmp_path / "shares2"
    subprocess.run([tools["ddg_share"], str(bw), str(S), "78", str(src), str(out2)], check=True, capture_output=True)
    a0, b0 = np.fromfile(out / "x_share0.dat", dt), np.fromfile(out2 / "x_share0.dat", dt)
    assert not np.array_equal(a0, b0)
    assert np.array_equal((b0 + np.fromfile(out2 / "x_share1.dat", dt)).astype(dt), np.asarray(inp.x_ring, dt).ravel())
