"""The C-ABI library loads and exports every function include/ddg_fss.h declares (no GPU needed)."""
import os
import ctypes
import re

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    src = open(os.path.join(REPO, "include", "ddg_fss.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(ddg_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_functions():
    assert "ddg_gate_round1" in declared_functions()


def test_library_exports_every_declared_symbol(ddg):
    L = ddg.lib()
    missing = [f for f in declared_functions() if not hasattr(L, f)]
    assert not missing, missing
    assert set(declared_functions()) <= set(ddg.SIGNATURES), "python signature table incomplete"


def test_argument_errors_are_status_codes(ddg):
    with pytest.raises(ddg.DdgError) as e:
        ddg.gate_round1(9, 32, 12, 10, None, None, None, None)
    assert e.value.code == 1
    with pytest.raises(ddg.DdgError):
        ddg.gate_round2(0, 48, 12, 10, 0, None, None, None, None, None, None, None)
    assert ddg.gate_key_bytes(0, 32, 12, 1000) > 1000 * 400


def test_split_lrs_layout(ddg):
    """The split-carry LRS gate: a 5-bit DCF with equality output over carry
    bits 7..11 and a 7-bit DCF over bits 0..6, both leaf-only (no tree
    levels), 7 key words; smaller keys than the single 12-bit DCF."""
    lay = ddg.gate_key_layout(ddg.GATE_LRS_SPLIT, 32, 12, 1000)
    assert (lay["hi_bits"], lay["hi_shift"], lay["lo_bits"]) == (5, 7, 7)
    assert lay["hi_levels"] == 0 and lay["lo_levels"] == 0 and lay["hi_mu_eq"] > 0
    assert ddg.gate_key_bytes(ddg.GATE_LRS_SPLIT, 32, 12, 1 << 16) < ddg.gate_key_bytes(ddg.GATE_LRS, 32, 12, 1 << 16)
    with pytest.raises(ddg.DdgError):
        ddg.gate_key_layout(ddg.GATE_LRS_SPLIT, 32, 1, 10)
    with pytest.raises(ddg.DdgError):
        ddg.gate_key_layout(ddg.GATE_RELU_ARS_TTF + 1, 32, 12, 10)


def test_ot_gate_layout(ddg):
    """OT-leaf ReLU kinds: 44 round keys, one receiver byte per digit slot,
    party 0's c word, then the SPLIT kind's 16 / 32 words.  bw=32, scale 12:
    19 + 12 bits in 5 + 3 radix-16 digits, 4 garbled by each party, 3 AND
    levels, 6 combines; bw=64: 13 + 3 digits, 4 levels, 14 combines."""
    from oracle import fss_ref as F

    for bw, plan in ((32, (8, 4, 3, 6)), (64, (16, 8, 4, 14))):
        for kind, words in ((ddg.GATE_RELU_OT, 16), (ddg.GATE_RELU_ARS_OT, 32)):
            n = 1000
            lay = ddg.ot_key_layout(kind, bw, 12, n)
            assert (lay["digits"], lay["g0"], lay["levels"], lay["combines"]) == plan
            info = F.ot_plan_info(bw, 12)
            assert (info["digits"], info["g0"], info["levels"], info["combines"]) == plan
            assert lay["ks"] == 0 and lay["recv"] >= 176 and lay["c0"] >= lay["recv"] + lay["slots"] * n
            assert lay["words"] >= lay["c0"] + 4 * n
            assert lay["bytes"] == ddg.gate_key_bytes(kind, bw, 12, n) >= lay["words"] + words * (bw // 8) * n
            # smaller keys than any DCF form of the same function
            split = ddg.GATE_RELU_SPLIT if kind == ddg.GATE_RELU_OT else ddg.GATE_RELU_ARS_SPLIT
            assert lay["bytes"] < ddg.gate_key_bytes(split, bw, 12, n)
        assert ddg.gate_round1_arrays(ddg.GATE_RELU_OT, bw, 12) == 3
    with pytest.raises(ddg.DdgError) as e:  # the interactive kinds have no one-shot round 1
        ddg.gate_round1(ddg.GATE_RELU_OT, 32, 12, 10, 1, 1, 1, 1)
    assert e.value.code == 1
    with pytest.raises(ddg.DdgError):
        ddg.ot_key_layout(ddg.GATE_RELU_SPLIT, 32, 12, 10)


def test_tt_gate_layout(ddg):
    """Truth-table kinds: digit tables (ReLU at bw=32: 4 hi digits of 5/5/5/4
    bits and 3 lo digits of 4, 10 rows; the carry: two 6-bit digits, 6 rows),
    one triple word, then the words of the SPLIT kind or of LRS; far smaller
    keys than the DCF kinds and no AES key."""
    from oracle import fss_ref as F

    cases = ((ddg.GATE_RELU_TT, 32, 10, 7, 2, 16), (ddg.GATE_RELU_ARS_TT, 32, 10, 7, 2, 32),
             (ddg.GATE_LRS_TT, 32, 6, 2, 1, 4), (ddg.GATE_RELU_ARS_TT, 64, 16, 16, 4, 32),
             (ddg.GATE_LRS_TT, 64, 6, 2, 1, 4))
    for kind, bw, rows, digits, levels, words in cases:
        n = 1000
        lay = ddg.tt_key_layout(kind, bw, 12, n)
        assert (lay["rows"], lay["digits"], lay["levels"]) == (rows, digits, levels)
        info = F.tt_plan_info(kind, bw, 12)
        assert (info["rows"], info["digits"], info["levels"]) == (rows, digits, levels)
        assert lay["tables"] == 0 and lay["tri"] >= 4 * rows * n and lay["words"] >= lay["tri"] + 4 * lay["tri_words"] * n
        assert lay["bytes"] == ddg.gate_key_bytes(kind, bw, 12, n) >= lay["words"] + words * (bw // 8) * n
    assert ddg.gate_key_bytes(ddg.GATE_RELU_ARS_TT, 32, 12, 1000) < ddg.gate_key_bytes(ddg.GATE_RELU_ARS_SPLIT3, 32,
                                                                                        12, 1000) / 3
    assert ddg.gate_key_bytes(ddg.GATE_LRS_TT, 32, 12, 1000) < ddg.gate_key_bytes(ddg.GATE_LRS_SPLIT, 32, 12, 1000)
    assert ddg.gate_round1_arrays(ddg.GATE_LRS_TT, 32, 12) == 1 and ddg.gate_round1_arrays(ddg.GATE_RELU_TT, 32, 12) == 3
    # the full-compare kinds: one more AND level, two opened arrays, the words of RELU / RELU_ARS
    for kind, words in ((ddg.GATE_RELU_TTF, 4), (ddg.GATE_RELU_ARS_TTF, 8)):
        lay = ddg.tt_key_layout(kind, 32, 12, 1000)
        assert (lay["rows"], lay["digits"], lay["levels"]) == (10, 7, 3)
        assert lay["bytes"] >= lay["words"] + words * 4 * 1000 and ddg.gate_round1_arrays(kind, 32, 12) == 2
        assert F.tt_plan_info(kind, 32, 12)["levels"] == 3
    assert ddg.gate_key_bytes(ddg.GATE_RELU_ARS_TTF, 32, 12, 1000) < ddg.gate_key_bytes(ddg.GATE_RELU_ARS_TT, 32, 12,
                                                                                         1000) / 2
    with pytest.raises(ddg.DdgError) as e:
        ddg.gate_round1(ddg.GATE_RELU_TT, 32, 12, 10, 1, 1, 1, 1)
    assert e.value.code == 1


def test_three_part_split_layout(ddg):
    """Three-part split ReLU at bw=32, scale 12: a 13-bit DCF with equality
    (7 levels) over bits 18..30, a 6-bit one (leaf only) over bits 12..17 and
    the 12-bit DCF (5 levels); 15 AES per element in all."""
    for kind, words in ((ddg.GATE_RELU_SPLIT3, 40), (ddg.GATE_RELU_ARS_SPLIT3, 80)):
        lay = ddg.gate_key_layout(kind, 32, 12, 1000)
        assert (lay["hi_bits"], lay["hi_shift"], lay["hi_levels"]) == (13, 18, 7)
        assert lay["mid_levels"] == 0 and lay["mid_mu_eq"] > lay["mid_mu"] > lay["mid_root"] > lay["hi_mu_eq"]
        assert (lay["lo_bits"], lay["lo_levels"]) == (12, 5) and lay["lo_root"] > lay["mid_mu_eq"]
        aes = lay["hi_levels"] + 1 + lay["mid_levels"] + 1 + lay["lo_levels"] + 1
        assert aes == 15
        assert lay["bytes"] - lay["words"] >= words * 4 * 1000
    with pytest.raises(ddg.DdgError):  # scale + 6 must stay below bw - 1
        ddg.gate_key_layout(ddg.GATE_RELU_SPLIT3, 32, 25, 10)


def test_layer_entry_points_reject_bad_arguments_without_a_gpu(ddg):
    """The per-layer interface checks its handles, cursor and wires before any
    device work: a null party, dealer or cursor is DDG_ERR_ARG."""
    L = ddg.lib()
    c = ddg.Cursor()
    w = ddg.Wire(None, 0, None)
    mw = ddg.MaskWire(None, 0, None, None)
    for st in (L.ddg_adjnorm_eval(None, c, 1, None, w), L.ddg_gcn_layer_eval(None, c, 0, 1, w, w, w),
               L.ddg_op_gate_eval(None, c, 0, w, w), L.ddg_maxpool_eval(None, c, 1, w, w),
               L.ddg_op_output_eval(None, c, 1, w, None, None), L.ddg_adjnorm_keygen(None, c, 1, mw),
               L.ddg_op_fc_keygen(None, c, 3, 1, 1, mw, mw), L.ddg_party_connect_callback(None, None)):
        assert st == 1
    assert L.ddg_dealer_destroy(None) == 0


def test_graph_and_pipeline_entry_points_reject_bad_arguments_without_a_gpu(ddg):
    """Forward graphs, queued replays and the forward pipeline check their
    handles before any device work: null handles are DDG_ERR_ARG, destroying
    a null handle is a no-op."""
    L = ddg.lib()
    out = ddg._vp()
    assert L.ddg_forward_graph_enqueue(None) == 1
    assert L.ddg_forward_graph_sync(None, None, None) == 1
    assert L.ddg_party_graph_create(None, 1, None, 0, ctypes.byref(out)) == 1
    assert L.ddg_forward_pipeline_create(None, None, 1, ctypes.byref(out)) == 1
    assert L.ddg_forward_pipeline_submit(None, None, None, None, None) == 1
    assert L.ddg_forward_pipeline_wait(None) == 1
    assert L.ddg_forward_pipeline_destroy(None) == 0
    assert L.ddg_forward_graph_destroy(None) == 0
