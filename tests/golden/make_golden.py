"""Generate tests/golden/*.npz from the reference's own Python code.

Runs only where the reference checkout is importable (pass its root as argv[1]
or set DDG_REFERENCE_ROOT); the committed .npz files are what the tests read.

What is pinned
--------------
ff_golden.npz: for bw in {32, 64} and 16 seeded synthetic drug graphs each,
the outputs of the reference's plaintext fixed-point model
``reference.fixed_forward.FixedAffinity`` (``_drug_path_fx`` -> PMVO(128) and
``_fusion_fx`` -> affinity at scale 12) on weights from
``reference.affinity_model.AffinityModel.from_random(94, seed)`` and the
model's own random gated-CNN protein vector.  Also checks that this build's
seeded weight generator (idash26-track3_b200/synth.py) draws exactly the
reference's float weights and that its gated CNN reproduces the reference's
protein vector.

The reference featuriser imports RDKit at module load; RDKit is absent, so a
minimal stand-in module providing only the names dense_graph.py touches at
import time is installed first (the array API used here never calls RDKit).
"""
from __future__ import annotations

import importlib
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def _install_rdkit_stub():
    rd = types.ModuleType("rdkit")
    chem = types.ModuleType("rdkit.Chem")
    hyb = types.SimpleNamespace(SP=1, SP2=2, SP3=3, SP3D=4, SP3D2=5)
    chem.rdchem = types.SimpleNamespace(HybridizationType=hyb)
    chem.MolFromSmiles = lambda s: None
    rd.Chem = chem
    sys.modules.setdefault("rdkit", rd)
    sys.modules.setdefault("rdkit.Chem", chem)


def main(ref_root: str):
    import torch

    _install_rdkit_stub()
    sys.path.insert(0, ref_root)
    sys.path.insert(0, REPO)
    from reference.affinity_model import AffinityModel
    from reference.fixed_forward import FixedAffinity

    synth = importlib.import_module("idash26-track3_b200.synth")

    out = {}
    B = 16
    for bw in (32, 64):
        seed = 11 if bw == 32 else 12
        torch.manual_seed(seed)
        model = AffinityModel.from_random(feat_dim=94, seed=seed)
        mine = synth.affinity_weights(seed)
        ref_layers = list(model.gcn) + list(model.drug_fc) + list(model.fusion)
        for (Wm, bm), (Wr, br) in zip(mine, ref_layers):
            assert np.array_equal(Wm, Wr) and np.array_equal(bm, br), "weight generator drifted"
        fm = FixedAffinity(model, scale=12, bw=bw)
        X, A_raw, mask = synth.gen_batch(B, seed=1000 + bw)
        A_hat = synth.normalized_adjacency(A_raw)
        rng = np.random.default_rng(seed + 7)
        seqs = [synth.random_protein(rng) for _ in range(B)]
        pmvo, aff, pvec = [], [], []
        for b in range(B):
            pv_fx = fm._protein_vec_fx(seqs[b])
            with torch.no_grad():
                enc = torch.tensor(synth.encode_protein(seqs[b]), dtype=torch.long).unsqueeze(0)
                pv = model.gated(enc).numpy().squeeze(0).astype(np.float64)
            p = fm._drug_path_fx(X[b], A_hat[b], mask[b])
            o = fm._fusion_fx(p, pv_fx)
            pmvo.append(np.asarray(p, np.int64))
            aff.append(np.asarray(o, np.int64))
            pvec.append(pv)
        mine_pv = synth.protein_vectors(seqs, seed)
        assert np.allclose(mine_pv, np.stack(pvec), atol=1e-6), "gated CNN drifted"
        out[f"bw{bw}_seed"] = np.array(seed)
        out[f"bw{bw}_X"] = X
        out[f"bw{bw}_A_raw"] = A_raw.astype(np.uint8)
        out[f"bw{bw}_mask"] = mask.astype(np.uint8)
        out[f"bw{bw}_pvec"] = np.stack(pvec)
        out[f"bw{bw}_pmvo"] = np.stack(pmvo)
        out[f"bw{bw}_out"] = np.stack(aff).reshape(B)
    np.savez_compressed(os.path.join(HERE, "ff_golden.npz"), **out)
    print("wrote", os.path.join(HERE, "ff_golden.npz"))


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("DDG_REFERENCE_ROOT", "")
    if not root or not os.path.isdir(os.path.join(root, "reference")):
        sys.exit("usage: make_golden.py <reference checkout root>")
    main(root)
