"""Seeded synthetic inputs and the offline file formats of the affinity branch.

The datasets (davis/kiba) and the trained checkpoints are not used; these
generators stand in for them with the shapes and value distributions of the
reference's offline pipeline:

* drug graphs: atom count ~ U[lo, hi], a random spanning tree (atom i bonds to
  one of atoms 0..i-1) plus 0-3 ring-closure bonds, dense 0/1 adjacency with
  self-loops on real atoms, zero-padded to nmax=138 (reference
  reference/dense_graph.py:109-119);
* node features: 94 columns laid out as the reference featuriser's one-hot
  blocks (reference/dense_graph.py:53-74: symbol 44+1, degree 11, #H 11+1,
  implicit valence 11+1, formal charge 5+1, hybridisation 5+1, aromatic,
  in-ring), L1-normalised per real atom;
* weights: the architecture of reference/affinity_model.py:75-86, drawn in
  the same order with the same N(0,1)*0.1 law so a seed gives the same
  float weights as ``AffinityModel.from_random``;
* protein: a seeded length-1000 sequence over the 25-letter alphabet encoded
  by a random-initialised gated CNN with the layer shapes of
  reference/affinity_model.py:34-56; its 128-d output is public.

File formats (reference/share_data.py:290-356, export_weights.py:38-75,
protein_plaintext.py:19-31, mpc_config.py:15-21): headerless little-endian
``<u4``/``<u8`` share files ``{x,adj,mask}_share{0,1}.dat``, ``protein_emb.dat``
and the int64 ``weights.bin`` blob ((in,out) row-major W then b per layer,
forward order) with its ``.json`` manifest.
"""
from __future__ import annotations

import json
import os

import numpy as np

NMAX = 138
FEAT = 94
POOL_DIM = 376
PROT_DIM = 128
SEQ_LEN = 1000
SEQ_ALPHABET = "ABCDEFGHIKLMNOPQRSTUVWXYZ"

# (name, in, out) in forward order -- reference gpu_mpc/deepdtagen_inference.cu:113-123
LAYERS = (
    ("gcn.0", 94, 188), ("gcn.1", 188, 282), ("gcn.2", 282, 376),
    ("drug_fc.0", 376, 1024), ("drug_fc.1", 1024, 128),
    ("fusion.0", 256, 1024), ("fusion.1", 1024, 512), ("fusion.2", 512, 256), ("fusion.3", 256, 1),
)

# one-hot block widths of the 94-wide feature row
_BLOCKS = (45, 11, 12, 12, 6, 6)


# ----------------------------------------------------------------- graphs

def gen_graph(rng: np.random.Generator, lo: int = 10, hi: int = 60, nmax: int = NMAX):
    """One molecule-shaped graph: (X (nmax,94) f32, A_raw (nmax,nmax) f32, mask (nmax,) f32)."""
    n = int(rng.integers(lo, hi + 1))
    A = np.zeros((nmax, nmax), dtype=np.float32)
    for i in range(1, n):
        j = int(rng.integers(0, i))
        A[i, j] = A[j, i] = 1.0
    ring = np.zeros(nmax, dtype=bool)
    for _ in range(int(rng.integers(0, 4))):
        for _try in range(20):
            a, b = (int(v) for v in rng.integers(0, n, size=2))
            if a != b and A[a, b] == 0:
                A[a, b] = A[b, a] = 1.0
                ring[a] = ring[b] = True
                break
    deg = A[:n, :n].sum(axis=1).astype(np.int64)
    for i in range(n):
        A[i, i] = 1.0
    X = np.zeros((nmax, FEAT), dtype=np.float32)
    sym_p = np.full(44, 0.1 / 41)
    sym_p[:3] = (0.6, 0.15, 0.15)
    for i in range(n):
        f = np.zeros(FEAT, dtype=np.float32)
        off = 0
        picks = (
            int(rng.choice(44, p=sym_p)),      # symbol
            min(int(deg[i]), 10),              # degree from the graph
            int(rng.integers(0, 4)),           # total #H
            int(rng.integers(0, 5)),           # implicit valence
            4,                                 # formal charge 0 (index of 0 in [-1,-2,1,2,0])
            int(rng.integers(0, 5)),           # hybridisation
        )
        for width, k in zip(_BLOCKS, picks):
            f[off + k] = 1.0
            off += width
        f[off] = float(rng.random() < 0.3)    # aromatic
        f[off + 1] = float(ring[i])           # in ring
        X[i] = f / f.sum()
    mask = np.zeros(nmax, dtype=np.float32)
    mask[:n] = 1.0
    return X, A, mask


def gen_batch(B: int, seed: int, atoms=(10, 60), nmax: int = NMAX):
    rng = np.random.default_rng(seed)
    Xs, As, Ms = [], [], []
    for _ in range(B):
        X, A, m = gen_graph(rng, atoms[0], atoms[1], nmax)
        Xs.append(X), As.append(A), Ms.append(m)
    return np.stack(Xs), np.stack(As), np.stack(Ms)


def normalized_adjacency(A_raw: np.ndarray) -> np.ndarray:
    """Float D^-1/2 (A+I) D^-1/2 over the real block (reference dense_graph.py:149-154)."""
    out = np.zeros_like(A_raw, dtype=np.float32)
    for b in range(A_raw.shape[0]):
        deg = A_raw[b].sum(axis=1)
        n = int((deg > 0).sum())
        sub = A_raw[b, :n, :n]
        dg = sub.sum(axis=1)
        dis = np.where(dg > 0, 1.0 / np.sqrt(dg), 0.0)
        out[b, :n, :n] = dis[:, None] * sub * dis[None, :]
    return out


# ----------------------------------------------------------------- weights

def affinity_weights(seed: int, feat: int = FEAT):
    """Nine (W (out,in) f32, b f32) pairs, drawn like AffinityModel.from_random."""
    rng = np.random.default_rng(seed)
    out = []
    for _, i, o in LAYERS:
        i = feat if i == 94 else i
        W = rng.standard_normal((o, i)).astype(np.float32) * 0.1
        b = rng.standard_normal(o).astype(np.float32) * 0.1
        out.append((W, b))
    return out


def quantize_weights(layers, scale: int = 12):
    """[(W_q (in,out) int64, b_q int64)] with np.rint, as export_weights.py:27-35."""
    q = []
    for W, b in layers:
        Wt = np.ascontiguousarray(np.asarray(W, np.float64).T)
        q.append((np.rint(Wt * (1 << scale)).astype(np.int64),
                  np.rint(np.asarray(b, np.float64) * (1 << scale)).astype(np.int64)))
    return q


def weights_blob(qlayers) -> np.ndarray:
    return np.concatenate([np.concatenate([W.ravel(), b.ravel()]) for W, b in qlayers]).astype("<i8")


def blob_to_layers(blob: np.ndarray):
    out, off = [], 0
    for _, i, o in LAYERS:
        W = blob[off:off + i * o].reshape(i, o).astype(np.int64)
        off += i * o
        b = blob[off:off + o].astype(np.int64)
        off += o
        out.append((W, b))
    if off != blob.size:
        raise ValueError(f"weights blob has {blob.size} int64 values, expected {off}")
    return out


def write_weights(path: str, qlayers, scale: int = 12) -> dict:
    blob = weights_blob(qlayers)
    blob.tofile(path)
    layers, off = [], 0
    for (name, i, o), (W, b) in zip(LAYERS, qlayers):
        layers.append({"name": name, "W_shape": [int(W.shape[0]), int(W.shape[1])], "b_shape": [int(b.size)],
                       "W_offset": off, "b_offset": off + W.size})
        off += W.size + b.size
    manifest = {"scale": int(scale), "bitwidth": 64, "total_elements": int(blob.size), "layers": layers}
    with open(path + ".json", "w") as f:
        json.dump(manifest, f, indent=2)
    return manifest


def read_weights(path: str):
    return blob_to_layers(np.fromfile(path, dtype="<i8"))


# ----------------------------------------------------------------- protein

def random_protein(rng: np.random.Generator, length: int = SEQ_LEN) -> str:
    return "".join(SEQ_ALPHABET[int(k)] for k in rng.integers(0, len(SEQ_ALPHABET), size=length))


def encode_protein(seq: str) -> np.ndarray:
    """Length-1000 token vector: letter k of the alphabet -> k+1, padding 0."""
    lut = {c: i + 1 for i, c in enumerate(SEQ_ALPHABET)}
    v = np.zeros(SEQ_LEN, dtype=np.int64)
    for i, ch in enumerate(seq[:SEQ_LEN]):
        v[i] = lut.get(ch, 0)
    return v


def gated_cnn(seed: int):
    """Random-initialised gated CNN protein encoder (torch, CPU, public)."""
    import torch
    import torch.nn as nn

    class _Gated(nn.Module):
        def __init__(self):
            super().__init__()
            self.embed = nn.Embedding(26, 128)
            self.conv = nn.ModuleList()
            self.gate = nn.ModuleList()
            for cin, cout in ((SEQ_LEN, 32), (32, 64), (64, 96)):
                self.conv.append(nn.Conv1d(cin, cout, 8))
                self.gate.append(nn.Conv1d(cin, cout, 8))
            self.fc = nn.Linear(96 * 107, PROT_DIM)

        def forward(self, tok):
            h = self.embed(tok)
            for c, g in zip(self.conv, self.gate):
                h = torch.relu(c(h) * torch.sigmoid(g(h)))
            return self.fc(h.reshape(h.shape[0], -1))

    torch.manual_seed(seed)
    return _Gated().eval()


def protein_vectors(seqs, seed: int) -> np.ndarray:
    import torch
    net = gated_cnn(seed)
    tok = torch.tensor(np.stack([encode_protein(s) for s in seqs]), dtype=torch.long)
    with torch.no_grad():
        return net(tok).numpy().astype(np.float64)


# ----------------------------------------------------------------- ring / shares

def ring_dtype(bw: int):
    return np.uint32 if bw == 32 else np.uint64


def to_ring(x, scale: int, bw: int) -> np.ndarray:
    """np.rint(x * 2^scale) reduced into Z_2^bw (share_data.py:297-308)."""
    fixed = np.rint(np.asarray(x, dtype=np.float64) * (1 << scale)).astype(np.int64)
    return fixed.astype(np.uint64).astype(ring_dtype(bw)) if bw == 32 else fixed.view(np.uint64)


def split_shares(ring_vals: np.ndarray, seed: int, bw: int):
    """share0 = uniform pad, share1 = value - pad (mod 2^bw) (share_data.py:311-334)."""
    dt = ring_dtype(bw)
    v = np.asarray(ring_vals, dtype=dt)
    pad = np.random.default_rng(seed).integers(0, np.iinfo(dt).max, size=v.shape, dtype=dt, endpoint=True)
    return pad, (v - pad).astype(dt)


class Inputs:
    """One micro-batch of secret-shared inputs for both parties plus its plaintext."""

    def __init__(self, B: int, bw: int, scale: int = 12, seed: int = 0, atoms=(10, 60), with_protein_cnn=True):
        self.B, self.bw, self.scale = B, bw, scale
        X, A, m = gen_batch(B, seed, atoms)
        self.X_float, self.A_raw, self.mask = X, A, m
        rng = np.random.default_rng(seed + 7)
        if with_protein_cnn:
            self.protein_float = protein_vectors([random_protein(rng) for _ in range(B)], seed)
        else:
            self.protein_float = rng.standard_normal((B, PROT_DIM)) * 0.05
        mask_tiled = np.broadcast_to(m[:, :, None], (B, NMAX, POOL_DIM))
        self.x_ring = to_ring(X, scale, bw)
        self.adj_ring = to_ring(A, 0, bw)
        self.mask_ring = to_ring(mask_tiled, scale, bw)
        self.protein_ring = to_ring(self.protein_float, scale, bw)
        self.x_sh = split_shares(self.x_ring, seed + 100, bw)
        self.adj_sh = split_shares(self.adj_ring, seed + 101, bw)
        self.mask_sh = split_shares(self.mask_ring, seed + 102, bw)
        zero = np.zeros_like(self.protein_ring)
        # protein: public value held by party 1, zeros on party 0
        # (reference deepdtagen_inference.cu:429-432)
        self.protein_sh = (zero, self.protein_ring.copy())

    def write(self, out_dir: str):
        os.makedirs(out_dir, exist_ok=True)
        dt = "<u4" if self.bw == 32 else "<u8"
        for name, sh in (("x", self.x_sh), ("adj", self.adj_sh), ("mask", self.mask_sh)):
            for p in (0, 1):
                np.asarray(sh[p]).astype(dt).tofile(os.path.join(out_dir, f"{name}_share{p}.dat"))
        self.protein_ring.astype(dt).tofile(os.path.join(out_dir, "protein_emb.dat"))
