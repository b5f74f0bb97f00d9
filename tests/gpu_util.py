"""Device-buffer helpers shared by the GPU tests (torch is only the allocator)."""
import numpy as np
import torch


def dev_bytes(nbytes: int) -> torch.Tensor:
    return torch.zeros(max(int(nbytes), 16), dtype=torch.uint8, device="cuda")


def to_dev(arr: np.ndarray) -> torch.Tensor:
    a = np.ascontiguousarray(arr)
    return torch.from_numpy(a.view(np.uint8).copy()).to("cuda")


def from_dev(t: torch.Tensor, dtype, count: int | None = None) -> np.ndarray:
    a = t.cpu().numpy().view(dtype)
    return a if count is None else a[:count]


def ptr(t: torch.Tensor) -> int:
    return t.data_ptr()


def ring_dt(bw: int):
    return np.uint32 if bw == 32 else np.uint64
