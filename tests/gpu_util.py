"""Helpers for GPU tests: column-major FP64 matrices in CUDA memory."""
import numpy as np
import torch


def to_dev(a: np.ndarray, ld: int | None = None) -> tuple[torch.Tensor, int]:
    """numpy (m, n) -> CUDA buffer holding the column-major matrix, leading dimension ld."""
    a = np.asarray(a, dtype=np.float64)
    m, n = a.shape
    ld = m if ld is None else ld
    host = np.zeros((n, ld), dtype=np.float64)
    host[:, :m] = a.T
    return torch.from_numpy(host).cuda(), ld


def from_dev(t: torch.Tensor, m: int, n: int) -> np.ndarray:
    """CUDA column-major buffer -> numpy (m, n)."""
    return t.cpu().numpy().T[:m, :n].copy()


def round_up(x: int, a: int) -> int:
    return (x + a - 1) // a * a


def empty_bytes(nbytes: int) -> torch.Tensor:
    return torch.empty(max(nbytes, 16), dtype=torch.uint8, device="cuda")
