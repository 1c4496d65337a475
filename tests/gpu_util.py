"""Helpers shared by the GPU tests (no test functions here)."""
from __future__ import annotations

import numpy as np
import torch

TOL = 1e-2  # |gpu - oracle| <= TOL + TOL * |oracle| for fp16 float ops (the stated tolerance)


def dev(a, dtype=torch.float16, device="cuda:0") -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).to(device=device, dtype=dtype)


def host(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def bits16(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def f16r(a) -> np.ndarray:
    return np.asarray(a, dtype=np.float32).astype(np.float16).astype(np.float32)


def assert_tol(actual, expected, tol: float = TOL, what: str = "") -> None:
    actual = np.asarray(actual, dtype=np.float64)
    expected = np.asarray(expected, dtype=np.float64)
    assert actual.shape == expected.shape, (actual.shape, expected.shape)
    err = np.abs(actual - expected)
    bad = err > tol + tol * np.abs(expected)
    assert not bad.any(), (f"{what}: {int(bad.sum())}/{bad.size} outside tolerance, "
                           f"max abs err {err.max():.3g} at {np.unravel_index(err.argmax(), err.shape)}")


def padded(n: int, dtype, canary: float = -1234.0, pad: int = 64, device="cuda:0"):
    """A buffer of n elements followed by `pad` canary elements; returns
    (whole, view_of_first_n)."""
    whole = torch.full((n + pad,), canary, dtype=dtype, device=device)
    return whole, whole[:n]


def canary_intact(whole: torch.Tensor, n: int, canary: float = -1234.0) -> bool:
    return bool((whole[n:].float() == canary).all().item())
