"""Shared test helpers: golden-fixture loading and ulp comparisons."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"


def load_golden(name: str) -> dict:
    """Load ``tests/golden/<name>.npz``; int16 arrays saved with a ``__bf16``
    suffix come back as bfloat16 tensors, other arrays as tensors (numeric)
    or numpy arrays (strings)."""
    out = {}
    with np.load(GOLDEN / f"{name}.npz") as z:
        for key in z.files:
            arr = z[key]
            if key.endswith("__bf16"):
                out[key[: -len("__bf16")]] = torch.from_numpy(arr.copy()).view(torch.bfloat16)
            elif arr.dtype.kind in "biuf" and arr.ndim > 0:
                out[key] = torch.from_numpy(arr.copy())
            elif arr.dtype.kind in "biuf":
                out[key] = arr.item()
            else:
                out[key] = arr
    return out


def _ordered_int(x: torch.Tensor) -> torch.Tensor:
    """Map floats to integers whose order and spacing follow the float's ulps."""
    if x.dtype == torch.float32:
        i = x.contiguous().view(torch.int32).to(torch.int64)
        return torch.where(i < 0, -(i & 0x7FFFFFFF), i)
    if x.dtype in (torch.bfloat16, torch.float16):
        i = x.contiguous().view(torch.int16).to(torch.int64)
        return torch.where(i < 0, -(i & 0x7FFF), i)
    raise TypeError(x.dtype)


def max_ulp_diff(a: torch.Tensor, b: torch.Tensor) -> int:
    """Largest distance in units in the last place between two same-dtype tensors."""
    assert a.dtype == b.dtype and a.shape == b.shape, (a.dtype, b.dtype, a.shape, b.shape)
    if a.numel() == 0:
        return 0
    return int((_ordered_int(a.cpu()) - _ordered_int(b.cpu())).abs().max())


def assert_rope_close(actual: torch.Tensor, expected: torch.Tensor) -> None:
    """RoPE-corrected K parity: fp32 within 1e-5 relative (1e-6 absolute floor);
    bf16 / fp16 within 1 ulp of the element type."""
    actual, expected = actual.cpu(), expected.cpu()
    assert actual.dtype == expected.dtype and actual.shape == expected.shape
    if actual.dtype == torch.float32:
        torch.testing.assert_close(actual, expected, rtol=1e-5, atol=1e-6)
    else:
        d = max_ulp_diff(actual, expected)
        assert d <= 1, f"max ulp difference {d} > 1"
