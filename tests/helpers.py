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


def pair_norm(x: torch.Tensor, style: str) -> torch.Tensor:
    """Per-element magnitude of the RoPE pair each element belongs to
    (interleaved pairs (2i, 2i+1) or neox pairs (i, i + D/2)); a rotation
    preserves it, so it is the scale the rounding error is measured on."""
    x = x.float()
    d = x.shape[-1]
    if style == "neox":
        a, b = x[..., : d // 2], x[..., d // 2 :]
        n = torch.sqrt(a * a + b * b)
        return torch.cat([n, n], dim=-1)
    a, b = x[..., 0::2], x[..., 1::2]
    n = torch.sqrt(a * a + b * b)
    return torch.stack([n, n], dim=-1).reshape(x.shape)


_MANT_BITS = {torch.float32: 23, torch.bfloat16: 7, torch.float16: 10}


def assert_rope_close(actual: torch.Tensor, expected: torch.Tensor, style: str = "interleaved") -> None:
    """RoPE-corrected K parity.

    bf16 / fp16: every element within 1 ulp of the element type, the ulp
    taken at the magnitude of the element's RoPE pair (the rotation's scale;
    near-zero outputs from cancellation are judged at that scale, not their
    own).  fp32: within 1e-5 relative to the pair magnitude.
    """
    actual, expected = actual.cpu(), expected.cpu()
    assert actual.dtype == expected.dtype and actual.shape == expected.shape
    if actual.numel() == 0:
        return
    diff = (actual.float() - expected.float()).abs()
    scale = torch.maximum(pair_norm(expected, style), pair_norm(actual, style))
    if actual.dtype == torch.float32:
        tol = 1e-5 * scale + 1e-30
    else:
        e = torch.floor(torch.log2(scale.clamp_min(1e-30)))
        tol = torch.exp2(e - _MANT_BITS[actual.dtype])
    bad = diff > tol
    assert not bad.any(), (
        f"{int(bad.sum())} elements outside tolerance; worst diff {float(diff.max()):.3e}, "
        f"at scale {float(scale.flatten()[int(torch.argmax((diff / tol).flatten()))]):.3e}"
    )
