"""GPU parity of partial-prefill attention against the CPU oracle and the
reference's golden fixtures.

Bar: bf16 / fp16 (tensor cores) within 2e-2 absolute of the fp32 oracle
computed from the same inputs; fp32 (CUDA cores) within the reference test's
1e-4 absolute / 1e-3 relative; rows outside the compute mask exactly zero.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from semblend_b200 import triton_kernels as tk
from tests.helpers import load_golden

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _spans_mask(S, n_spans, tail, frac, seed):
    """Seeded contiguous recompute spans plus the final `tail` tokens."""
    rng = np.random.default_rng(seed)
    mask = np.zeros(S, bool)
    mask[S - tail:] = True
    want = int(frac * S) - tail
    starts = np.sort(rng.choice(S - tail, n_spans, replace=False))
    lens = np.maximum(1, rng.multinomial(max(want, n_spans), np.ones(n_spans) / n_spans))
    for a, ln in zip(starts, lens):
        mask[a : min(a + ln, S - tail)] = True
    return torch.from_numpy(mask)


def _check_rows(out, q, k, v, mask, atol):
    """Compare every compute row against the fp32 blocked oracle, per batch."""
    B, Hq = q.shape[:2]
    for b in range(B):
        rows = torch.where(mask[b])[0]
        kk = oatt.expand_kv_heads(k[b].float().cpu(), Hq)
        vv = oatt.expand_kv_heads(v[b].float().cpu(), Hq)
        want = oatt.partial_prefill_attention_blocked(q[b].float().cpu(), kk, vv, rows)
        got = out[b][:, rows, :].float().cpu()
        torch.testing.assert_close(got, want, atol=atol, rtol=0)
        other = torch.ones(q.shape[2], dtype=torch.bool)
        other[rows] = False
        assert torch.all(out[b][:, other.to(out.device), :] == 0)


@pytest.mark.parametrize("name", ["attn_small", "attn_mid"])
def test_golden_fp32(name):
    g = load_golden(name)
    out = tk.partial_prefill_attention(g["q"].to(DEV), g["k"].to(DEV), g["v"].to(DEV), g["mask"].to(DEV))
    torch.testing.assert_close(out.cpu(), g["out"], atol=1e-4, rtol=1e-3)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("hq,hkv", [(4, 4), (28, 4), (16, 2)])
def test_tensor_core_vs_oracle(dtype, hq, hkv):
    g = torch.Generator().manual_seed(hq * 31 + hkv)
    B, S, D = 2, 1000, 128
    q = (torch.randn(B, hq, S, D, generator=g) / math.sqrt(D)).to(dtype)
    k = (torch.randn(B, hkv, S, D, generator=g) / math.sqrt(D)).to(dtype)
    v = torch.randn(B, hkv, S, D, generator=g).to(dtype)
    mask = torch.stack([_spans_mask(S, 8, 64, 0.2, 1), _spans_mask(S, 5, 37, 0.15, 2)])
    out = tk.partial_prefill_attention(q.to(DEV), k.to(DEV), v.to(DEV), mask.to(DEV))
    _check_rows(out, q, k, v, mask, atol=2e-2)


def test_reference_api_unbatched_bf16():
    g = torch.Generator().manual_seed(5)
    H, S, D = 8, 700, 128
    q = torch.randn(H, S, D, generator=g).to(torch.bfloat16)
    k = torch.randn(H, S, D, generator=g).to(torch.bfloat16)
    v = torch.randn(H, S, D, generator=g).to(torch.bfloat16)
    mask = torch.rand(S, generator=g) < 0.1
    mask[0] = True
    mask[-1] = True
    out = tk.partial_prefill_attention(q.to(DEV), k.to(DEV), v.to(DEV), mask.to(DEV))
    assert out.shape == (H, S, D) and out.dtype == torch.bfloat16
    _check_rows(out.unsqueeze(0), q.unsqueeze(0), k.unsqueeze(0), v.unsqueeze(0), mask.unsqueeze(0), 2e-2)


def test_edge_masks():
    g = torch.Generator().manual_seed(6)
    B, H, S, D = 3, 7, 300, 128
    q = torch.randn(B, H, S, D, generator=g).to(torch.bfloat16)
    k = torch.randn(B, 1, S, D, generator=g).to(torch.bfloat16)
    v = torch.randn(B, 1, S, D, generator=g).to(torch.bfloat16)
    mask = torch.zeros(B, S, dtype=torch.bool)
    mask[1, 0] = True  # a single row at position 0 (attends to itself only)
    mask[2, :] = True  # every row
    out = tk.partial_prefill_attention(q.to(DEV), k.to(DEV), v.to(DEV), mask.to(DEV))
    assert torch.all(out[0] == 0)  # batch element with no compute rows
    _check_rows(out, q, k, v, mask, atol=2e-2)
    torch.testing.assert_close(out[1, :, 0].float().cpu(), v[1, 0, 0].float().expand(H, D), atol=1e-2, rtol=0)


@pytest.mark.parametrize("D", [16, 64])
def test_other_head_dims_cuda_core(D):
    g = torch.Generator().manual_seed(D)
    B, Hq, Hkv, S = 1, 6, 3, 200
    q = torch.randn(B, Hq, S, D, generator=g).to(torch.bfloat16)
    k = torch.randn(B, Hkv, S, D, generator=g).to(torch.bfloat16)
    v = torch.randn(B, Hkv, S, D, generator=g).to(torch.bfloat16)
    mask = (torch.rand(B, S, generator=g) < 0.2)
    out = tk.partial_prefill_attention(q.to(DEV), k.to(DEV), v.to(DEV), mask.to(DEV))
    _check_rows(out, q, k, v, mask, atol=2e-2)


def test_fp32_matches_reference_math():
    g = torch.Generator().manual_seed(8)
    H, S, D = 3, 150, 32
    q, k, v = (torch.randn(H, S, D, generator=g) for _ in range(3))
    mask = torch.rand(S, generator=g) < 0.3
    want = oatt.partial_prefill_attention(q, k, v, mask)
    out = tk.partial_prefill_attention(q.to(DEV), k.to(DEV), v.to(DEV), mask.to(DEV))
    torch.testing.assert_close(out.cpu(), want, atol=1e-4, rtol=1e-3)


def test_long_context_rows_sample():
    """c4 geometry at S = 8192 (Qwen2.5-7B: 28 q heads, 4 KV heads): check a
    seeded sample of rows, including the final ones attending to every key."""
    g = torch.Generator().manual_seed(9)
    B, Hq, Hkv, S, D = 1, 28, 4, 8192, 128
    q = (torch.randn(B, Hq, S, D, generator=g) / math.sqrt(D)).to(torch.bfloat16)
    k = (torch.randn(B, Hkv, S, D, generator=g) / math.sqrt(D)).to(torch.bfloat16)
    v = (torch.randn(B, Hkv, S, D, generator=g) / math.sqrt(D)).to(torch.bfloat16)
    mask = _spans_mask(S, 64, 512, 0.10, 3).unsqueeze(0)
    out = tk.partial_prefill_attention(q.to(DEV), k.to(DEV), v.to(DEV), mask.to(DEV))
    rows = torch.where(mask[0])[0]
    pick = torch.cat([rows[:: max(1, rows.numel() // 40)], rows[-3:]]).unique()
    kk = oatt.expand_kv_heads(k[0].float(), Hq)
    vv = oatt.expand_kv_heads(v[0].float(), Hq)
    want = oatt.partial_prefill_attention_blocked(q[0].float(), kk, vv, pick)
    torch.testing.assert_close(out[0][:, pick.to(DEV), :].float().cpu(), want, atol=2e-2, rtol=0)


@pytest.mark.parametrize("scale", [-0.06, 0.4])
def test_tensor_core_negative_and_large_scale(scale):
    """A negative scale (row minimum becomes the reference) and a large one
    (logit spreads that force many rescales of the running output)."""
    g = torch.Generator().manual_seed(11)
    B, Hq, Hkv, S, D = 1, 8, 2, 900, 128
    q = torch.randn(B, Hq, S, D, generator=g).to(torch.bfloat16)
    k = torch.randn(B, Hkv, S, D, generator=g).to(torch.bfloat16)
    v = torch.randn(B, Hkv, S, D, generator=g).to(torch.bfloat16)
    mask = _spans_mask(S, 6, 40, 0.2, 4).unsqueeze(0)
    out = tk.partial_prefill_attention(q.to(DEV), k.to(DEV), v.to(DEV), mask.to(DEV), scale)
    rows = torch.where(mask[0])[0]
    kk = oatt.expand_kv_heads(k[0].float(), Hq)
    vv = oatt.expand_kv_heads(v[0].float(), Hq)
    want = oatt.partial_prefill_attention_blocked(q[0].float(), kk, vv, rows, scale=scale)
    torch.testing.assert_close(out[0][:, rows.to(DEV), :].float().cpu(), want, atol=2e-2, rtol=0)


@pytest.mark.parametrize("count", [1, 10, 18, 19, 36, 37])
def test_row_tile_pair_boundaries(count):
    """Row counts around the two-tile unit (G = 7 -> 18 rows per tile): second
    tile empty, partly filled, full, and a unit with a single row."""
    g = torch.Generator().manual_seed(count)
    B, Hq, Hkv, S, D = 1, 28, 4, 600, 128
    q = (torch.randn(B, Hq, S, D, generator=g) / math.sqrt(D)).to(torch.bfloat16)
    k = (torch.randn(B, Hkv, S, D, generator=g) / math.sqrt(D)).to(torch.bfloat16)
    v = torch.randn(B, Hkv, S, D, generator=g).to(torch.bfloat16)
    mask = torch.zeros(B, S, dtype=torch.bool)
    mask[0, torch.randperm(S, generator=g)[:count]] = True
    out = tk.partial_prefill_attention(q.to(DEV), k.to(DEV), v.to(DEV), mask.to(DEV))
    _check_rows(out, q, k, v, mask, atol=2e-2)
