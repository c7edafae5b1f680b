"""Masked QKV projection (``sb_masked_linear``) and the partial-prefill
orchestrator on the GPU, against the reference's golden outputs and the CPU
oracle; the reference's own scenarios (synapse_kv_connector/tests/
test_triton_kernels.py:310-385 and :501-765) run through the drop-ins.

Tolerances: the reference accumulates in fp32 and rounds once to the input
dtype; a different summation order moves the fp32 sum by at most
``K * 2^-24 * sum|x||w|``, and the final rounding by one ulp of the output
dtype, so outputs must agree within ``1 ulp + K * 2^-23 * (|x| @ |w|^T)``.
"""

from __future__ import annotations

import math

import pytest
import torch

from oracle import attention as oattn
from tests.helpers import load_golden

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _ulp_rel(dt: torch.dtype) -> float:
    return {torch.float32: 2.0**-23, torch.float16: 2.0**-10, torch.bfloat16: 2.0**-7}[dt]


def assert_projection_close(got, want, h, w, b=None):
    """|got - want| <= 1 ulp(|want|) + K 2^-23 (|h| @ |w|^T + |b|), elementwise."""
    got, want = got.float().cpu(), want.float().cpu()
    K = h.shape[1]
    mag = torch.nn.functional.linear(h.float().abs().cpu(), w.float().abs().cpu(),
                                     b.float().abs().cpu() if b is not None else None)
    tol = want.abs() * _ulp_rel(h.dtype) + K * 2.0**-23 * mag + 1e-30
    bad = (got - want).abs() > tol
    assert not bad.any(), f"{int(bad.sum())} elements out of tolerance; worst {(got - want).abs().max():.3e}"


def _proj(h, w, mask, b=None):
    from semblend_b200.triton_kernels import masked_qkv_projection

    return masked_qkv_projection(h.to(DEV), w.to(DEV), mask.to(DEV), b.to(DEV) if b is not None else None)


@pytest.mark.parametrize("name", ["proj_fp32", "proj_fp16"])
def test_projection_matches_reference_golden(name):
    g = load_golden(name)
    h, w, mask, want = g["h"], g["w"], g["mask"], g["out"]
    b = g.get("b")
    got = _proj(h, w, mask, b).cpu()
    assert got.dtype == want.dtype
    assert torch.all(got[~mask] == 0)
    assert_projection_close(got, want, h, w, b)


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("S,K,N,frac", [(300, 512, 1536, 0.3), (1000, 1024, 640, 0.9), (129, 256, 264, 0.5),
                                        (64, 40, 96, 0.5), (17, 128, 100, 1.0)])
def test_projection_matches_oracle(dt, S, K, N, frac):
    g = torch.Generator().manual_seed(S * 7 + K + N)
    h = torch.randn(S, K, generator=g).to(dt)
    w = (torch.randn(N, K, generator=g) / math.sqrt(K)).to(dt)
    b = torch.randn(N, generator=g).to(dt)
    mask = torch.rand(S, generator=g) < frac
    want = oattn.masked_qkv_projection(h, w, mask, b)
    got = _proj(h, w, mask, b).cpu()
    assert torch.all(got[~mask] == 0)
    assert_projection_close(got, want, h, w, b)


def test_projection_strided_rows_and_many_tiles():
    """A hidden-state view with a row stride larger than K, several M and N tiles
    per CTA (persistent loop, both TMEM accumulator buffers in use)."""
    g = torch.Generator().manual_seed(5)
    S, K, N = 148 * 128 * 2 + 77, 128, 512
    base = torch.randn(S, K + 64, generator=g).to(torch.bfloat16)
    h = base[:, 32 : 32 + K]
    w = (torch.randn(N, K, generator=g) / math.sqrt(K)).to(torch.bfloat16)
    mask = torch.rand(S, generator=g) < 0.8
    from semblend_b200.triton_kernels import masked_qkv_projection

    hd = base.to(DEV)[:, 32 : 32 + K]
    assert hd.stride(0) == K + 64
    got = masked_qkv_projection(hd, w.to(DEV), mask.to(DEV)).cpu()
    want = oattn.masked_qkv_projection(h, w, mask)
    assert_projection_close(got, want, h, w)


def test_projection_twice_in_a_row_is_deterministic():
    g = torch.Generator().manual_seed(9)
    h = torch.randn(700, 256, generator=g).to(torch.float16)
    w = torch.randn(768, 256, generator=g).to(torch.float16)
    mask = torch.rand(700, generator=g) < 0.4
    a = _proj(h, w, mask)
    b = _proj(h, w, mask)
    assert torch.equal(a, b)


# -- reference scenarios (test_triton_kernels.py:313-385) -----------------------------------------


def _ref_inputs(seq, hid, out, seed=0, bias=False):
    g = torch.Generator().manual_seed(seed)
    h = torch.randn(seq, hid, generator=g, dtype=torch.float32).half()
    w = torch.randn(out, hid, generator=g, dtype=torch.float32).half()
    b = torch.randn(out, generator=g, dtype=torch.float32).half() if bias else None
    return h, w, b


def test_all_compute_matches_linear():
    h, w, _ = _ref_inputs(8, 32, 48)
    got = _proj(h, w, torch.ones(8, dtype=torch.bool))
    torch.testing.assert_close(got, torch.nn.functional.linear(h.to(DEV), w.to(DEV)), atol=1e-2, rtol=1e-2)


def test_all_reuse_is_zero():
    h, w, _ = _ref_inputs(8, 32, 48)
    assert torch.all(_proj(h, w, torch.zeros(8, dtype=torch.bool)) == 0)


def test_mixed_mask():
    h, w, _ = _ref_inputs(8, 32, 48)
    mask = torch.tensor([True, False] * 4)
    got = _proj(h, w, mask).cpu()
    for i in (1, 3, 5, 7):
        assert torch.all(got[i] == 0)
    for i in (0, 2, 4, 6):
        assert not torch.all(got[i] == 0)


def test_with_bias():
    h, w, b = _ref_inputs(4, 16, 24, bias=True)
    got = _proj(h, w, torch.ones(4, dtype=torch.bool), b)
    want = torch.nn.functional.linear(h.to(DEV), w.to(DEV), b.to(DEV))
    torch.testing.assert_close(got, want, atol=1e-2, rtol=1e-2)


# -- partial_prefill (test_triton_kernels.py:501-765) ---------------------------------------------


def _pp_case(seq, hid, heads, hd, layers, donor_len, seed=0):
    g = torch.Generator().manual_seed(seed)
    h = torch.randn(seq, hid, generator=g).half()
    donor = torch.randn(layers, 2, heads, donor_len, hd, generator=g).half()
    wqkv = torch.randn(3 * heads * hd, hid, generator=g).half()
    wo = torch.randn(hid, heads * hd, generator=g).half()
    return h, donor, wqkv, wo


def _pp(h, donor, wqkv, wo, dpos, tpos, mask, heads, hd, **kw):
    from semblend_b200.triton_kernels import partial_prefill

    return partial_prefill(hidden_states=h.to(DEV), donor_kv=donor.to(DEV), qkv_weight=wqkv.to(DEV),
                           output_projection=wo.to(DEV), donor_positions=dpos.to(DEV),
                           target_positions=tpos.to(DEV), compute_mask=mask.to(DEV), num_heads=heads,
                           head_dim=hd, **kw)


def _check_against_oracle(res, h, donor, wqkv, wo, dpos, tpos, mask, heads, hd, **kw):
    want_out, want_kv = oattn.partial_prefill(h, donor, wqkv, wo, dpos, tpos, mask, heads, hd, **kw)
    kv = res.kv_cache.cpu()
    # donor rows are copied exactly; the new K/V rows come from the projection
    reuse = ~mask
    assert torch.equal(kv[..., reuse, :], want_kv[..., reuse, :])
    got_new, want_new = kv[..., mask, :].float(), want_kv[..., mask, :].float()
    u = _ulp_rel(h.dtype)
    assert torch.allclose(got_new, want_new, rtol=u, atol=float(want_new.abs().max()) * u + 1e-3)
    out = res.output.cpu()
    assert torch.all(out[reuse] == 0)
    scale = float(want_out.float().abs().max()) + 1e-6
    assert (out.float() - want_out.float()).abs().max() <= 2e-2 * scale


def test_partial_prefill_basic_half_reuse():
    h, donor, wqkv, wo = _pp_case(8, 32, 4, 8, 2, 8)
    dpos = torch.tensor([0, 1, 2, 3], dtype=torch.int32)
    mask = torch.tensor([False] * 4 + [True] * 4)
    res = _pp(h, donor, wqkv, wo, dpos, dpos, mask, 4, 8)
    from semblend_b200.triton_kernels import PartialPrefillResult

    assert isinstance(res, PartialPrefillResult)
    assert res.positions_computed == 4 and res.positions_reused == 4
    assert abs(res.computation_ratio - 0.5) < 1e-6
    assert res.output.shape == (8, 32)
    assert res.kv_cache.shape == (2, 2, 4, 8, 8)
    _check_against_oracle(res, h, donor, wqkv, wo, dpos, dpos, mask, 4, 8)


def test_partial_prefill_full_reuse():
    h, donor, wqkv, wo = _pp_case(4, 16, 2, 8, 1, 4)
    pos = torch.arange(4, dtype=torch.int32)
    res = _pp(h, donor, wqkv, wo, pos, pos, torch.zeros(4, dtype=torch.bool), 2, 8)
    assert res.positions_computed == 0 and res.positions_reused == 4
    assert res.computation_ratio == 0.0
    assert torch.equal(res.kv_cache.cpu(), donor)
    assert torch.all(res.output == 0)


def test_partial_prefill_no_reuse():
    h, donor, wqkv, wo = _pp_case(4, 16, 2, 8, 1, 4)
    empty = torch.zeros(0, dtype=torch.int32)
    mask = torch.ones(4, dtype=torch.bool)
    res = _pp(h, donor, wqkv, wo, empty, empty, mask, 2, 8)
    assert res.positions_computed == 4 and res.positions_reused == 0
    assert res.computation_ratio == 1.0
    _check_against_oracle(res, h, donor, wqkv, wo, empty, empty, mask, 2, 8)


def test_partial_prefill_sparse_reuse_copies_donor_rows():
    h, donor, wqkv, wo = _pp_case(16, 32, 4, 8, 2, 10)
    dpos = torch.tensor([0, 2, 4, 6, 8], dtype=torch.int32)
    tpos = torch.tensor([0, 3, 6, 9, 12], dtype=torch.int32)
    mask = torch.ones(16, dtype=torch.bool)
    mask[tpos.long()] = False
    res = _pp(h, donor, wqkv, wo, dpos, tpos, mask, 4, 8)
    assert res.positions_reused == 5 and res.positions_computed == 11
    kv = res.kv_cache.cpu()
    for d, t in zip(dpos.tolist(), tpos.tolist()):
        assert torch.equal(kv[:, :, :, t, :], donor[:, :, :, d, :])
    _check_against_oracle(res, h, donor, wqkv, wo, dpos, tpos, mask, 4, 8)


def test_partial_prefill_timing_reported():
    h, donor, wqkv, wo = _pp_case(64, 128, 8, 16, 4, 32)
    pos = torch.arange(16, dtype=torch.int32)
    mask = torch.ones(64, dtype=torch.bool)
    mask[:16] = False
    res = _pp(h, donor, wqkv, wo, pos, pos, mask, 8, 16)
    assert res.total_time_ms > 0
    assert res.scatter_time_ms >= 0


def test_partial_prefill_tensor_core_shapes_with_bias():
    """head_dim 128 and a hidden size that takes the tcgen05 projection."""
    g = torch.Generator().manual_seed(3)
    S, heads, hd, L = 300, 4, 128, 2
    hid = heads * hd
    h = torch.randn(S, hid, generator=g).to(torch.bfloat16)
    donor = torch.randn(L, 2, heads, 200, hd, generator=g).to(torch.bfloat16)
    wqkv = (torch.randn(3 * hid, hid, generator=g) / math.sqrt(hid)).to(torch.bfloat16)
    bqkv = torch.randn(3 * hid, generator=g).to(torch.bfloat16)
    wo = (torch.randn(hid, hid, generator=g) / math.sqrt(hid)).to(torch.bfloat16)
    bo = torch.randn(hid, generator=g).to(torch.bfloat16)
    dpos = torch.arange(0, 200, dtype=torch.int32)
    tpos = torch.arange(50, 250, dtype=torch.int32)
    mask = torch.ones(S, dtype=torch.bool)
    mask[tpos.long()] = False
    res = _pp(h, donor, wqkv, wo, dpos, tpos, mask, heads, hd, qkv_bias=bqkv.to(DEV), output_bias=bo.to(DEV))
    _check_against_oracle(res, h, donor, wqkv, wo, dpos, tpos, mask, heads, hd, qkv_bias=bqkv, output_bias=bo)
