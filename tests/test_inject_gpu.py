"""GPU parity of the fused inject kernel family against the CPU oracle and the
reference's golden fixtures.

Bar: V rows, pure copies and untouched rows bit-exact; RoPE-corrected K rows
within 1 ulp of the element type for bf16 / fp16 and within 1e-5 relative for
fp32, both measured at the magnitude of each element's RoPE pair
(tests/helpers.py:assert_rope_close).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import rope as orope
from semblend_b200 import _lib
from semblend_b200 import rope_correction as rc
from semblend_b200 import triton_kernels as tk
from tests.helpers import assert_rope_close, load_golden

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _split_check(out_gpu: torch.Tensor, expected: torch.Tensor, layout: str = "canonical",
                 style: str = "interleaved"):
    """K half within RoPE tolerance, V half bit-exact (paged caches)."""
    og = orope.canonical_view(out_gpu.cpu(), layout)
    ex = orope.canonical_view(expected, layout)
    assert torch.equal(og[:, 1].contiguous().view(torch.uint8), ex[:, 1].contiguous().view(torch.uint8))
    assert_rope_close(og[:, 0].contiguous(), ex[:, 0].contiguous(), style)


def _untouched_exact(out_gpu, before, block_table, t_pos, layout="canonical"):
    """Rows no pair targets keep their bits."""
    og = orope.canonical_view(out_gpu.cpu(), layout)
    bf = orope.canonical_view(before, layout)
    nb, _, _, bs, _ = bf.shape
    hit = torch.zeros(nb, bs, dtype=torch.bool)
    bt = block_table.tolist()
    for t in t_pos.tolist():
        if 0 <= t and t // bs < len(bt) and 0 <= bt[t // bs] < nb:
            hit[bt[t // bs], t % bs] = True
    keep = ~hit
    a = og.permute(0, 3, 1, 2, 4)[keep]
    b = bf.permute(0, 3, 1, 2, 4)[keep]
    assert torch.equal(a.contiguous().view(torch.uint8), b.contiguous().view(torch.uint8))


@pytest.fixture(autouse=True)
def _reset_counter():
    _lib.skipped_pairs(DEV, reset=True)
    yield


# ----------------------------------------------------------------------------
# Golden fixtures (the reference's own outputs)
# ----------------------------------------------------------------------------
@pytest.mark.parametrize("name", ["rcsp_fp32", "rcsp_bf16", "rcsp_fp16", "rcsp_c1mini"])
def test_rope_scatter_paged_golden(name):
    g = load_golden(name)
    cache = g["cache"].to(DEV)
    out = rc.rope_correct_scatter_paged(cache, g["donor"].to(DEV), g["block_table"].to(DEV),
                                        g["d_pos"].to(DEV), g["t_pos"].to(DEV), rope_base=g["rope_base"])
    assert out is cache
    _split_check(out, g["out"])
    _untouched_exact(out, g["cache"], g["block_table"], g["t_pos"])
    assert _lib.skipped_pairs(DEV) == 0


def test_scatter_flat_golden():
    g = load_golden("scatter_flat")
    t = g["target"].to(DEV)
    out = tk.scatter_donor_kv(t, g["donor"].to(DEV), g["d_pos"].to(DEV), g["t_pos"].to(DEV))
    assert out is t and torch.equal(out.cpu(), g["out"])


def test_scatter_paged_golden():
    g = load_golden("scatter_paged")
    c = g["cache"].to(DEV)
    out = tk.scatter_donor_kv_paged(c, g["donor"].to(DEV), g["block_table"].to(DEV), g["d_pos"].to(DEV),
                                    g["t_pos"].to(DEV))
    assert out is c and torch.equal(out.cpu(), g["out"])


@pytest.mark.parametrize("name", ["rck_3d_fp32", "rck_4d_bf16"])
def test_rope_correct_k_golden(name):
    g = load_golden(name)
    k = g["k"].to(DEV)
    out = rc.rope_correct_k(k, g["d_pos"].to(DEV), g["t_pos"].to(DEV), head_dim=g["head_dim"],
                            rope_base=g["rope_base"])
    assert out is not k and torch.equal(k.cpu(), g["k"])  # input untouched
    assert_rope_close(out.cpu(), g["out"])


@pytest.mark.parametrize("name", ["permute_fp32", "permute_bf16"])
def test_permute_golden(name):
    g = load_golden(name)
    c = g["cache"].to(DEV)
    rc.permute_paged_kv_with_rope(c, g["block_table"].to(DEV), [tuple(p) for p in g["pairs"].tolist()],
                                  rope_base=g["rope_base"])
    _split_check(c, g["out"])


def test_nope_golden():
    g = load_golden("nope_fp16")
    c = g["cache"].to(DEV)
    rc.nope_permute_paged_kv(c, g["block_table"].to(DEV), [tuple(p) for p in g["pairs"].tolist()],
                             rope_base=g["rope_base"])
    _split_check(c, g["out"])


@pytest.mark.parametrize("name,layout", [("ropedelta_canon", "canonical"), ("ropedelta_vllm", "vllm")])
def test_apply_rope_delta_golden(name, layout):
    g = load_golden(name)
    c = g["cache"].to(DEV)
    n = rc.apply_rope_delta_inplace(c, g["block_table"].to(DEV), g["positions"].tolist(), g["delta"],
                                    rope_base=g["rope_base"])
    assert n == g["count"]
    _split_check(c, g["out"], layout)


# ----------------------------------------------------------------------------
# Seeded cases against the oracle
# ----------------------------------------------------------------------------
def _case(seed, dtype, H=4, D=128, Sd=300, nb=40, bs=16, n_log=24, n_pairs=200, layout="canonical"):
    g = torch.Generator().manual_seed(seed)
    donor = torch.randn(2, H, Sd, D, generator=g).to(dtype)
    shape = {"canonical": (nb, 2, H, bs, D), "vllm": (2, nb, bs, H, D), "trtllm": (nb, 2, bs, H, D)}[layout]
    cache = torch.randn(*shape, generator=g).to(dtype)
    bt = torch.randperm(nb, generator=g)[:n_log].to(torch.int32)
    t = torch.randperm(n_log * bs, generator=g)[:n_pairs].to(torch.int32)
    d = torch.randint(0, Sd, (n_pairs,), generator=g, dtype=torch.int32)
    return donor, cache, bt, d, t


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("style", ["interleaved", "neox"])
@pytest.mark.parametrize("layout", ["canonical", "vllm", "trtllm"])
def test_rope_scatter_paged_vs_oracle(dtype, style, layout):
    donor, cache, bt, d, t = _case(1, dtype, layout=layout)
    want = orope.rope_correct_scatter_paged(cache, donor, bt, d, t, 1e6, style, layout)
    c = cache.to(DEV)
    rc.rope_correct_scatter_paged(c, donor.to(DEV), bt.to(DEV), d.to(DEV), t.to(DEV), rope_base=1e6,
                                  rotary_style=style, layout=layout)
    _split_check(c, want, layout, style)
    _untouched_exact(c, cache, bt, t, layout)


@pytest.mark.parametrize("D", [16, 32, 64, 96, 256])
def test_head_dims_and_vector_widths(D):
    donor, cache, bt, d, t = _case(2, torch.bfloat16, H=2, D=D, n_pairs=64)
    want = orope.rope_correct_scatter_paged(cache, donor, bt, d, t, 1e4, "neox")
    c = cache.to(DEV)
    rc.rope_correct_scatter_paged(c, donor.to(DEV), bt.to(DEV), d.to(DEV), t.to(DEV), rope_base=1e4,
                                  rotary_style="neox")
    _split_check(c, want, style="neox")


def test_strided_donor_scalar_path():
    donor, cache, bt, d, t = _case(3, torch.float32, H=2, D=32, n_pairs=50)
    big = torch.zeros(2, 2, donor.shape[2], 64)
    big[..., ::2] = donor  # last-dim stride 2 forces the scalar path
    want = orope.rope_correct_scatter_paged(cache, donor, bt, d, t, 1e4, "interleaved")
    c = cache.to(DEV)
    rc.rope_correct_scatter_paged(c, big.to(DEV)[..., ::2], bt.to(DEV), d.to(DEV), t.to(DEV), rope_base=1e4)
    _split_check(c, want)


def test_int64_positions_and_block_table():
    donor, cache, bt, d, t = _case(4, torch.bfloat16)
    want = orope.rope_correct_scatter_paged(cache, donor, bt, d, t, 1e6, "neox")
    c = cache.to(DEV)
    rc.rope_correct_scatter_paged(c, donor.to(DEV), bt.long().to(DEV), d.long().to(DEV), t.long().to(DEV),
                                  rope_base=1e6, rotary_style="neox")
    _split_check(c, want, style="neox")


def test_out_of_range_pairs_are_skipped_and_counted():
    donor, cache, bt, d, t = _case(5, torch.float32, Sd=64, nb=20, n_log=8, n_pairs=40)
    bt[3] = 25  # physical block out of range
    d = d % 64
    d[0] = 64  # donor position out of range
    d[1] = -1
    t[2] = 8 * 16 + 3  # logical block beyond the table
    t[3] = -5
    t[4] = 3 * 16 + 1  # lands in the bad physical block
    want = orope.rope_correct_scatter_paged(cache, donor, bt, d, t, 1e4)
    c = cache.to(DEV)
    rc.rope_correct_scatter_paged(c, donor.to(DEV), bt.to(DEV), d.to(DEV), t.to(DEV), rope_base=1e4)
    _split_check(c, want)
    bad = sum(1 for dp, tp in zip(d.tolist(), t.tolist())
              if not (0 <= dp < 64 and 0 <= tp and tp // 16 < 8 and 0 <= bt[tp // 16] < 20))
    assert _lib.skipped_pairs(DEV) == bad >= 6


def test_empty_pairs_is_noop():
    donor, cache, bt, _, _ = _case(6, torch.float32)
    c = cache.to(DEV)
    e = torch.zeros(0, dtype=torch.int32, device=DEV)
    assert rc.rope_correct_scatter_paged(c, donor.to(DEV), bt.to(DEV), e, e) is c
    assert tk.scatter_donor_kv_paged(c, donor.to(DEV), bt.to(DEV), e, e) is c
    assert torch.equal(c.cpu(), cache)


def test_zero_delta_is_bit_exact_copy():
    donor, cache, bt, d, t = _case(7, torch.bfloat16, Sd=24 * 16, n_pairs=300)
    d = t.clone()  # delta 0 everywhere
    c = cache.to(DEV)
    rc.rope_correct_scatter_paged(c, donor.to(DEV), bt.to(DEV), d.to(DEV), t.to(DEV), rope_base=1e6,
                                  rotary_style="neox")
    want = orope.scatter_donor_kv_paged(cache, donor, bt, d, t)
    assert torch.equal(c.cpu().view(torch.int16), want.view(torch.int16))


def test_cpu_tensors_fail_loudly():
    donor, cache, bt, d, t = _case(8, torch.float32)
    with pytest.raises(_lib.NativeLibraryError):
        rc.rope_correct_scatter_paged(cache, donor, bt, d, t)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_scatter_flat_vs_oracle(dtype):
    g = torch.Generator().manual_seed(9)
    target = torch.randn(3, 2, 4, 50, 64, generator=g).to(dtype)
    donor = torch.randn(3, 2, 4, 40, 64, generator=g).to(dtype)
    t = torch.randperm(60, generator=g)[:30].to(torch.int32)  # some beyond target_len
    d = torch.randint(0, 45, (30,), generator=g, dtype=torch.int32)  # some beyond donor_len
    want = orope.scatter_donor_kv(target, donor, d, t)
    x = target.to(DEV)
    tk.scatter_donor_kv(x, donor.to(DEV), d.to(DEV), t.to(DEV))
    assert torch.equal(x.cpu(), want)


@pytest.mark.parametrize("shape", [(4, 64, 128), (3, 2, 48, 64)])
@pytest.mark.parametrize("style", ["interleaved", "neox"])
def test_rope_correct_k_vs_oracle(shape, style):
    g = torch.Generator().manual_seed(10)
    k = torch.randn(*shape, generator=g).to(torch.bfloat16)
    S, D = shape[-2], shape[-1]
    d = torch.randperm(S, generator=g)[:20].to(torch.int32)
    t = torch.randint(0, 5000, (20,), generator=g, dtype=torch.int32)
    want = orope.rope_correct_k(k, d, t, head_dim=D, rope_base=1e6, rotary_style=style)
    out = rc.rope_correct_k(k.to(DEV), d.to(DEV), t.to(DEV), head_dim=D, rope_base=1e6, rotary_style=style)
    assert_rope_close(out.cpu(), want, style)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("style", ["interleaved", "neox"])
def test_permute_overlapping_vs_oracle(dtype, style):
    g = torch.Generator().manual_seed(11)
    cache = torch.randn(12, 2, 4, 16, 128, generator=g).to(dtype)
    bt = torch.randperm(12, generator=g)[:10].to(torch.int32)
    perm = np.random.default_rng(3).permutation(160)
    pairs = [(int(i), int(perm[i])) for i in range(160) if i != perm[i]]
    want = orope.permute_paged_kv_with_rope(cache, bt, pairs, 1e4, style)
    c = cache.to(DEV)
    rc.permute_paged_kv_with_rope(c, bt.to(DEV), pairs, rope_base=1e4, rotary_style=style)
    _split_check(c, want, style=style)


def test_permute_rejects_positions_outside_table():
    cache = torch.zeros(4, 2, 2, 16, 64, device=DEV)
    bt = torch.arange(2, dtype=torch.int32, device=DEV)
    with pytest.raises(IndexError):
        rc.permute_paged_kv_with_rope(cache, bt, [(0, 40)])
    with pytest.raises(IndexError):
        rc.nope_permute_paged_kv(cache, bt, [(-1, 3)])


def test_nope_chained_permutation_uses_snapshot_v():
    g = torch.Generator().manual_seed(12)
    cache = torch.randn(6, 2, 2, 16, 64, generator=g).to(torch.float16)
    bt = torch.arange(6, dtype=torch.int32)
    pairs = [(i, i + 16) for i in range(32)]  # sources 16..31 are also targets
    want = orope.nope_permute_paged_kv(cache, bt, pairs, 1e4, v_from_snapshot=True)
    c = cache.to(DEV)
    rc.nope_permute_paged_kv(c, bt.to(DEV), pairs, rope_base=1e4)
    _split_check(c, want)


def test_nope_equals_delta_within_rounding():
    g = torch.Generator().manual_seed(13)
    cache = torch.randn(8, 2, 4, 16, 128, generator=g)
    bt = torch.arange(8, dtype=torch.int32)
    pairs = [(5, 5 + dl) for dl in (0,)] + [(i, 64 + i * 3 % 60) for i in range(6, 30)]
    a = cache.to(DEV)
    b = cache.to(DEV)
    rc.permute_paged_kv_with_rope(a, bt.to(DEV), pairs)
    rc.nope_permute_paged_kv(b, bt.to(DEV), pairs)
    torch.testing.assert_close(a.cpu(), b.cpu(), atol=5e-3, rtol=5e-3)


def test_apply_rope_delta_round_trip():
    g = torch.Generator().manual_seed(14)
    cache = torch.randn(6, 2, 4, 16, 64, generator=g)
    bt = torch.tensor([2, 0, 5], dtype=torch.int32)
    c = cache.to(DEV)
    pos = list(range(0, 48, 3))
    assert rc.apply_rope_delta_inplace(c, bt.to(DEV), pos, 700) == len(pos)
    assert rc.apply_rope_delta_inplace(c, bt.to(DEV), pos, -700) == len(pos)
    torch.testing.assert_close(c.cpu(), cache, atol=2e-5, rtol=2e-5)


# ----------------------------------------------------------------------------
# Multi-request, multi-layer single launch
# ----------------------------------------------------------------------------
@pytest.mark.parametrize("as_list", [False, True])
@pytest.mark.parametrize("mode", ["delta", "nope", "copy"])
def test_inject_donors_matches_per_layer_oracle(as_list, mode):
    g = torch.Generator().manual_seed(15)
    L, H, D, bs, nb = 3, 4, 128, 16, 64
    cache = torch.randn(L, nb, 2, H, bs, D, generator=g).to(torch.bfloat16)
    perm = torch.randperm(nb, generator=g)
    reqs = []
    for r in range(3):
        Sd = 100 + 30 * r
        donor = torch.randn(L, 2, H, Sd, D, generator=g).to(torch.bfloat16)
        bt = perm[r * 20 : r * 20 + 20].to(torch.int32)
        t = torch.randperm(20 * bs, generator=g)[:90].to(torch.int32)
        d = torch.randint(0, Sd, (90,), generator=g, dtype=torch.int32)
        reqs.append((donor, bt, d, t))
    want = cache.clone()
    for donor, bt, d, t in reqs:
        for layer in range(L):
            if mode == "copy":
                want[layer] = orope.scatter_donor_kv_paged(want[layer], donor[layer], bt, d, t)
            elif mode == "delta":
                want[layer] = orope.rope_correct_scatter_paged(want[layer], donor[layer], bt, d, t, 5e5, "neox")
            else:  # NoPE equals the delta rotation up to rounding; compared loosely below
                want[layer] = orope.rope_correct_scatter_paged(want[layer], donor[layer], bt, d, t, 5e5, "neox")
    c = cache.to(DEV)
    kv = [c[layer] for layer in range(L)] if as_list else c
    rc.inject_donors(kv, [rc.DonorInjection(x.to(DEV), bt.to(DEV), d.to(DEV), t.to(DEV)) for x, bt, d, t in reqs],
                     rope_base=5e5, mode=mode, rotary_style="neox")
    got = c.cpu()
    for layer in range(L):
        if mode == "nope":
            torch.testing.assert_close(got[layer].float(), want[layer].float(), atol=2e-2, rtol=2e-2)
        else:
            _split_check(got[layer], want[layer], style="neox")


def test_inject_donors_many_requests_one_launch():
    """More descriptors than the kernel parameters hold (device descriptor
    table): 150 requests, some without pairs, some with out-of-range pairs."""
    g = torch.Generator().manual_seed(27)
    L, H, D, bs, nb = 2, 2, 64, 16, 400
    cache = torch.randn(L, nb, 2, H, bs, D, generator=g).to(torch.bfloat16)
    perm = torch.randperm(nb, generator=g)
    reqs, n_bad = [], 0
    for r in range(150):
        Sd = 20 + (r % 7) * 5
        donor = torch.randn(L, 2, H, Sd, D, generator=g).to(torch.bfloat16)
        bt = perm[(r * 2) % (nb - 2) : (r * 2) % (nb - 2) + 2].to(torch.int32)
        n = 0 if r % 11 == 0 else int(torch.randint(1, 20, (1,), generator=g))
        t = torch.randperm(2 * bs, generator=g)[:n].to(torch.int32)
        d = torch.randint(0, Sd, (n,), generator=g, dtype=torch.int32)
        if r % 13 == 5 and n:
            d[0] = Sd + 3  # out of the donor's range: skipped and counted
            n_bad += 1
        reqs.append((donor, bt, d, t))
    want = cache.clone()
    for donor, bt, d, t in reqs:
        for layer in range(L):
            want[layer] = orope.rope_correct_scatter_paged(want[layer], donor[layer], bt, d, t, 1e4, "neox")
    c = cache.to(DEV)
    _lib.skipped_pairs(DEV, reset=True)
    rc.inject_donors(c, [rc.DonorInjection(x.to(DEV), bt.to(DEV), d.to(DEV), t.to(DEV)) for x, bt, d, t in reqs],
                     rope_base=1e4, mode="delta", rotary_style="neox")
    got = c.cpu()
    assert _lib.skipped_pairs(DEV, reset=True) == n_bad
    for layer in range(L):
        _split_check(got[layer], want[layer], style="neox")


def _plan_case(seed, multi):
    """A plan over 6 layers (layers 1 and 4 recomputed in full) with reused and
    recomputed target positions, one donor or three."""
    from semblend_b200 import partial_attention as pa

    rng = np.random.default_rng(seed)
    L, target_len = 6, 300
    hints = [{"recomputeAll": layer in (1, 4)} for layer in range(L)]
    donors = {"a": 180, "b": 260, "c": 120} if multi else {"a": 280}
    actions, reuse = [], []
    for t in rng.permutation(target_len)[:250].tolist():
        if rng.random() < 0.8:
            did = str(rng.choice(list(donors)))
            dpos = int(rng.integers(0, donors[did]))
            act = {"action": "copy_from_donor", "targetPos": t, "donorPos": dpos}
            if multi:
                act["donorId"] = did
            actions.append(act)
            reuse.append((did, dpos, t))
        else:
            actions.append({"action": "recompute" if multi else "placeholder", "targetPos": t})
    if multi:
        plan = pa.build_multi_donor_attention_plan(target_len, actions, hints, L)
    else:
        copy = [t for _, _, t in reuse]
        plan = pa.build_attention_plan("a", target_len, donors["a"], copy, [], actions, hints, L)
    return plan, donors, reuse, L


@pytest.mark.parametrize("multi", [False, True])
@pytest.mark.parametrize("as_list", [False, True])
def test_inject_plan_one_launch_matches_per_layer_oracle(multi, as_list):
    plan, donor_lens, reuse, L = _plan_case(21 + multi, multi)
    g = torch.Generator().manual_seed(22)
    H, D, bs, nb = 2, 128, 16, 40
    cache = torch.randn(L, nb, 2, H, bs, D, generator=g).to(torch.bfloat16)
    bt = torch.randperm(nb, generator=g)[: (300 + bs - 1) // bs].to(torch.int32)
    donors = {k: torch.randn(L, 2, H, n, D, generator=g).to(torch.bfloat16) for k, n in donor_lens.items()}
    want = cache.clone()
    for did in donors:
        d = torch.tensor([dp for x, dp, _ in reuse if x == did], dtype=torch.int32)
        t = torch.tensor([tp for x, _, tp in reuse if x == did], dtype=torch.int32)
        for layer in range(L):
            if layer in (1, 4):
                continue
            want[layer] = orope.rope_correct_scatter_paged(want[layer], donors[did][layer], bt, d, t, 5e5, "neox")
    c = cache.to(DEV)
    kv = [c[layer] for layer in range(L)] if as_list else c
    dk = {k: v.to(DEV) for k, v in donors.items()} if multi else donors["a"].to(DEV)
    n = rc.inject_plan(kv, dk, bt.to(DEV), plan, rope_base=5e5, rotary_style="neox")
    assert n == L - 2
    got = c.cpu()
    for layer in range(L):
        if layer in (1, 4):
            assert torch.equal(got[layer], cache[layer])  # recomputed in full: untouched
        else:
            assert torch.equal(got[layer][:, 1], want[layer][:, 1])
            assert_rope_close(got[layer][:, 0].contiguous(), want[layer][:, 0].contiguous(), "neox")


# ----------------------------------------------------------------------------
# BASELINE configs[0] (c1) at full size
# ----------------------------------------------------------------------------
def test_c1_full_size_matches_oracle():
    """c1 exactly as configured: fp32 donor K/V [4096 tokens, 4 KV heads, 128],
    16 permuted 256-token chunks, neox RoPE theta 1e6, block 16, 256 of 1024
    blocks.  V and untouched rows bit-exact, K within 1e-5 relative at the
    RoPE pair's magnitude, all 4096 pairs applied."""
    import bench

    donor, cache, bt, d, t = bench.make_c1_inputs(bench.SEED + 1)
    want, applied = orope.rope_correct_scatter_paged(cache, donor, bt, d, t, 1e6, "neox", return_applied=True)
    assert applied == 4096
    c = cache.to(DEV)
    out = rc.rope_correct_scatter_paged(c, donor.to(DEV), bt.to(DEV), d.to(DEV), t.to(DEV), rope_base=1e6,
                                        rotary_style="neox")
    assert out is c
    _split_check(out, want, style="neox")
    _untouched_exact(out, cache, bt, t)
    assert _lib.skipped_pairs(DEV) == 0


# ----------------------------------------------------------------------------
# The bulk-copy-staged kernel (SB_INJECT_BULK_STAGED) against the direct path
# ----------------------------------------------------------------------------
@pytest.mark.parametrize("dtype,D,style,layout", [
    (torch.bfloat16, 128, "neox", "canonical"), (torch.bfloat16, 96, "neox", "vllm"),
    (torch.bfloat16, 16, "interleaved", "canonical"), (torch.float16, 64, "interleaved", "trtllm"),
    (torch.float32, 128, "neox", "canonical"), (torch.float32, 96, "interleaved", "canonical"),
])
def test_bulk_staging_equals_direct_path(dtype, D, style, layout):
    """Same bits as the direct path and within the bar of the oracle, with
    out-of-range pairs (donor positions past the donor, targets past the
    table) skipped and counted the same way; D = 96 leaves threads that own
    no pair."""
    donor, cache, bt, d, t = _case(11 + D, dtype, H=2, D=D, n_pairs=300, layout=layout)
    d[::37] = donor.shape[2] + 5
    t[5::41] = bt.shape[0] * 16 + 3
    want = orope.rope_correct_scatter_paged(cache, donor, bt, d, t, 1e6, style, layout)
    outs, skipped = [], []
    for staging in ("direct", "bulk"):
        c = cache.to(DEV)
        _lib.skipped_pairs(DEV, reset=True)
        rc.rope_correct_scatter_paged(c, donor.to(DEV), bt.to(DEV), d.to(DEV), t.to(DEV), rope_base=1e6,
                                      rotary_style=style, layout=layout, staging=staging)
        skipped.append(_lib.skipped_pairs(DEV))
        outs.append(c.cpu())
    assert torch.equal(outs[0].view(torch.uint8), outs[1].view(torch.uint8))
    assert skipped[0] == skipped[1] > 0
    _split_check(outs[1], want, layout, style)
    _untouched_exact(outs[1], cache, bt, t, layout)


def test_bulk_staging_many_requests_table():
    """More than 64 requests (the device descriptor table) with chunk-shifted
    pairs (long runs of contiguous donor rows) and several layers."""
    g = torch.Generator().manual_seed(31)
    L, H, D, bs, S = 3, 2, 128, 16, 512
    n_req = 70
    cache = torch.randn(L, n_req * (S // bs), 2, H, bs, D, generator=g).to(torch.bfloat16)
    rng = np.random.default_rng(31)
    injections, host = [], []
    perm = rng.permutation(n_req * (S // bs)).astype(np.int32)
    for r in range(n_req):
        donor = torch.randn(L, 2, H, S, D, generator=g).to(torch.bfloat16)
        shift = int(rng.integers(-128, 129))
        tpos = np.arange(max(0, shift), min(S, S + shift)).astype(np.int32)
        tpos = tpos[rng.random(tpos.shape[0]) > 0.1]
        dpos = (tpos - shift).astype(np.int32)
        bt = torch.from_numpy(perm[r * (S // bs):(r + 1) * (S // bs)].copy())
        host.append((donor, bt, torch.from_numpy(dpos), torch.from_numpy(tpos)))
    outs = []
    for staging in ("direct", "bulk"):
        c = cache.to(DEV)
        inj = [rc.DonorInjection(dk.to(DEV), bt.to(DEV), dp.to(DEV), tp.to(DEV)) for dk, bt, dp, tp in host]
        rc.inject_donors(c, inj, rope_base=1e6, rotary_style="neox", staging=staging)
        outs.append(c.cpu())
    assert torch.equal(outs[0].view(torch.uint8), outs[1].view(torch.uint8))
    donor, bt, dp, tp = host[7]
    for layer in range(L):
        want = orope.rope_correct_scatter_paged(cache[layer], donor[layer], bt, dp, tp, 1e6, "neox")
        rows = bt.long()
        _split_check(outs[1][layer][rows], want[rows], style="neox")


def test_c1_full_size_bulk_staging():
    import bench

    donor, cache, bt, d, t = bench.make_c1_inputs(bench.SEED + 1)
    want = orope.rope_correct_scatter_paged(cache, donor, bt, d, t, 1e6, "neox")
    c = cache.to(DEV)
    rc.rope_correct_scatter_paged(c, donor.to(DEV), bt.to(DEV), d.to(DEV), t.to(DEV), rope_base=1e6,
                                  rotary_style="neox", staging="bulk")
    _split_check(c, want, style="neox")
    _untouched_exact(c, cache, bt, t)
