"""Device position mappings and the vLLM hook's permutation calls on the GPU.

Covers :class:`semblend_b200.position_mapping.DevicePositionMapping` (host
round trips, per-donor selection, a chunk alignment's pairs driving the
permutation and the inject without visiting the host) and the calls the
reference's RoPE hook makes (synapse_kv_connector/model_runner_hook.py:495-555):
per-layer vLLM caches ``[2, num_blocks, block_size, H, D]`` passed with no
``layout``, which the default ``layout="auto"`` serves.  Results are checked
against the CPU oracle (V and untouched rows bit-exact, K within 1 ulp at its
RoPE pair's magnitude).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import rope as orope
from semblend_b200 import _lib
from semblend_b200 import rope_correction as rc
from semblend_b200.alignment import chunk_alignment
from semblend_b200.position_mapping import DevicePositionMapping, MultiDonorPositionMapping, PositionMapping
from tests.helpers import assert_rope_close

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


@pytest.fixture(autouse=True)
def _reset_counter():
    _lib.skipped_pairs(DEV, reset=True)
    yield


def _check(got: torch.Tensor, want: torch.Tensor, layout: str, style: str = "interleaved"):
    g = orope.canonical_view(got.cpu(), layout)
    w = orope.canonical_view(want, layout)
    assert torch.equal(g[:, 1].contiguous().view(torch.int16), w[:, 1].contiguous().view(torch.int16))
    assert_rope_close(g[:, 0].contiguous(), w[:, 0].contiguous(), style)


def test_host_round_trip_and_for_donor():
    pm = PositionMapping([5, 6, 7, 100], [0, 1, 2, 3])
    dm = DevicePositionMapping.from_host(pm, DEV)
    assert dm.num_pairs == 4 and dm.needs_correction and dm.to_host() == pm
    assert dm.donor_positions.dtype == torch.int32 and dm.donor_positions.device == DEV
    md = MultiDonorPositionMapping(("a", "b", "a", "c", "b"), (1, 2, 3, 4, 5), (10, 20, 30, 40, 50))
    dmd = DevicePositionMapping.from_host(md, DEV)
    assert dmd.donor_ids == ("a", "b", "c") and dmd.to_host() == md
    for did in ("a", "b", "c", "zz"):
        sub = dmd.for_donor(did)
        want = md.for_donor(did)
        assert sub.num_pairs == want.num_pairs
        assert sub.donor_positions.cpu().tolist() == list(want.donor_positions)
        assert sub.target_positions.cpu().tolist() == list(want.target_positions)
    same = DevicePositionMapping.from_host(PositionMapping([3, 4], [3, 4]), DEV)
    assert not same.needs_correction


def _chunked_case(seed: int, chunk: int = 64, n_chunks: int = 12):
    """A donor and a target made of the donor's chunks in another order, plus
    fresh chunks; the target's chunk alignment gives the pairs."""
    rng = np.random.default_rng(seed)
    donor = rng.integers(0, 50000, chunk * n_chunks)
    order = [4, 5, 6, 7, 0, 1, 2, 3, 10, 11]
    target = np.concatenate([donor[i * chunk:(i + 1) * chunk] for i in order] + [rng.integers(0, 50000, chunk)])
    return donor, target


def test_alignment_pairs_drive_the_permutation_on_device():
    """A chunk alignment's -1 padded pair arrays go straight into the in-place
    permutation: the result equals the oracle run on the same pairs read back
    to the host, and the padding is skipped (and counted)."""
    chunk = 64
    donor_tok, target_tok = _chunked_case(1, chunk)
    a = chunk_alignment(donor_tok.tolist(), target_tok.tolist(), chunk, context_gate=True, device=DEV)
    dm = DevicePositionMapping.from_alignment(a)
    n = dm.num_pairs
    assert n == 10 * chunk and dm.needs_correction
    g = torch.Generator().manual_seed(2)
    H, D, bs, nb = 4, 128, 16, 80
    cache = torch.randn(nb, 2, H, bs, D, generator=g).to(torch.bfloat16)
    # the donor's rows sit in this cache in donor order: the table covers both sequences
    bt = torch.randperm(nb, generator=g)[: (max(len(donor_tok), len(target_tok)) + bs - 1) // bs].to(torch.int32)
    d, t = dm.donor_positions[:n].cpu(), dm.target_positions[:n].cpu()
    want = orope.permute_paged_kv_with_rope(cache, bt, list(zip(d.tolist(), t.tolist())), 1e6, "neox")
    c = cache.to(DEV)
    rc.permute_paged_kv_with_rope(c, bt.to(DEV), dm, rope_base=1e6, rotary_style="neox")
    _check(c, want, "canonical", "neox")
    assert _lib.skipped_pairs(DEV) == dm.donor_positions.numel() - n  # the -1 padding


def test_injection_from_mapping_matches_oracle():
    chunk = 64
    donor_tok, target_tok = _chunked_case(3, chunk)
    a = chunk_alignment(donor_tok.tolist(), target_tok.tolist(), chunk, context_gate=False, device=DEV)
    dm = DevicePositionMapping.from_alignment(a)
    n = dm.num_pairs
    g = torch.Generator().manual_seed(4)
    L, H, D, bs, nb = 3, 2, 128, 16, 64
    donor = torch.randn(L, 2, H, len(donor_tok), D, generator=g).to(torch.bfloat16)
    cache = torch.randn(L, nb, 2, H, bs, D, generator=g).to(torch.bfloat16)
    bt = torch.randperm(nb, generator=g)[:48].to(torch.int32)
    d, t = dm.donor_positions[:n].cpu(), dm.target_positions[:n].cpu()
    c = cache.to(DEV)
    rc.inject_donors(c, [rc.DonorInjection.from_mapping(donor.to(DEV), bt.to(DEV), dm)], rope_base=1e6,
                     rotary_style="neox")
    for layer in range(L):
        want = orope.rope_correct_scatter_paged(cache[layer], donor[layer], bt, d, t, 1e6, "neox")
        _check(c[layer], want, "canonical", "neox")


def _hook_calls(kv_caches, block_table, pos_map, plan_recompute, rope_base):
    """The permutation calls the reference's RoPECorrectionHook.apply_rope_correction
    makes (model_runner_hook.py:495-555, delta mode): pairs whose positions
    differ, every layer the plan does not recompute in full, keyword arguments
    and no layout."""
    pairs = [(int(d), int(t)) for d, t in zip(pos_map.donor_positions, pos_map.target_positions) if d != t]
    corrected = []
    for layer, kv_cache in enumerate(kv_caches):
        if plan_recompute[layer]:
            continue
        rc.permute_paged_kv_with_rope(kv_cache=kv_cache, block_table=block_table, permutation=pairs,
                                      rope_base=rope_base)
        corrected.append(layer)
    return pairs, corrected


def test_vllm_hook_calls_without_layout():
    """An unchanged vLLM hook hands over per-layer caches in vLLM's
    [2, num_blocks, block_size, H, D] layout without a layout argument: the
    default layout="auto" reads them as vLLM's and the result equals the
    oracle's permutation in that layout (the reference's own permutation
    unpacks this shape as canonical and fails on it)."""
    g = torch.Generator().manual_seed(9)
    L, H, D, bs, nb = 4, 8, 128, 16, 40
    caches = [torch.randn(2, nb, bs, H, D, generator=g).to(torch.bfloat16) for _ in range(L)]
    bt = torch.randperm(nb, generator=g)[:24].to(torch.int32)
    rng = np.random.default_rng(9)
    tgt = rng.permutation(24 * bs)[:200]
    src = rng.permutation(24 * bs)[:200]
    src[:20] = tgt[:20]  # unmoved pairs: the hook drops them
    pm = PositionMapping(src.tolist(), tgt.tolist())
    recompute = [False, True, False, False]
    dev_caches = [c.to(DEV) for c in caches]
    pairs, corrected = _hook_calls(dev_caches, bt.to(DEV), pm, recompute, 5e5)
    assert corrected == [0, 2, 3] and len(pairs) == int((src != tgt).sum()) and len(pairs) <= 180
    for layer in range(L):
        if recompute[layer]:
            assert torch.equal(dev_caches[layer].cpu(), caches[layer])
            continue
        want = orope.permute_paged_kv_with_rope(caches[layer], bt, pairs, 5e5, "interleaved", layout="vllm")
        _check(dev_caches[layer], want, "vllm")
