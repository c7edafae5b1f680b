"""The allocation-free permutation entry point, called through the C ABI.

sb_permute_paged_noalloc exists for callers that cannot allocate device
memory when they permute (an engine hook inside the forward pass whose memory
pool is already sized, a step being captured into a CUDA graph, or a C / Go /
Java caller with no caching allocator): it keeps the source-row snapshot in a
fixed scratch array inside the library instead of a caller workspace.  Its
output must equal sb_permute_paged's on the same inputs, including on a second
call that reuses the scratch left behind by the first.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from semblend_b200 import _lib, _rows

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _case(seed: int, dtype: torch.dtype, H: int, n_pairs: int, style: str):
    g = torch.Generator().manual_seed(seed)
    nb, bs, D = 48, 16, 128
    cache = torch.randn(nb, 2, H, bs, D, generator=g).to(dtype).to(DEV)
    bt = torch.randperm(nb, generator=g)[:40].to(torch.int32).to(DEV)
    perm = np.random.default_rng(seed).permutation(40 * bs)[:n_pairs]
    assert perm.shape[0] == n_pairs, "the C calls read n_pairs positions: the arrays must hold that many"
    src = torch.from_numpy(np.sort(perm).astype(np.int32)).to(DEV)
    dst = torch.from_numpy(perm.astype(np.int32)).to(DEV)  # sources overlap targets
    rows, (n_layers, _, nh, _, hd), keep = _rows.paged_rows(cache, bt, "canonical")
    p = _rows.params(n_layers=n_layers, n_heads=nh, head_dim=hd, dtype=dtype, rotary_style=style,
                     k_angle=_lib.SB_ANGLE_DELTA, kv_select=_lib.SB_KV_BOTH,
                     inv_freq=_lib.inv_freq(1e6, hd, DEV))
    return cache, bt, src, dst, rows, p, keep


def _run_both(seed, dtype, H, n_pairs, style):
    lib = _lib.load()
    stream = _lib.stream_ptr(DEV)
    cache, bt, src, dst, rows, p, keep = _case(seed, dtype, H, n_pairs, style)
    ref = cache.clone()
    rows_ref, _, keep_ref = _rows.paged_rows(ref, bt, "canonical")
    ws_bytes = lib.sb_permute_workspace_bytes(n_pairs, 1, H, 128, p.dtype)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=DEV)
    assert lib.sb_permute_paged(rows_ref, src.data_ptr(), dst.data_ptr(), n_pairs, _lib.SB_INDEX_I32, p,
                                ws.data_ptr(), ws_bytes, None, stream) == _lib.SB_OK
    assert lib.sb_permute_paged_noalloc(rows, src.data_ptr(), dst.data_ptr(), n_pairs, _lib.SB_INDEX_I32, p,
                                        None, stream) == _lib.SB_OK
    torch.cuda.synchronize(DEV)
    assert not torch.equal(cache, _case(seed, dtype, H, n_pairs, style)[0])  # the call did permute
    assert torch.equal(cache.view(torch.uint8), ref.view(torch.uint8))
    del keep, keep_ref


def test_noalloc_permute_matches_workspace_entry_point_twice():
    # first call on the device (resolves the scratch address), then a second
    # call with other shapes that reuses the scratch the first left behind
    _run_both(seed=1, dtype=torch.bfloat16, H=4, n_pairs=600, style="neox")
    _run_both(seed=2, dtype=torch.float32, H=8, n_pairs=500, style="interleaved")


def test_noalloc_permute_rejects_oversized_requests():
    lib = _lib.load()
    cache, bt, src, dst, rows, p, keep = _case(3, torch.bfloat16, 4, 16, "neox")
    too_many = _lib.SB_PERMUTE_NOALLOC_SCRATCH_BYTES // (2 * 4 * 128 * 2) + 1
    before = cache.clone()
    st = lib.sb_permute_paged_noalloc(rows, src.data_ptr(), dst.data_ptr(), too_many, _lib.SB_INDEX_I32, p, None,
                                      _lib.stream_ptr(DEV))
    assert st == _lib.SB_ERR_TOO_LARGE
    assert torch.equal(cache, before)
    del keep


def test_noalloc_second_call_with_skipped_pairs_and_layers():
    """A first call leaves its rows in the shared scratch; a second call over a
    three-layer cache, some of whose sources lie beyond the block table or on
    unmapped blocks (entries -1), must still equal sb_permute_paged bit for bit
    and count the same skipped pairs: a skipped source is never read back from
    the stale scratch."""
    lib = _lib.load()
    stream = _lib.stream_ptr(DEV)
    _run_both(seed=4, dtype=torch.bfloat16, H=4, n_pairs=640, style="neox")  # fills the scratch

    g = torch.Generator().manual_seed(5)
    L, nb, H, bs, D, n_log = 3, 48, 2, 16, 128, 30
    cache = torch.randn(L, nb, 2, H, bs, D, generator=g).to(torch.bfloat16).to(DEV)
    bt_h = torch.randperm(nb, generator=g)[:n_log].to(torch.int32)
    bt_h[[3, 17]] = -1  # two unmapped logical blocks
    bt = bt_h.to(DEV)
    rng = np.random.default_rng(5)
    n_pairs = 300
    dst_h = rng.permutation(np.setdiff1d(np.arange(n_log * bs), np.r_[3 * bs:4 * bs, 17 * bs:18 * bs]))[:n_pairs]
    src_h = rng.integers(0, (n_log + 4) * bs, n_pairs)  # some beyond the table, some on unmapped blocks
    src = torch.from_numpy(src_h.astype(np.int32)).to(DEV)
    dst = torch.from_numpy(dst_h.astype(np.int32)).to(DEV)
    lb = src_h // bs
    expect_skipped = int(((lb >= n_log) | np.isin(lb, [3, 17])).sum())
    assert 0 < expect_skipped < n_pairs

    ref = cache.clone()
    rows, (n_layers, _, nh, _, hd), keep = _rows.paged_rows(cache, bt, "canonical", has_layer_dim=True)
    rows_ref, _, keep_ref = _rows.paged_rows(ref, bt, "canonical", has_layer_dim=True)
    assert n_layers == L
    p = _rows.params(n_layers=L, n_heads=nh, head_dim=hd, dtype=torch.bfloat16, rotary_style="neox",
                     k_angle=_lib.SB_ANGLE_DELTA, kv_select=_lib.SB_KV_BOTH, inv_freq=_lib.inv_freq(1e6, hd, DEV))
    err_a = torch.zeros(1, dtype=torch.int64, device=DEV)
    err_b = torch.zeros(1, dtype=torch.int64, device=DEV)
    ws_bytes = lib.sb_permute_workspace_bytes(n_pairs, L, H, D, p.dtype)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=DEV)
    assert lib.sb_permute_paged(rows_ref, src.data_ptr(), dst.data_ptr(), n_pairs, _lib.SB_INDEX_I32, p,
                                ws.data_ptr(), ws_bytes, err_a.data_ptr(), stream) == _lib.SB_OK
    assert lib.sb_permute_paged_noalloc(rows, src.data_ptr(), dst.data_ptr(), n_pairs, _lib.SB_INDEX_I32, p,
                                        err_b.data_ptr(), stream) == _lib.SB_OK
    torch.cuda.synchronize(DEV)
    assert int(err_a.item()) == expect_skipped and int(err_b.item()) == expect_skipped
    assert torch.equal(cache.view(torch.uint8), ref.view(torch.uint8))
    del keep, keep_ref


def test_permute_workspace_bytes_rejects_overflow():
    lib = _lib.load()
    assert lib.sb_permute_workspace_bytes(1 << 40, 1 << 20, 8, 128, _lib.SB_DTYPE_BF16) == -1
    assert lib.sb_permute_workspace_bytes(10, 2, 4, 128, _lib.SB_DTYPE_BF16) == 10 * 2 * 2 * 4 * 128 * 2
