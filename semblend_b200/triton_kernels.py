"""Partial-prefill kernels — drop-in for ``semblend_core.triton_kernels``.

Same public names, signatures and return conventions as the reference module
(semblend_core/triton_kernels.py, SemBlend 0.3.2).  Despite the module name
(kept so existing imports resolve), nothing here uses Triton: every entry point
runs a hand-written sm_100a kernel of ``libsemblend_b200``.  CPU tensors raise
:class:`~semblend_b200._lib.NativeLibraryError`; there is no CPU path.
"""

from __future__ import annotations

import torch

from . import _lib, _rows
from .rope_correction import _donor_rows, _launch, _pair_desc, _positions

HAS_TRITON = False  # kept for import compatibility; no Triton is used


def scatter_donor_kv(
    target: torch.Tensor,
    donor: torch.Tensor,
    donor_positions: torch.Tensor,
    target_positions: torch.Tensor,
) -> torch.Tensor:
    """Copy donor K,V rows into a flat target cache at position pairs.

    Mirrors semblend_core/triton_kernels.py:132-191: ``target`` is
    ``[L, 2, H, target_len, D]`` and ``donor`` ``[L, 2, H, donor_len, D]``;
    every layer, K/V and head row of each pair is copied bit for bit.  Pairs
    with a donor or target position out of range are skipped (:106-108).
    Modified in place and returned.
    """
    if donor_positions.shape[0] == 0:
        return target
    _lib.require_cuda(target, "target")
    _lib.require_cuda(donor, "donor")
    if target.ndim != 5 or donor.ndim != 5:
        raise ValueError("target and donor must be [L, 2, H, S, D]")
    L, two, H, _, D = target.shape
    if donor.shape[0] != L or donor.shape[1] != 2 or two != 2 or donor.shape[2] != H or donor.shape[4] != D:
        raise ValueError(f"donor shape {tuple(donor.shape)} does not match target {tuple(target.shape)}")
    if donor.dtype != target.dtype:
        raise TypeError(f"donor dtype {donor.dtype} differs from target dtype {target.dtype}")
    dev = target.device
    sp, tp = _positions(donor_positions, target_positions, dev)
    src = _rows.flat_rows(donor, layer_axis=0, kv_axis=1, head_axis=2, pos_axis=3, dim_axis=4)
    dst = _rows.flat_rows(target, layer_axis=0, kv_axis=1, head_axis=2, pos_axis=3, dim_axis=4)
    desc = _pair_desc(src, dst, sp, tp, _lib.SB_ROW_AT_SRC_POS, _lib.SB_ROW_AT_DST_POS)
    p = _rows.params(
        n_layers=L, n_heads=H, head_dim=D, dtype=target.dtype, rotary_style="interleaved",
        k_angle=_lib.SB_ANGLE_NONE, kv_select=_lib.SB_KV_BOTH, inv_freq=None,
    )
    _launch([desc], p, dev, "scatter_donor_kv")
    return target


def scatter_donor_kv_paged(
    kv_cache: torch.Tensor,
    donor_kv: torch.Tensor,
    block_table: torch.Tensor,
    donor_positions: torch.Tensor,
    target_positions: torch.Tensor,
    *,
    layout: str = "canonical",
) -> torch.Tensor:
    """Copy donor K,V rows into a paged cache through the block table.

    Mirrors semblend_core/triton_kernels.py:279-356: ``kv_cache`` is
    ``[num_blocks, 2, H, block_size, D]`` (or ``layout``), ``donor_kv``
    ``[2, H, donor_len, D]``.  Pairs whose donor position, logical block or
    physical block is out of range are skipped (:246-260).  Modified in place
    and returned.
    """
    if donor_positions.shape[0] == 0:
        return kv_cache
    _lib.require_cuda(kv_cache, "kv_cache")
    _lib.require_cuda(donor_kv, "donor_kv")
    layout = _rows.resolve_layout(kv_cache, layout)
    dev = kv_cache.device
    bt = _rows.device_index_tensor(block_table, dev, "block_table")
    dst, (_, _, nh, _, hd), keep = _rows.paged_rows(kv_cache, bt, layout)
    if donor_kv.ndim != 4 or donor_kv.shape[0] != 2 or donor_kv.shape[1] != nh or donor_kv.shape[3] != hd:
        raise ValueError(f"donor_kv must be [2, {nh}, donor_len, {hd}], got {tuple(donor_kv.shape)}")
    if donor_kv.dtype != kv_cache.dtype:
        raise TypeError(f"donor_kv dtype {donor_kv.dtype} differs from kv_cache dtype {kv_cache.dtype}")
    sp, tp = _positions(donor_positions, target_positions, dev)
    desc = _pair_desc(_donor_rows(donor_kv, False), dst, sp, tp, _lib.SB_ROW_AT_SRC_POS, _lib.SB_ROW_AT_DST_POS)
    p = _rows.params(
        n_layers=1, n_heads=nh, head_dim=hd, dtype=kv_cache.dtype, rotary_style="interleaved",
        k_angle=_lib.SB_ANGLE_NONE, kv_select=_lib.SB_KV_BOTH, inv_freq=None,
    )
    _launch([desc], p, dev, "scatter_donor_kv_paged")
    del keep
    return kv_cache


__all__ = [
    "HAS_TRITON",
    "scatter_donor_kv",
    "scatter_donor_kv_paged",
]
