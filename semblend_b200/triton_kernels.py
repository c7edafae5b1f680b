"""Partial-prefill kernels — drop-in for ``semblend_core.triton_kernels``.

Same public names, signatures and return conventions as the reference module
(semblend_core/triton_kernels.py, SemBlend 0.3.2).  Despite the module name
(kept so existing imports resolve), nothing here uses Triton: every entry point
runs a hand-written sm_100a kernel of ``libsemblend_b200``.  CPU tensors raise
:class:`~semblend_b200._lib.NativeLibraryError`; there is no CPU path.
"""

from __future__ import annotations

import math

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


def _attn_tensor(t: torch.Tensor) -> _lib.SbAttnTensor:
    """[B, H, S, D] view with a contiguous last dim as an sb_attn_tensor."""
    if t.stride(-1) != 1:
        raise ValueError("attention tensors need a contiguous head dimension")
    a = _lib.SbAttnTensor()
    a.data = t.data_ptr()
    # a size-1 dim may carry any stride: give it the packed one so tensor maps stay well formed
    st = list(t.stride())
    for i in (2, 1, 0):
        if t.shape[i] == 1:
            st[i] = st[i + 1] * t.shape[i + 1]
    a.stride_batch, a.stride_head, a.stride_seq = st[0], st[1], st[2]
    return a


def mask_to_rows(compute_mask: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Compact a ``[B, S]`` (or ``[S]``) bool mask into ascending row indices
    ``[B, S]`` (int32, valid up to ``counts[b]``) and ``counts [B]`` on the
    device, without synchronising (``sb_mask_to_rows``)."""
    _lib.require_cuda(compute_mask, "compute_mask")
    m = compute_mask if compute_mask.ndim == 2 else compute_mask.unsqueeze(0)
    m = m.to(torch.uint8).contiguous()
    B, S = m.shape
    rows = torch.empty(B, max(S, 1), dtype=torch.int32, device=m.device)
    counts = torch.empty(B, dtype=torch.int32, device=m.device)
    lib = _lib.load()
    _lib.check(lib.sb_mask_to_rows(m.data_ptr(), S, B, S, rows.data_ptr(), rows.shape[1], counts.data_ptr(),
                                   _lib.stream_ptr(m.device)), "sb_mask_to_rows")
    return rows, counts


def gqa_partial_attention(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    rows: torch.Tensor,
    counts: torch.Tensor,
    out: torch.Tensor,
    scale: float | None = None,
    max_rows: int | None = None,
    status: torch.Tensor | None = None,
) -> torch.Tensor:
    """Causal attention at compacted rows with grouped-query heads.

    ``query``/``out`` ``[B, Hq, S, D]``, ``key``/``value`` ``[B, Hkv, S, D]``
    (``Hq % Hkv == 0``; query head h reads KV head ``h // (Hq // Hkv)``),
    ``rows [B, R]`` ascending positions valid up to ``counts[b]``.  Writes
    ``out`` at those rows only and returns it.  bf16 / fp16 with D = 128 run
    on the tensor cores; fp32 and other head dims on CUDA cores.  ``status``
    (device int32) receives a value >= 2 if a kernel wait timed out.
    """
    for t, n in ((query, "query"), (key, "key"), (value, "value"), (out, "out"), (rows, "rows"), (counts, "counts")):
        _lib.require_cuda(t, n)
    B, Hq, S, D = query.shape
    Hkv = key.shape[1]
    if key.shape != (B, Hkv, S, D) or value.shape != key.shape or out.shape != query.shape:
        raise ValueError(f"shape mismatch: q {tuple(query.shape)} k {tuple(key.shape)} v {tuple(value.shape)}")
    if Hq % Hkv:
        raise ValueError(f"{Hq} query heads are not a multiple of {Hkv} KV heads")
    if not (query.dtype == key.dtype == value.dtype == out.dtype):
        raise TypeError("query, key, value and out must share a dtype")
    if rows.dtype != torch.int32 or counts.dtype != torch.int32:
        raise TypeError("rows and counts must be int32")
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if max_rows is None:
        max_rows = rows.shape[1]
    dev = query.device
    if status is None:
        status = torch.zeros(1, dtype=torch.int32, device=dev)
    lib = _lib.load()
    _lib.check(
        lib.sb_partial_attention(
            _attn_tensor(query), _attn_tensor(key), _attn_tensor(value), _attn_tensor(out),
            rows.data_ptr(), rows.stride(0) if rows.shape[0] > 1 else rows.shape[1], counts.data_ptr(),
            int(max_rows), B, Hq, Hkv, S, D, float(scale), _lib.dtype_code(query.dtype), status.data_ptr(),
            _lib.stream_ptr(dev),
        ),
        "sb_partial_attention",
    )
    return out


def partial_prefill_attention(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    compute_mask: torch.Tensor,
    scale: float | None = None,
) -> torch.Tensor:
    """Causal attention only at compute-mask rows; other rows are zero.

    Mirrors semblend_core/triton_kernels.py:655-734: ``query``/``key``/
    ``value`` ``[H, S, D]``, ``compute_mask [S]`` bool, returns
    ``[H, S, D]`` in the query's dtype.  Extensions: ``key``/``value`` may
    have fewer heads than ``query`` (grouped-query attention), and a leading
    batch dimension (``[B, H, S, D]`` with a ``[B, S]`` mask) is accepted.
    The compacted rows are built on the device (no ``.item()`` sync on the
    tensor-core path).
    """
    batched = query.ndim == 4
    q = query if batched else query.unsqueeze(0)
    k = key if batched else key.unsqueeze(0)
    v = value if batched else value.unsqueeze(0)
    _lib.require_cuda(q, "query")
    output = torch.zeros_like(q)
    S, D = q.shape[2], q.shape[3]
    if S == 0:
        return output if batched else output[0]
    rows, counts = mask_to_rows(compute_mask)
    tc_path = q.dtype in (torch.float16, torch.bfloat16) and D == 128
    max_rows = S if tc_path else int(counts.max().item())
    if max_rows > 0:
        gqa_partial_attention(q, k.to(q.dtype), v.to(q.dtype), rows, counts, output, scale, max_rows=max_rows)
    return output if batched else output[0]


__all__ = [
    "HAS_TRITON",
    "gqa_partial_attention",
    "mask_to_rows",
    "partial_prefill_attention",
    "scatter_donor_kv",
    "scatter_donor_kv_paged",
]
