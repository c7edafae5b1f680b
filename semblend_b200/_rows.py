"""Tensor → ``sb_rows`` descriptors for the KV layouts the hot path meets.

A paged KV cache is addressed by (block, kv, head, position-in-block, dim)
strides, so every layout is a stride permutation of the same rows:

==============  =============================  ===============================
layout          per-layer shape                used by
==============  =============================  ===============================
``canonical``   ``[nb, 2, H, bs, D]``          the reference kernels
                                               (semblend_core/rope_correction.py:212)
``vllm``        ``[2, nb, bs, H, D]``          vLLM FlashAttention backend
``trtllm``      ``[nb, 2, bs, H, D]``          TensorRT-LLM paged cache
                                               (semblend/integration/trtllm/
                                               kv_cache_adapter.py:10-16)
==============  =============================  ===============================

A leading layer dimension (``[L, *per_layer]``) or a list of per-layer tensors
lets one launch cover every layer.
"""

from __future__ import annotations

import threading
from collections.abc import Sequence

import torch

from . import _lib

LAYOUTS = ("canonical", "vllm", "trtllm")

# (block, kv, head, pos, dim) axis of each layout's per-layer tensor
_AXES = {
    "canonical": (0, 1, 2, 3, 4),
    "vllm": (1, 0, 3, 2, 4),
    "trtllm": (0, 1, 3, 2, 4),
}

_ptr_lock = threading.Lock()
_ptr_tables: dict[tuple, torch.Tensor] = {}


def detect_layout(kv_cache: torch.Tensor) -> str:
    """The reference's auto-detection (semblend_core/rope_correction.py:740):
    ``[2, nb, bs, H, D]`` with ``nb != 2`` is vLLM's layout, else canonical."""
    if kv_cache.ndim == 5 and kv_cache.shape[0] == 2 and kv_cache.shape[1] != 2:
        return "vllm"
    return "canonical"


def resolve_layout(kv_cache: torch.Tensor, layout: str) -> str:
    if layout == "auto":
        return detect_layout(kv_cache)
    if layout not in LAYOUTS:
        raise ValueError(f"unknown KV layout {layout!r}; expected one of {LAYOUTS} or 'auto'")
    return layout


def paged_geometry(per_layer_shape: Sequence[int], layout: str) -> tuple[int, int, int, int]:
    """(num_blocks, num_heads, block_size, head_dim) of a per-layer cache shape."""
    if len(per_layer_shape) != 5:
        raise ValueError(f"paged KV cache must be 5-D per layer, got shape {tuple(per_layer_shape)}")
    b, kv, h, p, d = _AXES[layout]
    if per_layer_shape[kv] != 2:
        raise ValueError(
            f"paged KV cache {tuple(per_layer_shape)} has no K/V axis of size 2 for layout {layout!r}"
        )
    return per_layer_shape[b], per_layer_shape[h], per_layer_shape[p], per_layer_shape[d]


def _layer_ptr_table(tensors: Sequence[torch.Tensor], device: torch.device) -> torch.Tensor:
    key = (device.index,) + tuple(t.data_ptr() for t in tensors)
    t = _ptr_tables.get(key)
    if t is None:
        for x in tensors:
            if x.data_ptr() % 16:
                raise ValueError("per-layer KV tensors must be 16-byte aligned")
        t = torch.tensor([x.data_ptr() for x in tensors], dtype=torch.int64).to(device)
        with _ptr_lock:
            if len(_ptr_tables) > 256:
                _ptr_tables.clear()
            _ptr_tables[key] = t
    return t


def paged_rows(
    kv_cache: torch.Tensor | Sequence[torch.Tensor],
    block_table: torch.Tensor,
    layout: str,
    *,
    has_layer_dim: bool = False,
) -> tuple[_lib.SbRows, tuple[int, int, int, int, int], list]:
    """Describe a paged cache.

    Returns the descriptor, ``(n_layers, num_blocks, num_heads, block_size,
    head_dim)`` and a list of tensors that must stay alive for the call.
    """
    keep: list = []
    if isinstance(kv_cache, (list, tuple)):
        layers = list(kv_cache)
        if not layers:
            raise ValueError("empty list of per-layer KV caches")
        ref = layers[0]
        for t in layers[1:]:
            if t.shape != ref.shape or t.stride() != ref.stride() or t.dtype != ref.dtype:
                raise ValueError("per-layer KV caches must share shape, strides and dtype")
        per_shape, per_stride = ref.shape, ref.stride()
        n_layers = len(layers)
        ptrs = _layer_ptr_table(layers, ref.device)
        keep.append(ptrs)
        base, layer_ptrs, stride_layer = ref.data_ptr(), ptrs.data_ptr(), 0
    else:
        if has_layer_dim:
            per_shape, per_stride = kv_cache.shape[1:], kv_cache.stride()[1:]
            n_layers, stride_layer = kv_cache.shape[0], kv_cache.stride(0)
        else:
            per_shape, per_stride = kv_cache.shape, kv_cache.stride()
            n_layers, stride_layer = 1, 0
        base, layer_ptrs = kv_cache.data_ptr(), None
    nb, nh, bs, hd = paged_geometry(per_shape, layout)
    b, kv, h, p, d = _AXES[layout]
    # a dimension of size 1 is only ever indexed at 0 and may carry any stride
    per_stride = [0 if n == 1 else st for n, st in zip(per_shape, per_stride)]
    if n_layers == 1:
        stride_layer = 0
    rows = _lib.SbRows()
    rows.base = base
    rows.layer_ptrs = layer_ptrs
    rows.stride_layer = stride_layer
    rows.stride_block = per_stride[b]
    rows.stride_kv = per_stride[kv]
    rows.stride_head = per_stride[h]
    rows.stride_pos = per_stride[p]
    rows.stride_dim = per_stride[d]
    rows.block_table = block_table.data_ptr()
    rows.n_logical = block_table.shape[0]
    rows.n_physical = nb
    rows.block_size = bs
    rows.block_table_dtype = _lib.index_code(block_table.dtype)
    return rows, (n_layers, nb, nh, bs, hd), keep


def flat_rows(
    t: torch.Tensor,
    *,
    layer_axis: int | None,
    kv_axis: int | None,
    head_axis: int,
    pos_axis: int,
    dim_axis: int,
) -> _lib.SbRows:
    """Describe a flat (unpaged) KV tensor by the axes of its dimensions."""
    s = [0 if n == 1 else st for n, st in zip(t.shape, t.stride())]  # size-1 dims: any stride
    rows = _lib.SbRows()
    rows.base = t.data_ptr()
    rows.layer_ptrs = None
    rows.stride_layer = s[layer_axis] if layer_axis is not None else 0
    rows.stride_block = 0
    rows.stride_kv = s[kv_axis] if kv_axis is not None else 0
    rows.stride_head = s[head_axis]
    rows.stride_pos = s[pos_axis]
    rows.stride_dim = s[dim_axis]
    rows.block_table = None
    rows.n_logical = t.shape[pos_axis]
    rows.n_physical = 0
    rows.block_size = 0
    rows.block_table_dtype = 0
    return rows


def device_index_tensor(x, device: torch.device, name: str) -> torch.Tensor:
    """Positions / block tables as a contiguous int32 or int64 tensor on ``device``."""
    if not isinstance(x, torch.Tensor):
        x = torch.as_tensor(x)
    if x.dtype not in (torch.int32, torch.int64):
        if x.is_floating_point() or x.dtype == torch.bool:
            raise TypeError(f"{name} must be an integer tensor, got {x.dtype}")
        x = x.to(torch.int64)
    if x.device != device:
        x = x.to(device, non_blocking=True)
    return x.contiguous()


def params(
    *,
    n_layers: int,
    n_heads: int,
    head_dim: int,
    dtype: torch.dtype,
    rotary_style: str,
    k_angle: int,
    kv_select: int,
    inv_freq: torch.Tensor | None,
    const_delta: int = 0,
    staging: str = "direct",
) -> _lib.SbInjectParams:
    if staging not in ("direct", "bulk"):
        raise ValueError(f"staging must be 'direct' or 'bulk', got {staging!r}")
    p = _lib.SbInjectParams()
    p.flags = _lib.SB_INJECT_BULK_STAGED if staging == "bulk" else 0
    p.n_layers = n_layers
    p.n_heads = n_heads
    p.head_dim = head_dim
    p.dtype = _lib.dtype_code(dtype)
    p.rotary_style = rotary_code(rotary_style)
    p.k_angle = k_angle
    p.kv_select = kv_select
    p.const_delta = const_delta
    p.inv_freq = inv_freq.data_ptr() if inv_freq is not None else None
    return p


def rotary_code(style: str) -> int:
    if style == "interleaved":
        return _lib.SB_ROTARY_INTERLEAVED
    if style == "neox":
        return _lib.SB_ROTARY_NEOX
    raise ValueError(f"rotary_style must be 'interleaved' or 'neox', got {style!r}")
