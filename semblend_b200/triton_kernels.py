"""Partial-prefill kernels — drop-in for ``semblend_core.triton_kernels``.

Same public names, signatures and return conventions as the reference module
(semblend_core/triton_kernels.py, SemBlend 0.3.2).  Despite the module name
(kept so existing imports resolve), nothing here uses Triton: every entry point
runs a hand-written sm_100a kernel of ``libsemblend_b200``.  CPU tensors raise
:class:`~semblend_b200._lib.NativeLibraryError`; there is no CPU path.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

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
    layout: str = "auto",
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


def masked_qkv_projection(
    hidden_states: torch.Tensor,
    qkv_weight: torch.Tensor,
    compute_mask: torch.Tensor,
    qkv_bias: torch.Tensor | None = None,
    status: torch.Tensor | None = None,
) -> torch.Tensor:
    """``hidden_states @ qkv_weight^T (+ qkv_bias)`` at compute-mask rows; reuse rows are zero.

    Mirrors semblend_core/triton_kernels.py:451-522 (fp32 accumulation, one
    rounding to the input dtype), but multiplies only the compute rows: bf16 /
    fp16 run a tcgen05 GEMM over the compacted rows (``sb_masked_linear``),
    fp32 (and 16-bit hidden sizes that are not a multiple of 8) a CUDA-core
    kernel.  ``status`` (device int32) receives a value >= 2 if a kernel wait
    timed out.
    """
    _lib.require_cuda(hidden_states, "hidden_states")
    S, K = hidden_states.shape
    N = qkv_weight.shape[0]
    if qkv_weight.shape[1] != K:
        raise ValueError(f"qkv_weight {tuple(qkv_weight.shape)} does not match hidden_states {tuple(hidden_states.shape)}")
    dt = hidden_states.dtype
    w = qkv_weight.to(dt).contiguous()
    b = qkv_bias.to(dt).contiguous() if qkv_bias is not None else None
    x = hidden_states if hidden_states.stride(1) == 1 else hidden_states.contiguous()
    out = torch.zeros(S, N, dtype=dt, device=x.device)
    if S == 0:
        return out
    rows, counts = mask_to_rows(compute_mask.reshape(-1)[:S].to(x.device))
    n = int(counts[0].item())
    if n == 0:
        return out
    lib = _lib.load()
    code = _lib.dtype_code(dt)
    ws_bytes = lib.sb_masked_linear_workspace_bytes(n, K, code)
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=x.device)
    if status is None:
        status = torch.zeros(1, dtype=torch.int32, device=x.device)
    ldx = x.stride(0) if S > 1 else K
    _lib.check(
        lib.sb_masked_linear(x.data_ptr(), ldx, w.data_ptr(), K, b.data_ptr() if b is not None else None,
                             rows.data_ptr(), n, N, K, out.data_ptr(), N, code, ws.data_ptr(), ws_bytes,
                             status.data_ptr(), _lib.stream_ptr(x.device)),
        "sb_masked_linear",
    )
    return out


@dataclass
class PartialPrefillResult:
    """Result of :func:`partial_prefill` (semblend_core/triton_kernels.py:742-766)."""

    output: torch.Tensor
    kv_cache: torch.Tensor
    positions_computed: int
    positions_reused: int
    computation_ratio: float
    scatter_time_ms: float
    projection_time_ms: float
    attention_time_ms: float
    total_time_ms: float


def partial_prefill(
    hidden_states: torch.Tensor,
    donor_kv: torch.Tensor,
    qkv_weight: torch.Tensor,
    output_projection: torch.Tensor,
    donor_positions: torch.Tensor,
    target_positions: torch.Tensor,
    compute_mask: torch.Tensor,
    num_heads: int,
    head_dim: int,
    qkv_bias: torch.Tensor | None = None,
    output_bias: torch.Tensor | None = None,
    scale: float | None = None,
) -> PartialPrefillResult:
    """Scatter donor KV, project only the compute rows, attend, project out.

    Mirrors the reference orchestrator (semblend_core/triton_kernels.py:769-923)
    step for step: a zero target cache ``[L, 2, H, S, D]``, donor rows
    scattered into it, the masked QKV projection, layer 0's K/V merged with
    the new rows in fp32, causal attention at the compute rows (fp32), the
    output projection in fp32 (a plain library GEMM: outside the kernels this
    package replaces), reuse rows zeroed, and the new K/V written into every
    layer; CUDA-event timings per stage.
    """
    _lib.require_cuda(hidden_states, "hidden_states")
    seq_len = hidden_states.shape[0]
    num_layers = donor_kv.shape[0]
    device = hidden_states.device
    if scale is None:
        scale = 1.0 / math.sqrt(head_dim)
    target_kv = torch.zeros((num_layers, 2, num_heads, seq_len, head_dim), dtype=hidden_states.dtype, device=device)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
    ev[0].record()
    scatter_donor_kv(target_kv, donor_kv.to(target_kv.dtype), donor_positions, target_positions)
    ev[1].record()
    qkv = masked_qkv_projection(hidden_states, qkv_weight, compute_mask, qkv_bias)
    qkv = qkv.float().view(seq_len, 3, num_heads, head_dim)
    q_new = qkv[:, 0].permute(1, 0, 2)
    k_new = qkv[:, 1].permute(1, 0, 2)
    v_new = qkv[:, 2].permute(1, 0, 2)
    ev[2].record()
    compute_indices = torch.where(compute_mask)[0]
    merged_k = target_kv[0, 0].float().clone()
    merged_v = target_kv[0, 1].float().clone()
    if compute_indices.numel() > 0:
        merged_k[:, compute_indices, :] = k_new[:, compute_indices, :]
        merged_v[:, compute_indices, :] = v_new[:, compute_indices, :]
    attn = partial_prefill_attention(q_new.contiguous(), merged_k, merged_v, compute_mask, scale)
    ev[3].record()
    final = torch.nn.functional.linear(
        attn.permute(1, 0, 2).reshape(seq_len, num_heads * head_dim), output_projection.float(),
        output_bias.float() if output_bias is not None else None,
    ).to(hidden_states.dtype)
    reuse_indices = torch.where(~compute_mask)[0]
    if reuse_indices.numel() > 0:
        final[reuse_indices] = 0.0
    if compute_indices.numel() > 0:
        for layer in range(num_layers):
            target_kv[layer, 0, :, compute_indices, :] = k_new[:, compute_indices, :].to(target_kv.dtype)
            target_kv[layer, 1, :, compute_indices, :] = v_new[:, compute_indices, :].to(target_kv.dtype)
    ev[4].record()
    torch.cuda.synchronize(device)
    n_comp = int(compute_mask.sum().item())
    return PartialPrefillResult(
        output=final, kv_cache=target_kv, positions_computed=n_comp, positions_reused=seq_len - n_comp,
        computation_ratio=n_comp / seq_len if seq_len > 0 else 1.0,
        scatter_time_ms=ev[0].elapsed_time(ev[1]), projection_time_ms=ev[1].elapsed_time(ev[2]),
        attention_time_ms=ev[2].elapsed_time(ev[3]), total_time_ms=ev[0].elapsed_time(ev[4]),
    )


__all__ = [
    "HAS_TRITON",
    "PartialPrefillResult",
    "masked_qkv_projection",
    "partial_prefill",
    "gqa_partial_attention",
    "mask_to_rows",
    "partial_prefill_attention",
    "scatter_donor_kv",
    "scatter_donor_kv_paged",
]
