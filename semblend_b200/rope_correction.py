"""RoPE-corrected donor-KV injection — drop-in for ``semblend_core.rope_correction``.

Same entry points, argument meaning and return conventions as the reference
module (semblend_core/rope_correction.py, SemBlend 0.3.2); every call runs the
sm_100a kernel of ``libsemblend_b200`` on the tensors' CUDA device.  There is
no CPU path: CPU tensors raise :class:`~semblend_b200._lib.NativeLibraryError`.

Behaviour kept from the reference:

* K is rotated by ``RoPE(target - donor)`` in fp32 and stored in the cache's
  dtype (the reference's CPU path, rope_correction.py:304-328; its Triton
  kernels store fp16 whatever the cache dtype, :183-188, which is a bug and is
  not reproduced); V is copied unchanged.
* ``theta = fp32(delta) * inv_freq`` with ``inv_freq`` built by the reference's
  own fp32 expression (:235-238); every product and sum is rounded separately.
* Pairs whose donor position, logical block or physical block is out of range
  are skipped (:117-129) and counted (:func:`semblend_b200.skipped_pairs`).
* In-place / returned-tensor conventions and early returns on empty input.

Additions, all keyword-only with reference-compatible defaults:

* ``rotary_style="interleaved" | "neox"`` — the reference rotates interleaved
  pairs ``(2i, 2i+1)``; Qwen/Llama checkpoints served by vLLM use neox
  half-rotation pairs ``(i, i + D/2)``.
* ``layout="auto" | "canonical" | "vllm" | "trtllm"`` for paged caches.  The
  default ``"auto"`` reads a per-layer cache as the reference's canonical
  ``[num_blocks, 2, H, block_size, D]`` unless that reading is impossible
  (dimension 1 is not 2) and the shape is vLLM's ``[2, num_blocks,
  block_size, H, D]`` (the reference's own detection, rope_correction.py:740).
  So every call the canonical reading accepts behaves as in the reference, and
  the vLLM hook's calls, which pass vLLM caches without a layout
  (model_runner_hook.py:538-555) and fail in the reference's permutation
  (rope_correction.py:432 unpacks the shape as canonical), are served.
* :func:`inject_donors` — every layer and every request of a step in one
  launch (the reference issues one launch per layer per request).
"""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib, _rows
from .position_mapping import DevicePositionMapping

HAS_TRITON = False  # kept for import compatibility; no Triton is used

_MODES = {"delta": _lib.SB_ANGLE_DELTA, "nope": _lib.SB_ANGLE_NOPE, "copy": _lib.SB_ANGLE_NONE}


def _check_head_dim(head_dim, hd: int, fn: str) -> int:
    if head_dim is None:
        return hd
    if int(head_dim) != hd:
        raise ValueError(
            f"{fn}: head_dim={head_dim} does not match the cache's last dimension {hd} "
            "(partial rotary embeddings are not supported)"
        )
    return hd


def _launch(descs: Sequence[_lib.SbInjectDesc], p: _lib.SbInjectParams, device: torch.device, what: str):
    """One kernel launch for all descriptors: up to SB_MAX_INJECT_DESC travel in
    the kernel parameters (sb_inject), more in a device table (sb_inject_many)."""
    lib = _lib.load()
    err = _lib.err_counter(device)
    stream = _lib.stream_ptr(device)
    arr = (_lib.SbInjectDesc * len(descs))(*descs)
    if len(descs) <= _lib.SB_MAX_INJECT_DESC:
        _lib.check(lib.sb_inject(arr, len(descs), p, err.data_ptr(), stream), what)
        return
    nbytes = int(lib.sb_inject_table_bytes(len(descs)))
    if nbytes < 0:
        _lib.check(nbytes, what)
    # the table is read by this launch only; the caching allocator keeps it for this stream until then
    table = torch.empty((nbytes + 15) // 16 * 16, dtype=torch.uint8, device=device)
    _lib.check(lib.sb_inject_many(arr, len(descs), p, table.data_ptr(), table.numel(), err.data_ptr(), stream),
               what)


def _pair_desc(src: _lib.SbRows, dst: _lib.SbRows, sp: torch.Tensor, tp: torch.Tensor,
               src_row: int, dst_row: int) -> _lib.SbInjectDesc:
    if sp.shape != tp.shape or sp.ndim != 1:
        raise ValueError(
            f"donor and target positions must be 1-D of equal length, got {tuple(sp.shape)} and {tuple(tp.shape)}"
        )
    if sp.dtype != tp.dtype:
        raise TypeError("donor and target positions must share one integer dtype")
    d = _lib.SbInjectDesc()
    d.src = src
    d.dst = dst
    d.src_pos = sp.data_ptr()
    d.dst_pos = tp.data_ptr()
    d.n_pairs = sp.shape[0]
    d.pos_dtype = _lib.index_code(sp.dtype)
    d.src_row = src_row
    d.dst_row = dst_row
    d.flags = 0
    return d


def _positions(donor_positions, target_positions, dev: torch.device) -> tuple[torch.Tensor, torch.Tensor]:
    sp = _rows.device_index_tensor(donor_positions, dev, "donor_positions")
    tp = _rows.device_index_tensor(target_positions, dev, "target_positions")
    if sp.dtype != tp.dtype:
        sp, tp = sp.to(torch.int64), tp.to(torch.int64)
    return sp, tp


def _donor_rows(donor_kv: torch.Tensor, has_layer_dim: bool) -> _lib.SbRows:
    if has_layer_dim:  # [L, 2, H, Sd, D]
        return _rows.flat_rows(donor_kv, layer_axis=0, kv_axis=1, head_axis=2, pos_axis=3, dim_axis=4)
    return _rows.flat_rows(donor_kv, layer_axis=None, kv_axis=0, head_axis=1, pos_axis=2, dim_axis=3)


def rope_correct_scatter_paged(
    kv_cache: torch.Tensor,
    donor_kv: torch.Tensor,
    block_table: torch.Tensor,
    donor_positions: torch.Tensor,
    target_positions: torch.Tensor,
    rope_base: float = 10000.0,
    head_dim: int | None = None,
    *,
    rotary_style: str = "interleaved",
    layout: str = "auto",
    staging: str = "direct",
) -> torch.Tensor:
    """Scatter donor KV into a paged cache with RoPE correction on K.

    Mirrors semblend_core/rope_correction.py:193-282: for each
    ``(donor_pos, target_pos)`` pair, K becomes ``RoPE(target - donor) × K``
    and V is copied; ``kv_cache`` ``[num_blocks, 2, H, block_size, D]`` (or
    the ``layout`` given) is modified in place and returned.
    ``donor_kv`` is ``[2, H, donor_len, D]``; ``block_table`` maps the
    request's logical blocks to physical blocks.  ``staging="bulk"`` selects
    the bulk-copy-staged kernel (same results).
    """
    if donor_positions.shape[0] == 0:
        return kv_cache
    _lib.require_cuda(kv_cache, "kv_cache")
    layout = _rows.resolve_layout(kv_cache, layout)
    dev = kv_cache.device
    bt = _rows.device_index_tensor(block_table, dev, "block_table")
    dst, (_, _, nh, _, hd), keep = _rows.paged_rows(kv_cache, bt, layout)
    hd = _check_head_dim(head_dim, hd, "rope_correct_scatter_paged")
    if donor_kv.ndim != 4 or donor_kv.shape[0] != 2 or donor_kv.shape[1] != nh or donor_kv.shape[3] != hd:
        raise ValueError(f"donor_kv must be [2, {nh}, donor_len, {hd}], got {tuple(donor_kv.shape)}")
    if donor_kv.dtype != kv_cache.dtype:
        raise TypeError(f"donor_kv dtype {donor_kv.dtype} differs from kv_cache dtype {kv_cache.dtype}")
    _lib.require_cuda(donor_kv, "donor_kv")
    sp, tp = _positions(donor_positions, target_positions, dev)
    src = _donor_rows(donor_kv, has_layer_dim=False)
    desc = _pair_desc(src, dst, sp, tp, _lib.SB_ROW_AT_SRC_POS, _lib.SB_ROW_AT_DST_POS)
    p = _rows.params(
        n_layers=1, n_heads=nh, head_dim=hd, dtype=kv_cache.dtype, rotary_style=rotary_style,
        k_angle=_lib.SB_ANGLE_DELTA, kv_select=_lib.SB_KV_BOTH,
        inv_freq=_lib.inv_freq(rope_base, hd, dev), staging=staging,
    )
    _launch([desc], p, dev, "rope_correct_scatter_paged")
    del keep
    return kv_cache


def rope_correct_k(
    k_tensor: torch.Tensor,
    donor_positions: torch.Tensor,
    target_positions: torch.Tensor,
    head_dim: int = 128,
    rope_base: float = 10000.0,
    *,
    rotary_style: str = "interleaved",
) -> torch.Tensor:
    """Return a copy of ``k_tensor`` whose rows at ``donor_positions`` are
    rotated by ``RoPE(target - donor)``.

    Mirrors semblend_core/rope_correction.py:336-399: ``k_tensor`` is
    ``[H, S, D]`` or ``[L, H, S, D]``; the rotated row stays at the *donor*
    position, as in the reference.  Each donor position may appear once (the
    reference applies repeated entries one after another).
    """
    _lib.require_cuda(k_tensor, "k_tensor")
    if k_tensor.ndim not in (3, 4):
        raise ValueError(f"k_tensor must be [H, S, D] or [L, H, S, D], got {tuple(k_tensor.shape)}")
    result = k_tensor.clone()
    if donor_positions.shape[0] == 0:
        return result
    hd = _check_head_dim(head_dim, k_tensor.shape[-1], "rope_correct_k")
    dev = k_tensor.device
    has_l = k_tensor.ndim == 4
    rows = _rows.flat_rows(
        result, layer_axis=0 if has_l else None, kv_axis=None,
        head_axis=-3, pos_axis=-2, dim_axis=-1,
    )
    sp, tp = _positions(donor_positions, target_positions, dev)
    desc = _pair_desc(rows, rows, sp, tp, _lib.SB_ROW_AT_SRC_POS, _lib.SB_ROW_AT_SRC_POS)
    p = _rows.params(
        n_layers=k_tensor.shape[0] if has_l else 1, n_heads=k_tensor.shape[-3], head_dim=hd,
        dtype=k_tensor.dtype, rotary_style=rotary_style, k_angle=_lib.SB_ANGLE_DELTA,
        kv_select=_lib.SB_KV_K, inv_freq=_lib.inv_freq(rope_base, hd, dev),
    )
    _launch([desc], p, dev, "rope_correct_k")
    return result


def _host_pairs(permutation) -> np.ndarray:
    """``permutation`` (list of (src, tgt) tuples, [P, 2] array or tensor) as int64 [P, 2]."""
    if isinstance(permutation, torch.Tensor):
        arr = permutation.detach().to("cpu", torch.int64).numpy()
    else:
        arr = np.asarray(permutation, dtype=np.int64)
    if arr.size == 0:
        return arr.reshape(0, 2)
    if arr.ndim != 2 or arr.shape[1] != 2:
        raise ValueError("permutation must be a sequence of (source_pos, target_pos) pairs")
    return arr


def _last_per_target(pairs: np.ndarray) -> np.ndarray:
    """Keep the last pair for each target position (the reference's serial
    writes leave the last one in place); order is preserved."""
    tgt = pairs[:, 1]
    rev = tgt[::-1]
    _, first_rev = np.unique(rev, return_index=True)
    if first_rev.shape[0] == tgt.shape[0]:
        return pairs
    keep = np.sort(tgt.shape[0] - 1 - first_rev)
    return pairs[keep]


def _upload_pairs(pairs: np.ndarray, device: torch.device) -> tuple[torch.Tensor, torch.Tensor]:
    host = torch.from_numpy(np.ascontiguousarray(pairs.T.astype(np.int32)))
    if torch.cuda.is_available():
        host = host.pin_memory()
    dev = host.to(device, non_blocking=True)
    return dev[0], dev[1]


def _permute(kv_cache, block_table, permutation, rope_base, mode, rotary_style, layout, fn):
    on_device = isinstance(permutation, DevicePositionMapping)
    if on_device:
        if permutation.donor_positions.numel() == 0:
            return
    else:
        pairs = _host_pairs(permutation)
        if pairs.shape[0] == 0:
            return
    _lib.require_cuda(kv_cache, "kv_cache")
    layout = _rows.resolve_layout(kv_cache, layout)
    dev = kv_cache.device
    bt = _rows.device_index_tensor(block_table, dev, "block_table")
    rows, (n_layers, _, nh, bs, hd), keep = _rows.paged_rows(kv_cache, bt, layout)
    if on_device:
        # pairs stay on the device: out-of-range ones (and -1 padding) are skipped and counted
        if permutation.device != dev:
            raise ValueError(f"{fn}: the position mapping is on {permutation.device}, the cache on {dev}")
        sp, tp = permutation.donor_positions, permutation.target_positions
        n = sp.shape[0]
    else:
        n_logical = bt.shape[0]
        if pairs.min() < 0 or (pairs // bs).max() >= n_logical:
            bad = pairs[(pairs < 0).any(axis=1) | ((pairs // bs) >= n_logical).any(axis=1)][0]
            raise IndexError(
                f"{fn}: position pair {tuple(int(v) for v in bad)} is outside the block table "
                f"({n_logical} blocks of {bs})"
            )
        pairs = _last_per_target(pairs)
        sp, tp = _upload_pairs(pairs, dev)
        n = pairs.shape[0]
    p = _rows.params(
        n_layers=n_layers, n_heads=nh, head_dim=hd, dtype=kv_cache.dtype, rotary_style=rotary_style,
        k_angle=_MODES[mode], kv_select=_lib.SB_KV_BOTH,
        inv_freq=_lib.inv_freq(rope_base, hd, dev) if mode != "copy" else None,
    )
    lib = _lib.load()
    ws_bytes = lib.sb_permute_workspace_bytes(n, n_layers, nh, hd, p.dtype)
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=dev)
    err = _lib.err_counter(dev)
    _lib.check(
        lib.sb_permute_paged(rows, sp.data_ptr(), tp.data_ptr(), n, _lib.SB_INDEX_I32, p,
                             ws.data_ptr(), ws_bytes, err.data_ptr(), _lib.stream_ptr(dev)),
        fn,
    )
    del keep


def permute_paged_kv_with_rope(
    kv_cache: torch.Tensor,
    block_table: torch.Tensor,
    permutation: list[tuple[int, int]],
    rope_base: float = 10000.0,
    *,
    rotary_style: str = "interleaved",
    layout: str = "auto",
) -> None:
    """Permute KV rows inside a paged cache in place, rotating K by
    ``RoPE(target - source)``.

    Mirrors semblend_core/rope_correction.py:407-476: every source row is
    snapshotted before any write, so sources may overlap targets.  Positions
    outside the block table raise ``IndexError`` as the reference's indexing
    does; when a target appears more than once the last pair wins.
    ``permutation`` may also be a
    :class:`~semblend_b200.position_mapping.DevicePositionMapping`: its pairs
    stay on the device, out-of-range pairs and -1 padding are skipped and
    counted instead of raising, and each target must appear once.
    """
    _permute(kv_cache, block_table, permutation, rope_base, "delta", rotary_style, layout,
             "permute_paged_kv_with_rope")


def nope_permute_paged_kv(
    kv_cache: torch.Tensor,
    block_table: torch.Tensor,
    permutation: list[tuple[int, int]],
    rope_base: float = 10000.0,
    *,
    rotary_style: str = "interleaved",
    layout: str = "auto",
) -> None:
    """NoPE two-step correction: strip ``RoPE(source)`` then apply
    ``RoPE(target)`` to K, copy V.

    Mirrors semblend_core/rope_correction.py:599-696 and its CPU arithmetic
    (:806-823).  V rows are read from the pre-write snapshot, as K rows are;
    the reference copies V one pair at a time from the live cache
    (:643-653), which differs only when a source is also an earlier target.
    """
    _permute(kv_cache, block_table, permutation, rope_base, "nope", rotary_style, layout,
             "nope_permute_paged_kv")


def apply_rope_delta_inplace(
    kv_cache: torch.Tensor,
    block_table: torch.Tensor,
    positions: list[int],
    delta: int,
    rope_base: float = 10000.0,
    *,
    rotary_style: str = "interleaved",
) -> int:
    """Rotate K at ``positions`` by ``RoPE(delta)`` in place; V is untouched.

    Mirrors semblend_core/rope_correction.py:699-783, including its layout
    auto-detection (vLLM ``[2, nb, bs, H, D]`` or canonical
    ``[nb, 2, H, bs, D]``).  Positions beyond the block table are skipped;
    returns the number of positions rotated (repeats count, and are applied
    again, as in the reference's loop).
    """
    if delta == 0 or not len(positions):
        return 0
    _lib.require_cuda(kv_cache, "kv_cache")
    layout = _rows.detect_layout(kv_cache)
    dev = kv_cache.device
    bt = _rows.device_index_tensor(block_table, dev, "block_table")
    rows, (n_layers, _, nh, bs, hd), keep = _rows.paged_rows(kv_cache, bt, layout)
    pos = np.asarray(positions, dtype=np.int64).reshape(-1)
    pos = pos[(pos >= 0) & (pos // bs < bt.shape[0])]
    modified = int(pos.shape[0])
    if modified == 0:
        return 0
    p = _rows.params(
        n_layers=n_layers, n_heads=nh, head_dim=hd, dtype=kv_cache.dtype, rotary_style=rotary_style,
        k_angle=_lib.SB_ANGLE_CONST, kv_select=_lib.SB_KV_K,
        inv_freq=_lib.inv_freq(rope_base, hd, dev), const_delta=int(delta),
    )
    # Repeated positions are rotated once per occurrence, one round at a time.
    uniq, counts = np.unique(pos, return_counts=True)
    for r in range(1, int(counts.max()) + 1):
        round_pos = uniq[counts >= r]
        host = torch.from_numpy(round_pos.astype(np.int32))
        dpos = host.to(dev, non_blocking=False)
        desc = _pair_desc(rows, rows, dpos, dpos, _lib.SB_ROW_AT_SRC_POS, _lib.SB_ROW_AT_SRC_POS)
        _launch([desc], p, dev, "apply_rope_delta_inplace")
    del keep
    return modified


@dataclass
class DonorInjection:
    """One request's inject job for :func:`inject_donors`.

    ``donor_kv`` is ``[L, 2, H, donor_len, D]`` (or ``[2, H, donor_len, D]``
    for a single layer); ``block_table`` the request's logical → physical
    block map; positions are device int32/int64 vectors of equal length.
    """

    donor_kv: torch.Tensor
    block_table: torch.Tensor
    donor_positions: torch.Tensor
    target_positions: torch.Tensor

    @classmethod
    def from_mapping(cls, donor_kv: torch.Tensor, block_table: torch.Tensor,
                     mapping: DevicePositionMapping) -> DonorInjection:
        """The job of one donor's device position mapping (its -1 padding,
        if any, is skipped by the kernel and counted as skipped pairs)."""
        return cls(donor_kv, block_table, mapping.donor_positions, mapping.target_positions)


def inject_donors(
    kv_cache: torch.Tensor | Sequence[torch.Tensor],
    injections: Sequence[DonorInjection],
    rope_base: float = 10000.0,
    *,
    mode: str = "delta",
    rotary_style: str = "interleaved",
    layout: str = "auto",
    staging: str = "direct",
) -> None:
    """Inject several requests' donor KV into a multi-layer paged cache.

    One launch covers every layer, head, request and pair (beyond 64
    requests the descriptors travel in a device table).  ``kv_cache`` is either ``[L, *per_layer]`` with a per-layer
    ``layout`` or a list of ``L`` per-layer tensors (vLLM's ``kv_caches``).
    ``mode`` is ``"delta"`` (``RoPE(target - donor)``, as
    :func:`rope_correct_scatter_paged`), ``"nope"`` (strip, then apply) or
    ``"copy"`` (as ``scatter_donor_kv_paged``).  ``staging="bulk"`` stages the
    source rows in shared memory through 1-D bulk copies instead of direct
    16-byte loads (same results; see ``SB_INJECT_BULK_STAGED``).
    """
    if not injections:
        return
    if mode not in _MODES:
        raise ValueError(f"mode must be one of {tuple(_MODES)}, got {mode!r}")
    first = kv_cache[0] if isinstance(kv_cache, (list, tuple)) else kv_cache
    _lib.require_cuda(first, "kv_cache")
    dev = first.device
    per_layer = first if isinstance(kv_cache, (list, tuple)) else first[0]
    layout = _rows.resolve_layout(per_layer, layout)
    descs, keep = [], []
    geom = template = None
    for inj in injections:
        if inj.donor_positions.shape[0] == 0:
            continue
        bt = _rows.device_index_tensor(inj.block_table, dev, "block_table")
        if template is None:
            # every request shares the cache: its geometry is read once, then each request's
            # descriptor is the template with that request's block table
            template, geom, k = _rows.paged_rows(kv_cache, bt, layout,
                                                 has_layer_dim=not isinstance(kv_cache, (list, tuple)))
            keep += k
            dst = template
        else:
            dst = _lib.SbRows.from_buffer_copy(template)
            dst.block_table = bt.data_ptr()
            dst.n_logical = bt.shape[0]
            dst.block_table_dtype = _lib.index_code(bt.dtype)
        keep.append(bt)
        g = geom
        n_layers, _, nh, _, hd = g
        dk = inj.donor_kv
        has_l = dk.ndim == 5
        want = ((n_layers,) if has_l else ()) + (2, nh)
        if dk.shape[: len(want)] != want or dk.shape[-1] != hd or (not has_l and n_layers != 1):
            raise ValueError(f"donor_kv shape {tuple(dk.shape)} does not match the cache ({n_layers} layers, {nh} heads, D={hd})")
        if dk.dtype != first.dtype:
            raise TypeError(f"donor_kv dtype {dk.dtype} differs from kv_cache dtype {first.dtype}")
        _lib.require_cuda(dk, "donor_kv")
        sp, tp = _positions(inj.donor_positions, inj.target_positions, dev)
        keep += [sp, tp]
        descs.append(_pair_desc(_donor_rows(dk, has_l), dst, sp, tp, _lib.SB_ROW_AT_SRC_POS, _lib.SB_ROW_AT_DST_POS))
    if not descs:
        return
    n_layers, _, nh, _, hd = geom
    p = _rows.params(
        n_layers=n_layers, n_heads=nh, head_dim=hd, dtype=first.dtype, rotary_style=rotary_style,
        k_angle=_MODES[mode], kv_select=_lib.SB_KV_BOTH,
        inv_freq=_lib.inv_freq(rope_base, hd, dev) if mode != "copy" else None, staging=staging,
    )
    _launch(descs, p, dev, "inject_donors")
    del keep


def inject_plan(
    kv_cache: torch.Tensor | Sequence[torch.Tensor],
    donor_kv,
    block_table: torch.Tensor,
    plan,
    rope_base: float = 10000.0,
    *,
    mode: str = "delta",
    rotary_style: str = "interleaved",
    layout: str = "auto",
) -> int:
    """Inject one request's donor rows for every partial layer of a
    :class:`~semblend_b200.partial_attention.PartialAttentionPlan` in one launch.

    The reference's hook converts the plan's per-layer position lists into
    tensors and calls the inject once per layer (model_runner_hook.py:499-555);
    here the plan is flattened once (:func:`~semblend_b200.partial_attention.plan_arrays`),
    layers the plan recomputes in full are left untouched, and the remaining
    layers are addressed through per-layer pointer tables, so no donor data is
    copied.  ``kv_cache`` is ``[L, *per_layer]`` or a list of ``L`` per-layer
    caches; ``donor_kv`` is ``[L, 2, H, S_donor, D]``, or for a multi-donor
    plan a mapping ``donor_id -> [L, 2, H, S_donor, D]``.  Returns the number
    of layers injected.
    """
    import numpy as np

    from .partial_attention import plan_arrays

    if mode not in _MODES:
        raise ValueError(f"mode must be one of {tuple(_MODES)}, got {mode!r}")
    arr = plan_arrays(plan)
    layers = np.nonzero(~arr.recompute_layers)[0].tolist()
    if not layers or arr.donor_positions.shape[0] == 0:
        return 0
    caches = list(kv_cache) if isinstance(kv_cache, (list, tuple)) else [kv_cache[i] for i in layers]
    if isinstance(kv_cache, (list, tuple)):
        caches = [caches[i] for i in layers]
    first = caches[0]
    _lib.require_cuda(first, "kv_cache")
    dev = first.device
    layout = _rows.resolve_layout(first, layout)
    bt = _rows.device_index_tensor(block_table, dev, "block_table")
    dst, g, keep = _rows.paged_rows(caches, bt, layout, has_layer_dim=False)
    keep.append(bt)
    _, _, nh, _, hd = g
    # group the reuse pairs by donor (one descriptor each)
    if isinstance(donor_kv, torch.Tensor):
        groups = {None: (donor_kv, np.arange(arr.donor_positions.shape[0]))}
    else:
        owner = dict(plan.donor_map)
        ids = np.array([owner.get(int(t)) for t in arr.target_positions], dtype=object)
        groups = {d: (donor_kv[d], np.nonzero(ids == d)[0]) for d in dict.fromkeys(ids.tolist())}
    descs = []
    for _, (dk, idx) in groups.items():
        if idx.shape[0] == 0:
            continue
        if dk.ndim != 5 or dk.shape[1:3] != (2, nh) or dk.shape[-1] != hd or dk.shape[0] <= max(layers):
            raise ValueError(f"donor_kv shape {tuple(dk.shape)} does not match the cache ({nh} heads, D={hd}) "
                             f"and layers up to {max(layers)}")
        if dk.dtype != first.dtype:
            raise TypeError(f"donor_kv dtype {dk.dtype} differs from kv_cache dtype {first.dtype}")
        _lib.require_cuda(dk, "donor_kv")
        per_layer = [dk[i] for i in layers]
        src = _donor_rows(per_layer[0], False)
        table = _rows._layer_ptr_table(per_layer, dev)
        src.layer_ptrs = table.data_ptr()
        keep += per_layer + [table]
        pair_idx = torch.from_numpy(idx)
        sp = torch.from_numpy(arr.donor_positions)[pair_idx].to(dev)
        tp = torch.from_numpy(arr.target_positions)[pair_idx].to(dev)
        keep += [sp, tp]
        descs.append(_pair_desc(src, dst, sp, tp, _lib.SB_ROW_AT_SRC_POS, _lib.SB_ROW_AT_DST_POS))
    if not descs:
        return 0
    p = _rows.params(
        n_layers=len(layers), n_heads=nh, head_dim=hd, dtype=first.dtype, rotary_style=rotary_style,
        k_angle=_MODES[mode], kv_select=_lib.SB_KV_BOTH,
        inv_freq=_lib.inv_freq(rope_base, hd, dev) if mode != "copy" else None,
    )
    _launch(descs, p, dev, "inject_plan")
    del keep
    return len(layers)


__all__ = [
    "HAS_TRITON",
    "DonorInjection",
    "apply_rope_delta_inplace",
    "inject_donors",
    "inject_plan",
    "nope_permute_paged_kv",
    "permute_paged_kv_with_rope",
    "rope_correct_k",
    "rope_correct_scatter_paged",
]
