"""Partial-attention plans — drop-in for ``semblend_core.partial_attention``.

Same types and functions, with the same results, as the reference module
(semblend_core/partial_attention.py, SemBlend 0.3.2): a plan records, per
layer, whether the layer is recomputed in full and, per target position,
whether it reuses a donor row (and which) or is recomputed.  These are host
data structures; the GPU kernels consume them as flat arrays, which
:func:`plan_arrays` and :func:`plan_layer_tensors` build in one vectorised pass
(the reference walks O(layers × positions) Python objects per call,
partial_attention.py:159-198, and converts pair lists per layer,
rope_correction.py:434-435).
"""

from __future__ import annotations

import operator
from collections import Counter
from dataclasses import dataclass, field
from enum import Enum

import numpy as np


class AttentionMode(Enum):
    """Attention computation mode for a position or layer."""

    FULL = "full"
    REUSE = "reuse"
    PARTIAL = "partial"
    SKIP_LAYER = "skip_layer"


@dataclass(frozen=True)
class PositionMask:
    """Mode of one target position (and its donor position when reused)."""

    target_pos: int
    mode: AttentionMode
    donor_pos: int | None = None


@dataclass(frozen=True)
class LayerMask:
    """Strategy of one layer: full recompute, or per-position partial attention."""

    layer_idx: int
    recompute_all: bool
    deviation_score: float
    position_masks: list[PositionMask] = field(default_factory=list)
    verification_source: str = "bathtub"


@dataclass(frozen=True)
class PartialAttentionPlan:
    """Per-layer, per-position attention plan (partial_attention.py:73-102)."""

    target_len: int
    donor_len: int
    donor_id: str
    layer_masks: list[LayerMask]
    num_reuse_positions: int
    num_partial_positions: int
    num_full_layers: int
    computation_ratio: float
    donor_map: tuple[tuple[int, str], ...] = ()


def _hint(layer_hints, layer_idx):
    if layer_hints and layer_idx < len(layer_hints):
        h = layer_hints[layer_idx]
        return (bool(h.get("recomputeAll", h.get("recompute_all", False))),
                h.get("deviationScore", h.get("deviation_score", 0.0)))
    return False, 0.0


def _layers(position_masks, target_len, layer_hints, num_layers):
    layer_masks, full = [], 0
    for layer_idx in range(num_layers):
        recompute_all, deviation = _hint(layer_hints, layer_idx)
        if recompute_all:
            full += 1
            masks = [PositionMask(target_pos=i, mode=AttentionMode.FULL) for i in range(target_len)]
        else:
            masks = list(position_masks)
        layer_masks.append(LayerMask(layer_idx=layer_idx, recompute_all=recompute_all,
                                     deviation_score=deviation, position_masks=masks))
    return layer_masks, full


def _ratio(num_layers, num_full, num_partial, target_len):
    """Fraction of full-prefill work (partial_attention.py:203-219)."""
    if num_layers > 0 and target_len > 0:
        total = num_layers * target_len
        return ((num_layers - num_full) * num_partial + num_full * target_len) / total
    return 1.0


def build_attention_plan(donor_id: str, target_len: int, donor_len: int, copy_positions: list[int],
                         placeholder_positions: list[int], slot_actions: list[dict],
                         layer_hints: list[dict] | None = None, num_layers: int = 32) -> PartialAttentionPlan:
    """Plan from a transfer plan's slot actions (partial_attention.py:105-230):
    ``copy_from_donor`` actions reuse the donor row, ``placeholder`` actions are
    recomputed; layers whose hint sets ``recomputeAll`` are recomputed in full."""
    position_masks = []
    for sa in slot_actions:
        action = sa.get("action", "")
        target_pos = sa.get("targetPos", sa.get("target_pos", 0))
        if action == "copy_from_donor":
            position_masks.append(PositionMask(target_pos=target_pos, mode=AttentionMode.REUSE,
                                               donor_pos=sa.get("donorPos", sa.get("donor_pos"))))
        elif action == "placeholder":
            position_masks.append(PositionMask(target_pos=target_pos, mode=AttentionMode.PARTIAL))
    layer_masks, full = _layers(position_masks, target_len, layer_hints, num_layers)
    num_partial = len(placeholder_positions)
    return PartialAttentionPlan(
        target_len=target_len, donor_len=donor_len, donor_id=donor_id, layer_masks=layer_masks,
        num_reuse_positions=len(copy_positions), num_partial_positions=num_partial, num_full_layers=full,
        computation_ratio=_ratio(num_layers, full, num_partial, target_len),
    )


def build_multi_donor_attention_plan(target_len: int, slot_actions: list[dict],
                                     layer_hints: list[dict] | None = None,
                                     num_layers: int = 32) -> PartialAttentionPlan:
    """Plan from multi-donor slot actions (partial_attention.py:306-435):
    ``copy_from_donor`` (with ``donorId``) reuses, ``recompute`` recomputes."""
    position_masks, donor_map, n_copy, n_partial, donor_len = [], {}, 0, 0, 0
    for sa in slot_actions:
        action = sa.get("action", "")
        target_pos = sa.get("targetPos", sa.get("target_pos", 0))
        donor_id = sa.get("donorId", sa.get("donor_id"))
        dp = sa.get("donorPos", sa.get("donor_pos"))
        if dp is not None and dp >= donor_len:
            donor_len = dp + 1
        if action == "copy_from_donor":
            position_masks.append(PositionMask(target_pos=target_pos, mode=AttentionMode.REUSE, donor_pos=dp))
            n_copy += 1
            if donor_id:
                donor_map[target_pos] = donor_id
        elif action == "recompute":
            position_masks.append(PositionMask(target_pos=target_pos, mode=AttentionMode.PARTIAL))
            n_partial += 1
    layer_masks, full = _layers(position_masks, target_len, layer_hints, num_layers)
    primary = Counter(donor_map.values()).most_common(1)[0][0] if donor_map else ""
    return PartialAttentionPlan(
        target_len=target_len, donor_len=donor_len, donor_id=primary, layer_masks=layer_masks,
        num_reuse_positions=n_copy, num_partial_positions=n_partial, num_full_layers=full,
        computation_ratio=_ratio(num_layers, full, n_partial, target_len), donor_map=tuple(donor_map.items()),
    )


_LAYER_CACHE = "_sb_layer_cache"


def _partial_layer(plan: PartialAttentionPlan, layer_idx: int):
    """(mask, pairs) of a partial layer.  Layers whose position lists hold the
    same PositionMask objects in the same order — every partial layer of a
    plan from build_attention_plan — share one result, computed on the first
    call; a list that was since changed no longer matches and is recomputed."""
    pms = plan.layer_masks[layer_idx].position_masks
    cache = plan.__dict__.get(_LAYER_CACHE)
    if cache is None:
        cache = []
        object.__setattr__(plan, _LAYER_CACHE, cache)  # frozen dataclass: a private side table
    for src, mask, pairs in cache:
        if len(src) == len(pms) and all(map(operator.is_, src, pms)):
            return mask, pairs
    mask = np.zeros(plan.target_len, dtype=bool)
    for pm in pms:
        if pm.mode in (AttentionMode.PARTIAL, AttentionMode.FULL) and pm.target_pos < plan.target_len:
            mask[pm.target_pos] = True
    pairs = [(pm.donor_pos, pm.target_pos) for pm in pms
             if pm.mode == AttentionMode.REUSE and pm.donor_pos is not None]
    cache.append((tuple(pms), mask, pairs))
    return mask, pairs


def compute_attention_mask(plan: PartialAttentionPlan, layer_idx: int) -> np.ndarray:
    """Bool ``[target_len]``: True where the layer recomputes the position
    (partial_attention.py:233-270); all True for unknown or full layers.  The
    reference walks the layer's position list on every call; here partial
    layers sharing one list are walked once per plan."""
    if layer_idx >= len(plan.layer_masks) or plan.layer_masks[layer_idx].recompute_all:
        return np.ones(plan.target_len, dtype=bool)
    return _partial_layer(plan, layer_idx)[0].copy()


def compute_donor_kv_indices(plan: PartialAttentionPlan, layer_idx: int) -> list[tuple[int, int]]:
    """``(donor_pos, target_pos)`` pairs of the layer's reused positions
    (partial_attention.py:273-303); empty for unknown or full layers."""
    if layer_idx >= len(plan.layer_masks) or plan.layer_masks[layer_idx].recompute_all:
        return []
    return list(_partial_layer(plan, layer_idx)[1])


# ---------------------------------------------------------------------------
# Flat arrays for the kernels
# ---------------------------------------------------------------------------
@dataclass(frozen=True)
class PlanArrays:
    """A plan as flat arrays.

    ``recompute_layers [L]`` bool; for every other layer the same
    ``compute_mask [target_len]`` and reuse pairs ``donor_positions`` /
    ``target_positions`` (int32) apply — the reference builds identical
    per-position lists for all of them.
    """

    recompute_layers: np.ndarray
    compute_mask: np.ndarray
    donor_positions: np.ndarray
    target_positions: np.ndarray


def plan_arrays(plan: PartialAttentionPlan) -> PlanArrays:
    """One pass over the plan's first partial layer (all partial layers share
    their position list)."""
    L = len(plan.layer_masks)
    rec = np.fromiter((lm.recompute_all for lm in plan.layer_masks), dtype=bool, count=L)
    partial = next((lm for lm in plan.layer_masks if not lm.recompute_all), None)
    mask = np.zeros(plan.target_len, dtype=bool)
    if partial is None:
        return PlanArrays(rec, np.ones(plan.target_len, bool), np.empty(0, np.int32), np.empty(0, np.int32))
    pms = partial.position_masks
    modes = [pm.mode for pm in pms]
    tgt = np.fromiter((pm.target_pos for pm in pms), dtype=np.int64, count=len(pms))
    is_comp = np.fromiter((m in (AttentionMode.PARTIAL, AttentionMode.FULL) for m in modes), bool, len(pms))
    is_reuse = np.fromiter((m == AttentionMode.REUSE and pm.donor_pos is not None for m, pm in zip(modes, pms)),
                           bool, len(pms))
    sel = tgt[is_comp]
    mask[sel[sel < plan.target_len]] = True
    dpos = np.fromiter((pm.donor_pos for pm, r in zip(pms, is_reuse) if r), dtype=np.int64, count=int(is_reuse.sum()))
    return PlanArrays(rec, mask, dpos.astype(np.int32), tgt[is_reuse].astype(np.int32))


def plan_layer_tensors(plan: PartialAttentionPlan, device):
    """:func:`plan_arrays` uploaded once: ``(recompute_layers, compute_mask,
    donor_positions, target_positions)`` as torch tensors on ``device``."""
    import torch

    a = plan_arrays(plan)
    return (torch.from_numpy(a.recompute_layers).to(device), torch.from_numpy(a.compute_mask).to(device),
            torch.from_numpy(a.donor_positions).to(device), torch.from_numpy(a.target_positions).to(device))


__all__ = [
    "AttentionMode",
    "LayerMask",
    "PartialAttentionPlan",
    "PlanArrays",
    "PositionMask",
    "build_attention_plan",
    "build_multi_donor_attention_plan",
    "compute_attention_mask",
    "compute_donor_kv_indices",
    "plan_arrays",
    "plan_layer_tensors",
]
