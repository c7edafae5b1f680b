"""CPU oracle: RoPE-corrected donor-KV inject family — test infrastructure only.

Restates the reference's CPU arithmetic (SemBlend 0.3.2,
semblend_core/rope_correction.py and triton_kernels.py) with torch CPU fp32
ops in the reference's order, vectorised over pairs.  Transcendentals are
evaluated on tensors of the same shape the reference evaluates them on, so the
values match the reference bit for bit on the same host.

Out-of-range pairs are skipped with the reference Triton kernels' conditions
(rope_correction.py:117-129, triton_kernels.py:106-108, :246-260); where a
target row is written twice, the last pair wins (the reference's serial CPU
writes).  ``rotary_style="neox"`` conjugates the reference's interleaved
rotation by the head-dim permutation (i, i + D/2) -> (2i, 2i + 1), which is
exact data movement.
"""

from __future__ import annotations

import torch

_AXES = {"canonical": (0, 1, 2, 3, 4), "vllm": (1, 0, 3, 2, 4), "trtllm": (0, 1, 3, 2, 4)}


def inv_freq(rope_base: float, head_dim: int) -> torch.Tensor:
    """rope_correction.py:235-238."""
    return 1.0 / (rope_base ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))


def canonical_view(cache: torch.Tensor, layout: str) -> torch.Tensor:
    """A [nb, 2, H, bs, D] view of a per-layer paged cache in ``layout``."""
    return cache.permute(*_AXES[layout])


def _perm(d: int) -> torch.Tensor:
    h = d // 2
    p = torch.empty(d, dtype=torch.long)
    p[0::2] = torch.arange(h)
    p[1::2] = torch.arange(h, d)
    return p


def to_interleaved(x: torch.Tensor, style: str) -> torch.Tensor:
    return x if style == "interleaved" else x[..., _perm(x.shape[-1])]


def from_interleaved(x: torch.Tensor, style: str) -> torch.Tensor:
    if style == "interleaved":
        return x
    return x[..., torch.argsort(_perm(x.shape[-1]))]


def _rotate(k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Interleaved-pair rotation of fp32 ``k`` [..., D] (rope_correction.py:317-326)."""
    ke = k[..., 0::2]
    ko = k[..., 1::2]
    out = torch.zeros_like(k)
    out[..., 0::2] = ke * cos - ko * sin
    out[..., 1::2] = ke * sin + ko * cos
    return out


def _rotate_inv(k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Rotation by the negated angle (rope_correction.py:810-813)."""
    ke = k[..., 0::2].clone()
    ko = k[..., 1::2].clone()
    out = torch.zeros_like(k)
    out[..., 0::2] = ke * cos + ko * sin
    out[..., 1::2] = -ke * sin + ko * cos
    return out


def _per_scalar_tables(values: list[float], inv: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin of ``value * inv_freq`` for each value, each evaluated on a
    [D/2] tensor as the reference's per-pair loop does (rope_correction.py:313-315)."""
    cache: dict[float, tuple[torch.Tensor, torch.Tensor]] = {}
    cos_rows, sin_rows = [], []
    for v in values:
        cs = cache.get(v)
        if cs is None:
            theta = v * inv
            cs = (torch.cos(theta), torch.sin(theta))
            cache[v] = cs
        cos_rows.append(cs[0])
        sin_rows.append(cs[1])
    if not values:
        e = torch.empty(0, inv.shape[0])
        return e, e
    return torch.stack(cos_rows), torch.stack(sin_rows)


def _valid_paged(pos: int, bt: list[int], bs: int, nb: int) -> tuple[int, int] | None:
    if pos < 0:
        return None
    lb = pos // bs
    if lb >= len(bt):
        return None
    pb = bt[lb]
    if pb < 0 or pb >= nb:
        return None
    return pb, pos % bs


def _paged_pairs(d_pos, t_pos, bt, bs, nb, src_len):
    """Valid (d, t, phys, off) tuples, last pair per physical row kept."""
    rows: dict[tuple[int, int], tuple[int, int]] = {}
    for dp, tp in zip(d_pos, t_pos):
        if dp < 0 or dp >= src_len:
            continue
        loc = _valid_paged(tp, bt, bs, nb)
        if loc is None:
            continue
        rows.pop(loc, None)
        rows[loc] = (dp, tp)
    out = [(dp, tp, pb, off) for (pb, off), (dp, tp) in rows.items()]
    return out


def rope_correct_scatter_paged(kv_cache, donor_kv, block_table, donor_positions, target_positions,
                               rope_base=10000.0, rotary_style="interleaved", layout="canonical",
                               return_applied=False, inplace=False):
    """rope_correction.py:285-328 (CPU path) with the Triton skip conditions.
    Returns an updated copy of ``kv_cache`` (``kv_cache`` itself, updated, with
    ``inplace`` — the reference's CPU path writes in place); with
    ``return_applied`` also the number of pairs that were applied (in range,
    last write per target row)."""
    out = kv_cache if inplace else kv_cache.clone()
    cv = canonical_view(out, layout)
    nb, _, _, bs, D = cv.shape
    inv = inv_freq(rope_base, D)
    pairs = _paged_pairs(donor_positions.tolist(), target_positions.tolist(),
                         block_table.tolist(), bs, nb, donor_kv.shape[2])
    if not pairs:
        return (out, 0) if return_applied else out
    d = torch.tensor([p[0] for p in pairs])
    pb = torch.tensor([p[2] for p in pairs])
    off = torch.tensor([p[3] for p in pairs])
    cv[pb, 1, :, off, :] = donor_kv[1, :, d, :].permute(1, 0, 2)
    k = to_interleaved(donor_kv[0, :, d, :].permute(1, 0, 2).float(), rotary_style)  # [P, H, D]
    cos, sin = _per_scalar_tables([float(p[1] - p[0]) for p in pairs], inv)
    kr = _rotate(k, cos[:, None, :], sin[:, None, :])
    cv[pb, 0, :, off, :] = from_interleaved(kr, rotary_style).to(out.dtype)
    return (out, len(pairs)) if return_applied else out


def scatter_donor_kv_paged(kv_cache, donor_kv, block_table, donor_positions, target_positions,
                           layout="canonical"):
    """triton_kernels.py:338-355 with the Triton skip conditions (:246-260)."""
    out = kv_cache.clone()
    cv = canonical_view(out, layout)
    nb, _, _, bs, _ = cv.shape
    pairs = _paged_pairs(donor_positions.tolist(), target_positions.tolist(),
                         block_table.tolist(), bs, nb, donor_kv.shape[2])
    for dp, _, pb, off in pairs:
        cv[pb, :, :, off, :] = donor_kv[:, :, dp, :]
    return out


def scatter_donor_kv(target, donor, donor_positions, target_positions):
    """triton_kernels.py:185-189 with the Triton skip conditions (:106-108)."""
    out = target.clone()
    St, Sd = target.shape[3], donor.shape[3]
    rows: dict[int, int] = {}
    for dp, tp in zip(donor_positions.tolist(), target_positions.tolist()):
        if 0 <= dp < Sd and 0 <= tp < St:
            rows.pop(tp, None)
            rows[tp] = dp
    if rows:
        t = torch.tensor(list(rows.keys()))
        d = torch.tensor(list(rows.values()))
        out[:, :, :, t, :] = donor[:, :, :, d, :]
    return out


def rope_correct_k(k_tensor, donor_positions, target_positions, head_dim=128, rope_base=10000.0,
                   rotary_style="interleaved"):
    """rope_correction.py:362-399: rotate rows at donor positions of a copy."""
    dtype = k_tensor.dtype
    inv = inv_freq(rope_base, head_dim)
    deltas = (target_positions - donor_positions).float()
    theta = deltas.unsqueeze(-1) * inv.unsqueeze(0)
    cos_vals = torch.cos(theta)
    sin_vals = torch.sin(theta)
    result = k_tensor.clone()
    for i in range(donor_positions.shape[0]):
        dp = int(donor_positions[i])
        row = result[..., dp, :].float()
        row = to_interleaved(row, rotary_style)
        row = _rotate(row, cos_vals[i], sin_vals[i])
        result[..., dp, :] = from_interleaved(row, rotary_style).to(dtype)
    return result


def _dedupe_last(pairs):
    rows: dict[int, tuple[int, int]] = {}
    for s, t in pairs:
        rows.pop(t, None)
        rows[t] = (s, t)
    return list(rows.values())


def permute_paged_kv_with_rope(kv_cache, block_table, permutation, rope_base=10000.0,
                               rotary_style="interleaved", layout="canonical"):
    """rope_correction.py:427-476 (device-agnostic torch).  Returns a copy."""
    out = kv_cache.clone()
    if not len(permutation):
        return out
    cv = canonical_view(out, layout)
    _, _, _, bs, D = cv.shape
    pairs = _dedupe_last([(int(s), int(t)) for s, t in permutation])
    src = torch.tensor([p[0] for p in pairs], dtype=torch.long)
    tgt = torch.tensor([p[1] for p in pairs], dtype=torch.long)
    bt = block_table.long()
    src_b, src_o = bt[src // bs], src % bs
    tgt_b, tgt_o = bt[tgt // bs], tgt % bs
    src_k = cv[src_b, 0, :, src_o, :].clone()
    src_v = cv[src_b, 1, :, src_o, :].clone()
    cv[tgt_b, 1, :, tgt_o, :] = src_v
    deltas = (tgt - src).float()
    theta = deltas.unsqueeze(-1) * inv_freq(rope_base, D).unsqueeze(0)
    cos_v = torch.cos(theta).unsqueeze(1)
    sin_v = torch.sin(theta).unsqueeze(1)
    k = to_interleaved(src_k.float(), rotary_style)
    kr = _rotate(k, cos_v, sin_v)
    cv[tgt_b, 0, :, tgt_o, :] = from_interleaved(kr, rotary_style).to(out.dtype)
    return out


def nope_permute_paged_kv(kv_cache, block_table, permutation, rope_base=10000.0,
                          rotary_style="interleaved", layout="canonical", v_from_snapshot=False):
    """rope_correction.py:620-696 with the CPU K arithmetic (:797-823).

    The reference copies V one pair at a time from the live cache (:643-653);
    ``v_from_snapshot=True`` reads V from the pre-write snapshot instead, as
    ``permute_paged_kv_with_rope`` does.  The two agree whenever no source is
    an earlier pair's target.  Returns a copy.
    """
    out = kv_cache.clone()
    if not len(permutation):
        return out
    cv = canonical_view(out, layout)
    _, _, _, bs, D = cv.shape
    pairs = [(int(s), int(t)) for s, t in permutation]
    bt = block_table.tolist()
    snap_k = torch.stack([cv[bt[s // bs], 0, :, s % bs, :].clone() for s, _ in pairs])
    snap_v = torch.stack([cv[bt[s // bs], 1, :, s % bs, :].clone() for s, _ in pairs])
    for i, (s, t) in enumerate(pairs):
        v = snap_v[i] if v_from_snapshot else cv[bt[s // bs], 1, :, s % bs, :].clone()
        cv[bt[t // bs], 1, :, t % bs, :] = v
    inv = inv_freq(rope_base, D)
    cs, ss = _per_scalar_tables([float(s) for s, _ in pairs], inv)
    ct, st = _per_scalar_tables([float(t) for _, t in pairs], inv)
    k = to_interleaved(snap_k.float(), rotary_style)
    raw = _rotate_inv(k, cs[:, None, :], ss[:, None, :])
    kr = _rotate(raw, ct[:, None, :], st[:, None, :])
    kr = from_interleaved(kr, rotary_style).to(out.dtype)
    for i, (_, t) in enumerate(pairs):
        cv[bt[t // bs], 0, :, t % bs, :] = kr[i]
    return out


def apply_rope_delta_inplace(kv_cache, block_table, positions, delta, rope_base=10000.0,
                             rotary_style="interleaved"):
    """rope_correction.py:732-783.  Returns (updated copy, count)."""
    out = kv_cache.clone()
    if delta == 0 or not len(positions):
        return out, 0
    vllm = out.shape[0] == 2 and out.ndim == 5 and out.shape[1] != 2
    D = out.shape[4]
    bs = out.shape[2] if vllm else out.shape[3]
    theta = float(delta) * inv_freq(rope_base, D)
    cos_v, sin_v = torch.cos(theta), torch.sin(theta)
    n = 0
    for pos in positions:
        blk_idx = pos // bs
        if pos < 0 or blk_idx >= block_table.shape[0]:
            continue
        blk, off = int(block_table[blk_idx]), pos % bs
        k = (out[0, blk, off, :, :] if vllm else out[blk, 0, :, off, :]).float()
        k = from_interleaved(_rotate(to_interleaved(k, rotary_style), cos_v, sin_v), rotary_style)
        if vllm:
            out[0, blk, off, :, :] = k.to(out.dtype)
        else:
            out[blk, 0, :, off, :] = k.to(out.dtype)
        n += 1
    return out, n
