"""Chunk-hash alignment of a target token sequence to a donor on the GPU.

The reference aligns on the host (semblend_core/alignment.py, SemBlend 0.3.2):
SHA-256 of every full chunk of token ids (:120-130), greedy exact matching of
target chunks to donor chunks with an optional context gate (:133-268), and
an expansion into one ``SlotAction`` object per position.  Here the hashes,
the matching and the expansion into position pairs run on the device
(``sb_chunk_digests``, ``sb_chunk_align``), so the pairs feed the inject kernel
without visiting the host.  :func:`compute_chunk_alignment` keeps the
reference's signature and result type for callers that want it (the
``SlotAction`` list is built on the host from the device result).
"""

from __future__ import annotations

import os
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib

DEFAULT_CHUNK_SIZE = 256
# the reference's default (alignment.py:43): the context gate is on unless SEMBLEND_CONTEXT_GATE=0
_CONTEXT_GATE_ENABLED = os.environ.get("SEMBLEND_CONTEXT_GATE", "1") != "0"


def _tokens(t, device) -> torch.Tensor:
    x = torch.as_tensor(t)
    if x.dtype not in (torch.int32, torch.int64):
        x = x.to(torch.int64)
    if device is not None:
        x = x.to(device, non_blocking=True)
    return x.contiguous()


def _device(device, *seqs) -> torch.device:
    """The CUDA device to run on: ``device``, else the first CUDA tensor's,
    else the current one; raises NativeLibraryError without a CUDA device."""
    if device is None:
        first = next((x for x in seqs if isinstance(x, torch.Tensor) and x.is_cuda), None)
        if first is not None:
            return first.device
        if not torch.cuda.is_available():
            raise _lib.NativeLibraryError("no CUDA device: the semblend_b200 kernels run on CUDA devices only "
                                          "(there is no CPU implementation)")
        return torch.device("cuda", torch.cuda.current_device())
    device = torch.device(device)
    if device.type != "cuda":
        raise _lib.NativeLibraryError(f"device {device}: the semblend_b200 kernels run on CUDA devices only")
    return device


def chunk_digests(tokens: torch.Tensor, chunk_size: int = DEFAULT_CHUNK_SIZE) -> torch.Tensor:
    """First 128 bits of SHA-256 of every full chunk (token ids as little-endian
    uint32), ``[n_full_chunks, 4]`` int32 holding the big-endian words."""
    _lib.require_cuda(tokens, "tokens")
    t = _tokens(tokens, None)
    n = t.shape[0] // chunk_size
    out = torch.empty(n, 4, dtype=torch.int32, device=t.device)
    if n:
        lib = _lib.load()
        _lib.check(lib.sb_chunk_digests(t.data_ptr(), _lib.index_code(t.dtype), t.shape[0], chunk_size,
                                        out.data_ptr(), _lib.stream_ptr(t.device)), "sb_chunk_digests")
    return out


@dataclass
class DeviceAlignment:
    """Device result of :func:`chunk_alignment`.

    ``match [n_target_chunks]`` int32: donor chunk per target chunk (-1:
    recompute; a trailing partial chunk is always -1).  ``donor_positions`` /
    ``target_positions`` int32 hold the pairs of the matched chunks in target
    order; the first ``n_pairs`` (a device int64 scalar) entries are valid and
    the rest are -1, so the whole arrays can go to an inject without a host
    synchronisation (the -1 pairs are skipped, and counted as skipped).
    """

    match: torch.Tensor
    donor_positions: torch.Tensor
    target_positions: torch.Tensor
    n_pairs: torch.Tensor
    donor_len: int
    target_len: int
    chunk_size: int

    def pairs(self) -> tuple[torch.Tensor, torch.Tensor]:
        """The valid pairs (reads ``n_pairs``: one host synchronisation)."""
        n = int(self.n_pairs.item())
        return self.donor_positions[:n], self.target_positions[:n]


def chunk_alignment(donor_tokens, target_tokens, chunk_size: int = DEFAULT_CHUNK_SIZE,
                    context_gate: bool | None = None, device=None) -> DeviceAlignment:
    """Exact chunk alignment on the device (compute_chunk_alignment's
    matching, alignment.py:181-252), without a host synchronisation."""
    gate = _CONTEXT_GATE_ENABLED if context_gate is None else bool(context_gate)
    device = _device(device, target_tokens, donor_tokens)
    d = _tokens(donor_tokens, device)
    t = _tokens(target_tokens, device)
    nd_full = d.shape[0] // chunk_size
    if d.dtype == t.dtype:
        # one hashing launch for both sequences (the donor's partial chunk is never hashed)
        both = chunk_digests(torch.cat([d[: nd_full * chunk_size], t]), chunk_size)
        dd, td = both[:nd_full], both[nd_full:]
    else:
        dd, td = chunk_digests(d, chunk_size), chunk_digests(t, chunk_size)
    n_full = td.shape[0]
    n_chunks = (t.shape[0] + chunk_size - 1) // chunk_size
    match = torch.full((n_chunks,), -1, dtype=torch.int32, device=device)
    # the kernel writes -1 past n_pairs: an inject handed the whole arrays skips them (counted as skipped pairs)
    n_pos = n_full * chunk_size
    dpos = torch.empty(max(n_pos, 1), dtype=torch.int32, device=device)
    tpos = torch.empty_like(dpos)
    if n_pos == 0:
        dpos.fill_(-1)
        tpos.fill_(-1)
    n_pairs = torch.empty(1, dtype=torch.int64, device=device)
    lib = _lib.load()
    _lib.check(lib.sb_chunk_align(dd.data_ptr() if dd.shape[0] else None, dd.shape[0], td.data_ptr(), n_full,
                                  chunk_size, int(gate), match.data_ptr(), dpos.data_ptr(), tpos.data_ptr(),
                                  n_pairs.data_ptr(), _lib.stream_ptr(device)), "sb_chunk_align")
    return DeviceAlignment(match, dpos, tpos, n_pairs, int(d.shape[0]), int(t.shape[0]), chunk_size)


def chunk_alignment_batch(donors, targets, chunk_size: int = DEFAULT_CHUNK_SIZE, context_gate: bool | None = None,
                          device=None) -> list[DeviceAlignment]:
    """:func:`chunk_alignment` for several (donor, target) pairs at once — a
    request against each of its donor candidates, or many requests — in one
    hashing launch and two matching launches (``sb_chunk_align_batch``), with
    no host synchronisation.  Returns one :class:`DeviceAlignment` per pair,
    views into shared result buffers."""
    donors, targets = list(donors), list(targets)
    if len(donors) != len(targets):
        raise ValueError(f"{len(donors)} donors for {len(targets)} targets")
    n = len(targets)
    if n == 0:
        return []
    if n > 65535:
        raise ValueError("at most 65535 pairs per batch")
    gate = _CONTEXT_GATE_ENABLED if context_gate is None else bool(context_gate)
    c = int(chunk_size)
    if c <= 0:
        raise ValueError(f"chunk_size must be positive, got {chunk_size}")
    device = _device(device, *targets, *donors)
    ds = [_tokens(x, device) for x in donors]
    ts = [_tokens(x, device) for x in targets]
    dtype = ds[0].dtype if all(x.dtype == ds[0].dtype for x in ds + ts) else torch.int64
    nd = [x.shape[0] // c for x in ds]
    nt = [x.shape[0] // c for x in ts]
    nm = [(x.shape[0] + c - 1) // c for x in ts]
    if max(nt) > 65536:
        raise ValueError("a target has more than 65536 chunks")
    if max(nd) * c > 0x7FFFFFFF:
        raise ValueError("donor positions must fit in int32")
    # every sequence's full chunks, donors first: chunk boundaries stay at multiples of chunk_size
    parts = [x[: k * c].to(dtype) for x, k in zip(ds, nd)] + [x[: k * c].to(dtype) for x, k in zip(ts, nt)]
    dig = chunk_digests(torch.cat(parts), c)
    n_d = sum(nd)
    dd, td = dig[:n_d], dig[n_d:]
    offs = np.zeros((3, n + 1), np.int64)
    offs[0, 1:], offs[1, 1:], offs[2, 1:] = np.cumsum(nd), np.cumsum(nt), np.cumsum(nm)
    if offs[1, -1] * c > 0x7FFFFFFF or offs[2, -1] > 0x7FFFFFFF:
        raise ValueError("batch too large for int32 offsets")
    offs_d = torch.from_numpy(offs.astype(np.int32)).to(device)
    match = torch.empty(max(int(offs[2, -1]), 1), dtype=torch.int32, device=device)
    n_pos = int(offs[1, -1]) * c
    dpos = torch.empty(max(n_pos, 1), dtype=torch.int32, device=device)
    tpos = torch.empty_like(dpos)
    n_pairs = torch.empty(n, dtype=torch.int64, device=device)
    lib = _lib.load()
    _lib.check(lib.sb_chunk_align_batch(dd.data_ptr() if n_d else None, td.data_ptr() if td.shape[0] else None,
                                        offs_d.data_ptr(), n, max(nt), c, int(gate), match.data_ptr(),
                                        dpos.data_ptr(), tpos.data_ptr(), n_pairs.data_ptr(),
                                        _lib.stream_ptr(device)), "sb_chunk_align_batch")
    out = []
    for r in range(n):
        t0, t1 = int(offs[1, r]) * c, int(offs[1, r + 1]) * c
        out.append(DeviceAlignment(match[offs[2, r] : offs[2, r + 1]], dpos[t0:t1], tpos[t0:t1], n_pairs[r : r + 1],
                                   int(ds[r].shape[0]), int(ts[r].shape[0]), c))
    return out


def estimate_chunk_reuse(donor_tokens, target_tokens, chunk_size: int = DEFAULT_CHUNK_SIZE, device=None) -> float:
    """Chunk stage of estimate_reuse_ratio (alignment.py:752-774): matched
    tokens / target length with greedy, ungated chunk matching (no fallback)."""
    a = chunk_alignment(donor_tokens, target_tokens, chunk_size, context_gate=False, device=device)
    return float(a.n_pairs.item()) / max(a.target_len, 1)


def token_overlap(donor_tokens, target_tokens, device=None) -> torch.Tensor:
    """Multiset overlap (sum over ids of min(donor count, target count)) as a
    device int64 scalar ``[1]`` (``sb_token_overlap``; no host synchronisation)."""
    device = _device(device, target_tokens, donor_tokens)
    d, t = _tokens(donor_tokens, device), _tokens(target_tokens, device)
    lib = _lib.load()
    nbytes = lib.sb_token_overlap_workspace_bytes(d.shape[0], t.shape[0])
    if nbytes < 0:
        _lib.check(int(nbytes), "sb_token_overlap_workspace_bytes")
    ws = torch.empty((nbytes + 7) // 8, dtype=torch.int64, device=device)
    out = torch.empty(1, dtype=torch.int64, device=device)
    _lib.check(lib.sb_token_overlap(d.data_ptr() if d.numel() else None, _lib.index_code(d.dtype), d.shape[0],
                                    t.data_ptr() if t.numel() else None, _lib.index_code(t.dtype), t.shape[0],
                                    ws.data_ptr(), ws.numel() * 8, out.data_ptr(), _lib.stream_ptr(device)),
               "sb_token_overlap")
    return out


def estimate_reuse_ratio(donor_tokens, target_tokens, chunk_size: int = DEFAULT_CHUNK_SIZE, device=None) -> float:
    """estimate_reuse_ratio (alignment.py:741-787) on the device: tokens of the
    target chunks that find an unused donor chunk with the same digest, or —
    when no chunk matches — the multiset token overlap, over the target
    length.  Both stages run on the device; reading the ratio is the one host
    synchronisation."""
    a = chunk_alignment(donor_tokens, target_tokens, chunk_size, context_gate=False, device=device)
    dev = a.match.device
    ov = token_overlap(donor_tokens, target_tokens, device=dev)
    matched = torch.where(a.n_pairs > 0, a.n_pairs, ov)
    return float(matched.item()) / max(a.target_len, 1)


def estimate_reuse_ratio_batch(donors, target_tokens, chunk_size: int = DEFAULT_CHUNK_SIZE,
                               device=None) -> list[float]:
    """:func:`estimate_reuse_ratio` of several donors against one target: one
    batched chunk alignment (``sb_chunk_align_batch``), one token-overlap
    launch per donor, and a single host synchronisation for all of them (the
    reference calls its estimate once per candidate, donor_store.py:256-262,
    :359-365)."""
    donors = list(donors)
    if not donors:
        return []
    device = _device(device, target_tokens, *donors)
    t = _tokens(target_tokens, device)
    res = chunk_alignment_batch(donors, [t] * len(donors), chunk_size, context_gate=False, device=device)
    ov = torch.cat([token_overlap(d, t, device=device) for d in donors])
    n_pairs = torch.cat([a.n_pairs for a in res])
    matched = torch.where(n_pairs > 0, n_pairs, ov).cpu().tolist()
    return [m / max(int(t.shape[0]), 1) for m in matched]


@dataclass(frozen=True)
class SlotAction:
    """The reference's SlotAction (alignment.py:100-104): ``action`` is
    ``"copy_from_donor"`` or ``"recompute"``."""

    action: str
    target_pos: int
    donor_pos: int | None = None


@dataclass(frozen=True)
class AlignmentResult:
    """The fields of the reference's AlignmentResult (alignment.py:107-118) that
    exact chunk alignment sets."""

    reuse_ratio: float
    slot_actions: list[SlotAction]
    edit_distance: int
    donor_len: int
    target_len: int
    fuzzy_chunks: int = 0
    exact_chunks: int = 0


def compute_chunk_alignment(donor_tokens, target_tokens, chunk_size: int = DEFAULT_CHUNK_SIZE,
                            context_gate: bool | None = None) -> AlignmentResult:
    """compute_chunk_alignment (alignment.py:133-268) with the hashing and
    matching on the device; the per-position ``slot_actions`` are built on the
    host from the chunk matches, as the reference returns them."""
    a = chunk_alignment(donor_tokens, target_tokens, chunk_size, context_gate)
    match = a.match.cpu().tolist()
    actions: list[SlotAction] = []
    n_reused = 0
    for ti, di in enumerate(match):
        t0 = ti * chunk_size
        n = min(chunk_size, a.target_len - t0)
        if di >= 0:
            actions.extend(SlotAction("copy_from_donor", t0 + i, di * chunk_size + i) for i in range(n))
            n_reused += n
        else:
            actions.extend(SlotAction("recompute", t0 + i) for i in range(n))
    return AlignmentResult(reuse_ratio=n_reused / max(a.target_len, 1), slot_actions=actions,
                           edit_distance=a.target_len - n_reused, donor_len=a.donor_len, target_len=a.target_len,
                           exact_chunks=sum(1 for m in match if m >= 0))


def _token_set_alignment(donor_tokens, target_tokens) -> AlignmentResult:
    """The reference's alignment when no whole chunk matches and rapidfuzz is
    absent (alignment.py:852-853 -> :945-1020): each target token takes the
    earliest unused donor position holding the same id.  Host logic, as in the
    reference: it only runs for a store's winning candidates."""
    free: dict[int, list[int]] = {}
    for pos, tok in enumerate(donor_tokens):
        free.setdefault(int(tok), []).append(pos)
    taken: dict[int, int] = {}
    actions: list[SlotAction] = []
    n_reused = 0
    for t_pos, tok in enumerate(target_tokens):
        tok = int(tok)
        cands = free.get(tok)
        i = taken.get(tok, 0)
        if cands is not None and i < len(cands):
            taken[tok] = i + 1
            actions.append(SlotAction("copy_from_donor", t_pos, cands[i]))
            n_reused += 1
        else:
            actions.append(SlotAction("recompute", t_pos))
    n = len(target_tokens)
    return AlignmentResult(reuse_ratio=n_reused / max(n, 1), slot_actions=actions, edit_distance=n - n_reused,
                           donor_len=len(donor_tokens), target_len=n)


def compute_alignment(donor_tokens, target_tokens, chunk_size: int = DEFAULT_CHUNK_SIZE) -> AlignmentResult:
    """compute_alignment (alignment.py:790-837) without its fuzzy-chunk stage:
    the exact chunk alignment on the device, and when it reuses nothing, the
    token-set alignment the reference falls back to without rapidfuzz.  (The
    reference's fuzzy chunk matching, on by default there, is token-level
    host work outside this library.)"""
    res = compute_chunk_alignment(donor_tokens, target_tokens, chunk_size)
    if res.reuse_ratio > 0:
        return res
    d = donor_tokens.tolist() if isinstance(donor_tokens, torch.Tensor) else list(donor_tokens)
    t = target_tokens.tolist() if isinstance(target_tokens, torch.Tensor) else list(target_tokens)
    return _token_set_alignment(d, t)


__all__ = [
    "AlignmentResult",
    "DEFAULT_CHUNK_SIZE",
    "DeviceAlignment",
    "SlotAction",
    "chunk_alignment",
    "chunk_alignment_batch",
    "chunk_digests",
    "compute_alignment",
    "compute_chunk_alignment",
    "estimate_chunk_reuse",
    "estimate_reuse_ratio",
    "estimate_reuse_ratio_batch",
    "token_overlap",
]
