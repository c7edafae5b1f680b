"""CPU oracle: chunk-hash alignment — test infrastructure only.

Restates semblend_core/alignment.py (SemBlend 0.3.2): `_chunk_hash` (:120-130:
SHA-256 of the chunk's token ids packed as little-endian uint32, first 128
bits), the exact chunk matching of `compute_chunk_alignment` (:133-268: each
target chunk, in order, takes the first unused donor chunk with the same hash;
the optional context gate then drops matches with no matched neighbour) and
`estimate_reuse_ratio` (:741-787: the chunk stage, else the token-multiset
overlap).  Python's hashlib is the checker's SHA-256.
"""

from __future__ import annotations

import hashlib
import struct

import numpy as np


def chunk_digest(tokens) -> tuple[int, int, int, int]:
    """The first 128 bits of SHA-256 over the little-endian uint32 token ids,
    as four big-endian 32-bit words (alignment.py:120-130)."""
    data = struct.pack(f"<{len(tokens)}I", *[int(t) for t in tokens])
    d = hashlib.sha256(data).digest()[:16]
    return tuple(int.from_bytes(d[4 * w : 4 * w + 4], "big") for w in range(4))


def digests(tokens, chunk: int) -> np.ndarray:
    """Digests of the full chunks of a sequence, ``[n_full, 4]`` uint32."""
    n = len(tokens) // chunk
    return np.array([chunk_digest(tokens[i * chunk : (i + 1) * chunk]) for i in range(n)], np.uint32).reshape(n, 4)


def chunk_matches(donor_tokens, target_tokens, chunk: int, context_gate: bool) -> np.ndarray:
    """Donor chunk index per target chunk (-1: recompute), alignment.py:174-222."""
    dd, td = digests(donor_tokens, chunk), digests(target_tokens, chunk)
    n_t = (len(target_tokens) + chunk - 1) // chunk
    by_hash: dict[tuple, list[int]] = {}
    for i, d in enumerate(map(tuple, dd)):
        by_hash.setdefault(d, []).append(i)
    used: set[int] = set()
    match = np.full(n_t, -1, np.int64)
    for t, d in enumerate(map(tuple, td)):
        for c in by_hash.get(d, []):
            if c not in used:
                match[t] = c
                used.add(c)
                break
    if context_gate:
        m = match >= 0
        keep = np.zeros_like(m)
        keep[1:] |= m[:-1]
        keep[:-1] |= m[1:]
        match = np.where(m & keep, match, -1)
    return match


def estimate_chunk_reuse(donor_tokens, target_tokens, chunk: int) -> float:
    """Chunk stage of estimate_reuse_ratio (:752-774): matched tokens / target length."""
    m = chunk_matches(donor_tokens, target_tokens, chunk, False)
    return float((m >= 0).sum() * chunk) / max(len(target_tokens), 1)


def token_overlap(donor_tokens, target_tokens) -> int:
    """Multiset overlap: each target token consumes one unused donor occurrence
    of the same id (alignment.py:776-785)."""
    counts: dict[int, int] = {}
    for tok in donor_tokens:
        counts[int(tok)] = counts.get(int(tok), 0) + 1
    n = 0
    for tok in target_tokens:
        c = counts.get(int(tok), 0)
        if c > 0:
            counts[int(tok)] = c - 1
            n += 1
    return n


def estimate_reuse_ratio(donor_tokens, target_tokens, chunk: int) -> float:
    """estimate_reuse_ratio (alignment.py:741-787): the chunk stage, else the
    token-overlap fallback, over the target length."""
    m = chunk_matches(donor_tokens, target_tokens, chunk, False)
    matched = int((m >= 0).sum()) * chunk
    if matched == 0:
        matched = token_overlap(donor_tokens, target_tokens)
    return matched / max(len(target_tokens), 1)
