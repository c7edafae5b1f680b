"""Drop-in for the SGLang integration's donor store
(semblend/integration/sglang/radix_backend.py:124-211) on the GPU search.

The reference keeps normalised embeddings in an LRU ``OrderedDict`` keyed by
the first 256 token ids and answers ``find_donor`` with a Python loop over
every entry: the best cosine strictly above ``min_similarity``, the earliest
(least recently added) entry on ties, skipping the entry whose key matches
``exclude_tokens``.  Here the embeddings live in a device matrix (one row per
slot) and ``find_donor`` is one top-k search; the strict threshold, the
exclusion and the tie rule are applied to its few candidates on the host.
"""

from __future__ import annotations

import time
from collections import OrderedDict

import numpy as np
import torch

from .search import DeviceDonorMatrix

KEY_TOKENS = 256  # radix_backend.py:165: the first 256 token ids are the dedup key
_FETCH = 8  # candidates per query: the excluded entry plus exact ties of the best
_FETCH_MAX = 32  # the search's largest k: more exact ties than this resolve by slot order


class _DonorEntry:
    """A cached donor prompt (radix_backend.py:124-142)."""

    __slots__ = ("token_ids", "embedding", "timestamp", "num_tokens", "slot", "seq")

    def __init__(self, token_ids, embedding, timestamp, num_tokens, slot=-1, seq=0):
        self.token_ids = token_ids
        self.embedding = embedding
        self.timestamp = timestamp
        self.num_tokens = num_tokens
        self.slot = slot
        self.seq = seq


class RadixDonorStore:
    """``_SemBlendDonorStore`` (radix_backend.py:144-211) with a device matrix."""

    def __init__(self, max_entries: int = 1000, min_similarity: float = 0.60, embedding_dim: int = 384,
                 device=None) -> None:
        self._entries: OrderedDict[tuple[int, ...], _DonorEntry] = OrderedDict()
        self._max_entries = max_entries
        self._min_similarity = min_similarity
        self._matrix = DeviceDonorMatrix(max_entries, embedding_dim, device)
        self._slot_entry: list[_DonorEntry | None] = [None] * max_entries
        self._free = list(range(max_entries - 1, -1, -1))
        self._seq = 0

    @property
    def size(self) -> int:
        return len(self._entries)

    def add_donor(self, token_ids: tuple[int, ...], embedding: np.ndarray) -> None:
        """Register a completed request as a potential donor (radix_backend.py:159-179)."""
        key = token_ids[:KEY_TOKENS]
        if key in self._entries:
            self._entries.move_to_end(key)
            self._seq += 1
            self._entries[key].seq = self._seq  # iteration order of the reference's dict
            return
        emb = embedding / (np.linalg.norm(embedding) + 1e-10)
        if not self._free:  # full: the least recently added entry gives up its slot
            _, old = self._entries.popitem(last=False)
            self._matrix.invalidate([old.slot])
            self._slot_entry[old.slot] = None
            self._free.append(old.slot)
        slot = self._free.pop()
        self._seq += 1
        entry = _DonorEntry(token_ids, emb, time.monotonic(), len(token_ids), slot, self._seq)
        self._entries[key] = entry
        self._slot_entry[slot] = entry
        self._matrix.write_rows([slot], np.asarray(emb, dtype=np.float32).reshape(1, -1))
        while len(self._entries) > self._max_entries:
            _, old = self._entries.popitem(last=False)
            self._matrix.invalidate([old.slot])
            self._slot_entry[old.slot] = None
            self._free.append(old.slot)

    def find_donor(self, query_embedding: np.ndarray, exclude_tokens: tuple[int, ...] | None = None):
        """Best entry with cosine strictly above ``min_similarity``, or None
        (radix_backend.py:181-211)."""
        if not self._entries:
            return None
        q = np.asarray(query_embedding, dtype=np.float32)
        q = q / (np.linalg.norm(q) + 1e-10)
        qt = torch.from_numpy(q).reshape(1, -1)
        exclude = exclude_tokens[:KEY_TOKENS] if exclude_tokens else None
        n = len(self._entries)
        k = min(_FETCH, n)
        while True:
            ids, scores = self._matrix.search(qt, k, self._min_similarity)
            ids, scores = ids[0].cpu().tolist(), scores[0].cpu().tolist()
            best, best_sim = None, self._min_similarity
            for slot, sim in zip(ids, scores):
                if slot < 0:
                    break
                entry = self._slot_entry[slot]
                if entry is None or (exclude is not None and entry.token_ids[:KEY_TOKENS] == exclude):
                    continue
                # strictly above the running best; on an exact tie the earlier-added entry wins
                if sim > best_sim or (best is not None and sim == best_sim and entry.seq < best.seq):
                    best, best_sim = entry, sim
            # the search orders ties by slot, not by age: when the tie reaches the last fetched
            # candidate, fetch more so the earliest-added tied entry is among them
            if best is None or k >= min(n, _FETCH_MAX) or ids[-1] < 0 or scores[-1] != best_sim:
                return best
            k = min(n, _FETCH_MAX, 4 * k)


# the reference's class name, for callers that construct it directly
_SemBlendDonorStore = RadixDonorStore

__all__ = ["RadixDonorStore", "_SemBlendDonorStore"]
