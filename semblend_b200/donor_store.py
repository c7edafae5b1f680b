"""GPU donor store — drop-in for ``semblend_core.donor_store``.

Same classes (``DonorNode``, ``DonorMatch``, ``DonorStore``), constructor and
method signatures as the reference (semblend_core/donor_store.py, SemBlend
0.3.2).  The row bookkeeping (LRU eviction, ring-buffer slot reuse, zero rows
for missing embeddings, the valid mask; donor_store.py:130-168) is kept
verbatim in meaning on the host, and every row write is mirrored into a
:class:`~semblend_b200.search.DeviceDonorMatrix` on the GPU.  The cosine /
threshold / top-k stage of ``find_donor`` and ``find_donors`` (:205-229,
:323-341) runs as the exact tensor-core search kernel, for any ``top_k``; the
candidates' reuse estimates (``estimate_reuse_ratio``, :256-262, :359-365)
run on the device for all candidates at once; the Jaccard pre-filter stays
host logic, and the winners' ``compute_alignment`` is the reference's when its
package is installed, else :func:`semblend_b200.alignment.compute_alignment`.  ``alignment=
(estimate_reuse_ratio, compute_alignment)`` overrides both.

:meth:`DonorStore.search_batch` exposes the cosine stage for a batch of
queries (the form the benchmark and batched schedulers use).
"""

from __future__ import annotations

import logging
import time
from collections import OrderedDict
from dataclasses import dataclass

import numpy as np
import torch

from .search import DeviceDonorMatrix

logger = logging.getLogger(__name__)

DEFAULT_CHUNK_SIZE = 256  # semblend_core/alignment.py:35


def _compute_alignment():
    """The reference's compute_alignment when its package is installed (fuzzy
    chunks, exact chunks, then its Levenshtein / token-set fallbacks:
    token-level host work); otherwise this library's: exact chunks on the
    device, then the token-set fallback (alignment.py:790-837 without the
    fuzzy stage)."""
    try:
        from semblend_core.alignment import compute_alignment
    except ImportError:
        from .alignment import compute_alignment
    return compute_alignment


def _reference_indexes(max_entries: int, chunk_size: int, chunk_index):
    """ChunkIndex / TokenIndex of the reference package when installed."""
    try:
        from semblend_core.chunk_index import ChunkIndex
        from semblend_core.token_index import TokenIndex
    except ImportError:
        return chunk_index, None
    ci = chunk_index or ChunkIndex(max_donors=max_entries, chunk_size=chunk_size)
    return ci, TokenIndex(max_donors=max_entries, chunk_size=chunk_size)


@dataclass
class DonorNode:
    """A cached donor entry with embedding and token data."""

    request_id: str
    token_ids: list[int]
    embedding: np.ndarray | None  # [dim] normalized
    timestamp: float
    prompt_text: str = ""
    segment_embeddings: object | None = None


@dataclass(frozen=True)
class DonorMatch:
    """Result of a donor lookup with alignment."""

    donor: DonorNode
    similarity: float
    alignment: object


class DonorStore:
    """Donor store whose embedding matrix lives in HBM and whose cosine stage
    runs on the tensor cores (exact fp32 results)."""

    def __init__(
        self,
        max_entries: int = 10_000,
        embedding_dim: int = 384,
        min_similarity: float = 0.60,
        chunk_size: int = DEFAULT_CHUNK_SIZE,
        chunk_index=None,
        *,
        device: torch.device | str | int | None = None,
        alignment=None,
    ) -> None:
        self._max_entries = max_entries
        self._embedding_dim = embedding_dim
        self._min_similarity = min_similarity
        self._chunk_size = chunk_size
        self._entries: OrderedDict[str, DonorNode] = OrderedDict()
        self._valid_mask = np.zeros(max_entries, dtype=bool)
        self._id_to_idx: dict[str, int] = {}
        self._next_idx = 0
        self._matrix = DeviceDonorMatrix(max_entries, embedding_dim, device)
        self._chunk_index, self._token_index = _reference_indexes(max_entries, chunk_size, chunk_index)
        self._alignment = alignment

    # -- properties of the reference -------------------------------------------
    @property
    def size(self) -> int:
        return len(self._entries)

    @property
    def embedding_dim(self) -> int:
        return self._embedding_dim

    @property
    def token_index(self):
        return self._token_index

    @property
    def chunk_index(self):
        return self._chunk_index

    @property
    def device_matrix(self) -> DeviceDonorMatrix:
        return self._matrix

    @property
    def _embeddings(self) -> np.ndarray:
        """Host copy of the row matrix (for inspection; synchronises)."""
        return self._matrix.emb.cpu().numpy()

    def _compute_alignment_fn(self):
        if self._alignment is not None:
            return self._alignment[1]
        return _compute_alignment()

    def _reuse_ratios(self, donors: list[DonorNode], query_tokens: list[int]) -> list[float]:
        """estimate_reuse_ratio of each candidate donor against the query: one
        batched device call, or the caller's function per donor."""
        if not donors:
            return []
        if self._alignment is not None:
            est = self._alignment[0]
            return [est(d.token_ids, query_tokens, chunk_size=self._chunk_size) for d in donors]
        from .alignment import estimate_reuse_ratio_batch

        return estimate_reuse_ratio_batch([d.token_ids for d in donors], query_tokens, self._chunk_size,
                                          device=self._matrix.device)

    # -- row bookkeeping (donor_store.py:130-168) ---------------------------------
    def add_donor(self, node: DonorNode) -> None:
        self.add_donors([node])

    def add_donors(self, nodes: list[DonorNode]) -> None:
        """Add donors in order with one device update for the whole batch."""
        rows, vals, evicted = [], [], []
        for node in nodes:
            if node.request_id in self._entries:
                self._entries.move_to_end(node.request_id)
                continue
            while len(self._entries) >= self._max_entries:
                evicted_id, _ = self._entries.popitem(last=False)
                evicted_idx = self._id_to_idx.pop(evicted_id, None)
                if evicted_idx is not None:
                    self._valid_mask[evicted_idx] = False
                    evicted.append(evicted_idx)
                if self._chunk_index is not None:
                    self._chunk_index.remove_donor(evicted_id)
                if self._token_index is not None:
                    self._token_index.remove_donor(evicted_id)
            idx = self._next_idx % self._max_entries
            self._next_idx += 1
            emb = node.embedding
            if emb is not None and len(emb) == self._embedding_dim:
                vals.append(np.asarray(emb, dtype=np.float32))
            else:
                vals.append(np.zeros(self._embedding_dim, dtype=np.float32))
            rows.append(idx)
            self._valid_mask[idx] = True
            self._id_to_idx[node.request_id] = idx
            self._entries[node.request_id] = node
            if node.token_ids and self._chunk_index is not None:
                self._chunk_index.add_donor_chunks(node.request_id, node.token_ids)
                self._token_index.add_donor(node.request_id, node.token_ids)
        # a slot may be evicted and rewritten in one batch: invalidate first
        still_invalid = [i for i in dict.fromkeys(evicted) if not self._valid_mask[i]]
        self._matrix.invalidate(still_invalid)
        if rows:
            last = {}
            for r, v in zip(rows, vals):
                last[r] = v  # the last write to a slot wins
            self._matrix.write_rows(list(last.keys()), np.stack(list(last.values())))

    # -- cosine stage ------------------------------------------------------------
    def search_batch(self, queries, k: int, min_similarity: float | None = None):
        """Cosine stage for a batch: ``(rows [Q, k], similarities [Q, k])``
        as device tensors; rows are storage indices (``-1`` padded)."""
        thr = self._min_similarity if min_similarity is None else min_similarity
        return self._matrix.search(queries, k, thr)

    def _cosine_candidates(self, query_embedding, fetch_k: int):
        """The fetch_k most similar valid rows at or above the threshold (all
        of them when fewer pass), as the reference's argpartition keeps
        (donor_store.py:222-226, :335-341); here in (similarity desc, row asc)
        order."""
        if fetch_k <= 0:
            return np.empty(0, np.int64), np.empty(0, np.float32)
        ids, sims = self._matrix.search(np.asarray(query_embedding, dtype=np.float32), int(fetch_k),
                                        self._min_similarity)
        ids = ids[0].cpu().numpy()
        sims = sims[0].cpu().numpy()
        keep = ids >= 0
        return ids[keep], sims[keep]

    def _scored_candidates(self, cand, sims, query_tokens, min_reuse_ratio):
        """(similarity, donor, reuse) of the candidates that pass the Jaccard
        pre-filter and the reuse estimate (donor_store.py:240-262, :351-365)."""
        idx_to_id = {v: k for k, v in self._id_to_idx.items()}
        query_set = set(query_tokens)
        kept = []
        for storage_idx, sim in zip(cand.tolist(), sims.tolist()):
            donor_id = idx_to_id.get(int(storage_idx))
            if donor_id is None:
                continue
            donor = self._entries.get(donor_id)
            if donor is None or donor.token_ids == query_tokens:
                continue
            donor_set = set(donor.token_ids)
            union = len(query_set | donor_set)
            jaccard = len(query_set & donor_set) / union if union > 0 else 0.0
            if jaccard < min_reuse_ratio:
                continue
            kept.append((float(sim), donor))
        reuses = self._reuse_ratios([d for _, d in kept], query_tokens)
        return [(sim, donor, reuse) for (sim, donor), reuse in zip(kept, reuses) if reuse >= min_reuse_ratio]

    def find_donor(self, query_embedding, query_tokens: list[int], top_k: int = 5,
                   min_reuse_ratio: float = 0.5) -> DonorMatch | None:
        """donor_store.py:170-297 with the cosine stage on the GPU."""
        if not self._entries:
            return None
        t0 = time.monotonic()
        if int(self._valid_mask.sum()) == 0:
            return None
        if query_embedding is None or len(query_embedding) != self._embedding_dim:
            return None
        cand, sims = self._cosine_candidates(query_embedding, top_k)
        if cand.shape[0] == 0:
            return None
        best, best_score = None, 0.0
        for sim, donor, reuse in self._scored_candidates(cand, sims, query_tokens, min_reuse_ratio):
            score = sim * reuse
            if score > best_score:
                best_score, best = score, (sim, donor)
        match = None
        if best is not None:
            sim, donor = best
            compute_alignment = self._compute_alignment_fn()
            alignment = compute_alignment(donor.token_ids, query_tokens, chunk_size=self._chunk_size)
            if alignment.reuse_ratio >= min_reuse_ratio:
                match = DonorMatch(donor=donor, similarity=sim, alignment=alignment)
        elapsed = (time.monotonic() - t0) * 1000
        if elapsed > 5:
            logger.debug("DonorStore.find_donor: %.1fms (N=%d)", elapsed, self.size)
        return match

    def find_donors(self, query_embedding, query_tokens: list[int], top_k: int = 5,
                    min_reuse_ratio: float = 0.5) -> list[DonorMatch]:
        """donor_store.py:299-407 with the cosine stage on the GPU."""
        if not self._entries or query_embedding is None:
            return []
        if len(query_embedding) != self._embedding_dim:
            return []
        if int(self._valid_mask.sum()) == 0:
            return []
        cand, sims = self._cosine_candidates(query_embedding, top_k * 2)
        if cand.shape[0] == 0:
            return []
        now = time.monotonic()
        scored = []
        for sim, donor, reuse in self._scored_candidates(cand, sims, query_tokens, min_reuse_ratio):
            age = now - donor.timestamp
            recency_bonus = max(0.0, 0.01 * (1.0 - age / 60.0))
            scored.append((sim * reuse + recency_bonus, sim, donor))
        scored.sort(key=lambda x: x[0], reverse=True)
        compute_alignment = self._compute_alignment_fn()
        matches = []
        for _, sim, donor in scored[:top_k]:
            alignment = compute_alignment(donor.token_ids, query_tokens, chunk_size=self._chunk_size)
            if alignment.reuse_ratio < min_reuse_ratio:
                continue
            matches.append(DonorMatch(donor=donor, similarity=sim, alignment=alignment))
        return matches

    # -- token-only lookups and accessors (host logic of the reference) ---------
    def find_candidates_jaccard(self, query_tokens: list[int], top_k: int = 5, min_jaccard: float = 0.30,
                                min_reuse_ratio: float = 0.5) -> list[DonorMatch]:
        """donor_store.py:409-466 (token sets only; no embedding search)."""
        if not self._entries or not query_tokens:
            return []
        query_set = set(query_tokens)
        scored = []
        for donor in self._entries.values():
            if donor.token_ids == query_tokens:
                continue
            donor_set = set(donor.token_ids)
            union = len(query_set | donor_set)
            jaccard = len(query_set & donor_set) / union if union > 0 else 0.0
            if jaccard >= min_jaccard:
                scored.append((jaccard, donor))
        scored.sort(key=lambda x: x[0], reverse=True)
        compute_alignment = self._compute_alignment_fn()
        matches = []
        for jaccard, donor in scored[: top_k * 2]:
            alignment = compute_alignment(donor.token_ids, query_tokens, chunk_size=self._chunk_size)
            if alignment.reuse_ratio < min_reuse_ratio:
                continue
            matches.append((jaccard * alignment.reuse_ratio,
                            DonorMatch(donor=donor, similarity=jaccard, alignment=alignment)))
        matches.sort(key=lambda x: x[0], reverse=True)
        return [m for _, m in matches[:top_k]]

    def get_donor(self, donor_id: str) -> DonorNode | None:
        return self._entries.get(donor_id)

    def get_donor_tokens(self, donor_id: str) -> list[int] | None:
        node = self._entries.get(donor_id)
        return node.token_ids if node is not None else None

    def get_all_donor_tokens(self) -> dict[str, list[int]]:
        return {did: list(node.token_ids) for did, node in self._entries.items()}

    def find_multi_donor(self, query_tokens: list[int], min_reuse_ratio: float = 0.5, context_gate=None,
                         min_fuzzy_overlap: float = 0.90, pq_store=None, target_text: str = "", embedder=None):
        """donor_store.py:488-538; delegates to the reference's multi-donor
        alignment (token work outside the GPU path)."""
        from semblend_core.multi_donor_alignment import compute_multi_donor_alignment

        result = compute_multi_donor_alignment(
            target_tokens=query_tokens, chunk_index=self._chunk_index,
            donor_token_store=self.get_all_donor_tokens(), chunk_size=self._chunk_size,
            context_gate=context_gate, min_fuzzy_overlap=min_fuzzy_overlap, pq_store=pq_store,
            target_text=target_text, embedder=embedder, token_index=self._token_index,
        )
        if result is not None and result.reuse_ratio < min_reuse_ratio:
            return None
        return result


__all__ = ["DonorMatch", "DonorNode", "DonorStore"]
