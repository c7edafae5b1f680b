"""CPU oracle: DonorStore cosine / threshold / top-k stage — test
infrastructure only.

Restates semblend_core/donor_store.py (SemBlend 0.3.2): the per-query
cosine stage of ``find_donors`` (:323-341) and ``find_donor`` (:205-229), and
the store's row bookkeeping in ``add_donor`` (:130-168).  numpy fp32, the
library the reference uses.
"""

from __future__ import annotations

from collections import OrderedDict

import numpy as np


def normalize_query(query: np.ndarray) -> np.ndarray:
    """donor_store.py:326: q / (||q|| + 1e-8) in fp32."""
    q = np.asarray(query, dtype=np.float32)
    return q / (np.linalg.norm(q) + 1e-8)


def cosine_candidates(embeddings, valid_mask, query, min_similarity, fetch_k):
    """donor_store.py:323-341: (storage indices, similarities) of the up to
    ``fetch_k`` best valid rows with similarity >= ``min_similarity``, in
    argpartition's (unspecified) order."""
    valid_indices = np.where(valid_mask)[0]
    if valid_indices.shape[0] == 0:
        return np.empty(0, np.int64), np.empty(0, np.float32)
    qn = normalize_query(query)
    sims = embeddings[valid_indices] @ qn
    keep = sims >= min_similarity
    if not keep.any():
        return np.empty(0, np.int64), np.empty(0, np.float32)
    cand = valid_indices[keep]
    sims = sims[keep]
    k = min(len(cand), fetch_k)
    if len(cand) > k:
        part = np.argpartition(sims, -k)[-k:]
        cand, sims = cand[part], sims[part]
    return cand.astype(np.int64), sims.astype(np.float32)


def sort_candidates(ids, scores):
    """Canonical order: score descending, then storage index ascending."""
    order = np.lexsort((ids, -scores))
    return ids[order], scores[order]


def topk_batch(embeddings, valid_mask, queries, min_similarity, k):
    """Per-query :func:`cosine_candidates` + canonical sort for a batch of
    queries; returns ``ids [Q, k]`` (-1 padded) and ``scores [Q, k]``
    (-inf padded)."""
    nq = queries.shape[0]
    ids = np.full((nq, k), -1, np.int64)
    scores = np.full((nq, k), -np.inf, np.float32)
    for i in range(nq):
        c, s = cosine_candidates(embeddings, valid_mask, queries[i], min_similarity, k)
        c, s = sort_candidates(c, s)
        ids[i, : c.shape[0]] = c
        scores[i, : c.shape[0]] = s
    return ids, scores


def topk_batch_gemm(embeddings, valid_mask, queries, min_similarity, k, block=256):
    """Same selection with one fp32 GEMM per block of queries (a stronger CPU
    baseline than the reference's per-query matvec; equal up to summation
    order)."""
    nq = queries.shape[0]
    ids = np.full((nq, k), -1, np.int64)
    scores = np.full((nq, k), -np.inf, np.float32)
    valid_indices = np.where(valid_mask)[0]
    ev = embeddings[valid_indices]
    for b0 in range(0, nq, block):
        qb = np.stack([normalize_query(q) for q in queries[b0 : b0 + block]])
        sims = qb @ ev.T  # [b, N]
        for j in range(qb.shape[0]):
            s = sims[j]
            keep = np.where(s >= min_similarity)[0]
            if keep.shape[0] == 0:
                continue
            if keep.shape[0] > k:
                part = keep[np.argpartition(s[keep], -k)[-k:]]
            else:
                part = keep
            c, sc = sort_candidates(valid_indices[part].astype(np.int64), s[part])
            ids[b0 + j, : c.shape[0]] = c
            scores[b0 + j, : c.shape[0]] = sc
    return ids, scores


class StoreRows:
    """Row bookkeeping of DonorStore.add_donor (donor_store.py:130-168):
    LRU eviction, ring-buffer slot assignment, zero rows for missing
    embeddings and the valid mask."""

    def __init__(self, max_entries: int, dim: int):
        self.max_entries = max_entries
        self.dim = dim
        self.embeddings = np.zeros((max_entries, dim), np.float32)
        self.valid = np.zeros(max_entries, bool)
        self.entries: OrderedDict[str, int] = OrderedDict()
        self.next_idx = 0

    def add(self, request_id: str, embedding) -> None:
        if request_id in self.entries:
            self.entries.move_to_end(request_id)
            return
        while len(self.entries) >= self.max_entries:
            _, idx = self.entries.popitem(last=False)
            self.valid[idx] = False
        idx = self.next_idx % self.max_entries
        self.next_idx += 1
        if embedding is not None and len(embedding) == self.dim:
            self.embeddings[idx] = embedding
        else:
            self.embeddings[idx] = 0.0
        self.valid[idx] = True
        self.entries[request_id] = idx


class RadixStore:
    """The SGLang integration's donor store (semblend/integration/sglang/
    radix_backend.py:144-211): LRU OrderedDict keyed by the first 256 token
    ids, a Python loop for the best cosine strictly above the threshold."""

    def __init__(self, max_entries: int, min_similarity: float):
        from collections import OrderedDict

        self.entries = OrderedDict()
        self.max_entries = max_entries
        self.min_similarity = min_similarity

    def add_donor(self, token_ids, embedding):
        key = token_ids[:256]
        if key in self.entries:
            self.entries.move_to_end(key)
            return
        self.entries[key] = (token_ids, embedding / (np.linalg.norm(embedding) + 1e-10))
        while len(self.entries) > self.max_entries:
            self.entries.popitem(last=False)

    def find_donor(self, query, exclude_tokens=None):
        if not self.entries:
            return None, None
        qn = query / (np.linalg.norm(query) + 1e-10)
        best, best_sim = None, self.min_similarity
        for toks, emb in self.entries.values():
            if exclude_tokens and toks[:256] == exclude_tokens[:256]:
                continue
            sim = float(np.dot(emb, qn))
            if sim > best_sim:
                best, best_sim = toks, sim
        return best, (best_sim if best is not None else None)
