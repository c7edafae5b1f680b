"""Donor search sharded by rows across the ranks of a process group.

Each rank holds a contiguous slice of the donor rows in its own
:class:`~semblend_b200.search.DeviceDonorMatrix` and searches it exactly
(global row ids = local row + the shard's first row); one
``all_gather_into_tensor`` of the per-shard ``[Q, k]`` ids and similarities
(NCCL over NVLink on GPUs) and a k-way merge by (similarity desc, row asc)
give every rank the global top-k.  The merged result equals a single-device
search over all rows.  The reference searches one process's matrix
(semblend_core/donor_store.py:323-341); this is the multi-GPU form of that
stage.
"""

from __future__ import annotations

from collections.abc import Callable

import torch
import torch.distributed as dist

from .search import DEFAULT_CAPACITY, DeviceDonorMatrix, cosine_topk, merge_topk


def shard_bounds(n_rows: int, world: int) -> list[tuple[int, int]]:
    """Contiguous, near-equal row ranges ``[(begin, end)]`` for each rank."""
    return [(r * n_rows // world, (r + 1) * n_rows // world) for r in range(world)]


class ShardedDonorMatrix:
    """Row-sharded donor matrix; ``search`` returns the global top-k on every rank.

    ``local_search(queries, k, thr, id_offset) -> (ids, scores)`` and
    ``merge(ids [W, Q, k], scores [W, Q, k]) -> (ids, scores)`` default to the
    GPU kernels; they are parameters so the exchange and merge logic can run
    on CPU process groups too.
    """

    def __init__(self, n_rows: int, dim: int, group=None, device=None, shadow_dtype=torch.float16,
                 local_search: Callable | None = None, merge: Callable | None = None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.n_rows = int(n_rows)
        self.dim = int(dim)
        self.row_begin, self.row_end = shard_bounds(self.n_rows, self.world)[self.rank]
        self.local = None
        if local_search is None:
            self.local = DeviceDonorMatrix(max(self.row_end - self.row_begin, 1), dim, device, shadow_dtype)
        self._local_search = local_search
        self._merge = merge or merge_topk

    @property
    def n_local(self) -> int:
        return self.row_end - self.row_begin

    def write_range(self, begin: int, values: torch.Tensor) -> None:
        """Write global rows ``[begin, begin + n)``; each rank keeps the part in its shard."""
        a = max(begin, self.row_begin)
        b = min(begin + values.shape[0], self.row_end)
        if a < b and self.local is not None:
            self.local.write_range(a - self.row_begin, values[a - begin : b - begin])

    def search(self, queries: torch.Tensor, k: int, min_similarity: float,
               capacity: int = DEFAULT_CAPACITY) -> tuple[torch.Tensor, torch.Tensor]:
        """Global top-``k`` (ids, similarities) ``[Q, k]``, identical on every rank."""
        if self._local_search is not None:
            ids, scores = self._local_search(queries, k, min_similarity, self.row_begin)
        else:
            m = self.local
            q = queries.to(device=m.device, dtype=torch.float32).contiguous()
            ids, scores = cosine_topk(m.emb, m.emb16, m.valid, m.stats, q, k, min_similarity,
                                      n_rows=self.n_local, id_offset=self.row_begin, capacity=capacity,
                                      status=m._status, workspace_owner=m)
        if self.world == 1:
            return ids, scores
        nq, kk = ids.shape
        # dim-0 concatenation [W * Q, k] (the form every backend accepts), viewed as [W, Q, k]
        all_ids = torch.empty((self.world * nq, kk), dtype=ids.dtype, device=ids.device)
        all_sc = torch.empty((self.world * nq, kk), dtype=scores.dtype, device=scores.device)
        dist.all_gather_into_tensor(all_ids, ids.contiguous(), group=self.group)
        dist.all_gather_into_tensor(all_sc, scores.contiguous(), group=self.group)
        return self._merge(all_ids.view(self.world, nq, kk), all_sc.view(self.world, nq, kk))
