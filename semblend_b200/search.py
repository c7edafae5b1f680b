"""Device-resident donor embedding matrix and exact cosine top-k search.

:class:`DeviceDonorMatrix` mirrors the reference DonorStore's row storage
(``_embeddings [max_entries, dim]`` fp32 and ``_valid_mask``,
semblend_core/donor_store.py:95-96) in HBM, plus the 16-bit screening copy and
the rounding statistics the tensor-core search needs.  :meth:`search` runs
``sb_cosine_topk`` — the reference's per-query stage (normalise, cosine,
threshold, top-k; donor_store.py:323-341) for a whole batch of queries.

Results are exact: every returned similarity is an fp32 dot product of the
normalised query with the stored fp32 row, and the returned rows are the
``k`` best rows with similarity ``>= min_similarity`` ordered by (similarity
descending, row ascending); ``-1`` / ``-inf`` pad queries with fewer hits.
"""

from __future__ import annotations

import threading

import numpy as np
import torch

from . import _lib

DEFAULT_CAPACITY = 4096  # screening candidates kept per query before rescoring
MAX_K = 32  # the largest k of one sb_cosine_topk call


def _pad64(d: int) -> int:
    return (d + 63) // 64 * 64


class DeviceDonorMatrix:
    """Fixed-capacity fp32 row matrix on one CUDA device with a 16-bit
    screening copy.

    ``shadow_dtype`` is ``torch.float16`` (default: 10 mantissa bits, so the
    proven screening error bound is 4x tighter than bf16 and fewer candidates
    need exact rescoring; fine for embeddings with |value| < 65504, which
    normalised sentence embeddings always are) or ``torch.bfloat16`` (any
    range).  Results are exact either way; a row that overflows fp16 makes
    the bound infinite (every row a candidate) rather than wrong.
    """

    def __init__(self, max_entries: int, dim: int, device: torch.device | str | int | None = None,
                 shadow_dtype: torch.dtype = torch.float16):
        if device is None:
            if not torch.cuda.is_available():
                raise _lib.NativeLibraryError("DeviceDonorMatrix needs a CUDA device (there is no CPU search path)")
            device = torch.device("cuda", torch.cuda.current_device())
        self.device = torch.device(device) if not isinstance(device, int) else torch.device("cuda", device)
        if self.device.type != "cuda":
            raise _lib.NativeLibraryError("DeviceDonorMatrix needs a CUDA device (there is no CPU search path)")
        self.max_entries = int(max_entries)
        self.dim = int(dim)
        self.dim_pad = _pad64(self.dim)
        if self.dim_pad > 512:
            raise ValueError(f"embedding dim {dim} > 512 is not supported by the search kernel")
        if shadow_dtype not in (torch.float16, torch.bfloat16):
            raise ValueError("shadow_dtype must be torch.float16 or torch.bfloat16")
        self.shadow_dtype = shadow_dtype
        self.emb = torch.zeros(self.max_entries, self.dim, dtype=torch.float32, device=self.device)
        self.emb16 = torch.zeros(self.max_entries, self.dim_pad, dtype=shadow_dtype, device=self.device)
        self.valid = torch.zeros(self.max_entries, dtype=torch.uint8, device=self.device)
        # [max ||e - e16||, max ||e16||] over rows ever written (upper bounds)
        self.stats = torch.zeros(2, dtype=torch.float32, device=self.device)
        self._ws: torch.Tensor | None = None
        self._status = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._lock = threading.Lock()

    # -- row updates -----------------------------------------------------------
    def write_rows(self, rows: torch.Tensor | np.ndarray | list[int], values) -> None:
        """Store fp32 ``values [n, dim]`` at row indices ``rows`` and mark them valid."""
        rows_t = torch.as_tensor(np.asarray(rows, dtype=np.int64)).to(self.device, non_blocking=True)
        vals = torch.as_tensor(values, dtype=torch.float32).reshape(-1, self.dim)
        if vals.shape[0] != rows_t.shape[0]:
            raise ValueError("rows and values disagree in length")
        if rows_t.numel() == 0:
            return
        vals = vals.to(self.device, non_blocking=True)
        self.emb.index_copy_(0, rows_t, vals)
        self.valid.index_fill_(0, rows_t, 1)
        self._prepare(rows_t)

    def write_range(self, begin: int, values: torch.Tensor) -> None:
        """Store contiguous rows ``[begin, begin + n)`` from a device or host tensor."""
        n = values.shape[0]
        if n == 0:
            return
        self.emb[begin : begin + n].copy_(values, non_blocking=True)
        self.valid[begin : begin + n] = 1
        lib = _lib.load()
        _lib.check(
            lib.sb_search_prepare_rows(
                self.emb.data_ptr(), self.dim, self.emb16.data_ptr(), self.dim_pad, self.dim, self.dim_pad,
                _lib.dtype_code(self.shadow_dtype), None, begin, n, self.stats.data_ptr(),
                _lib.stream_ptr(self.device),
            ),
            "sb_search_prepare_rows",
        )

    def invalidate(self, rows) -> None:
        rows_t = torch.as_tensor(np.asarray(rows, dtype=np.int64)).to(self.device, non_blocking=True)
        if rows_t.numel():
            self.valid.index_fill_(0, rows_t, 0)

    def _prepare(self, rows_t: torch.Tensor) -> None:
        lib = _lib.load()
        _lib.check(
            lib.sb_search_prepare_rows(
                self.emb.data_ptr(), self.dim, self.emb16.data_ptr(), self.dim_pad, self.dim, self.dim_pad,
                _lib.dtype_code(self.shadow_dtype), rows_t.data_ptr(), 0, rows_t.shape[0], self.stats.data_ptr(),
                _lib.stream_ptr(self.device),
            ),
            "sb_search_prepare_rows",
        )

    # -- search ------------------------------------------------------------------
    def search(self, queries, k: int, min_similarity: float, *, n_rows: int | None = None,
               id_offset: int = 0, capacity: int = DEFAULT_CAPACITY) -> tuple[torch.Tensor, torch.Tensor]:
        """Top-``k`` rows per query (see module docstring); returns device
        tensors ``ids [Q, k]`` (int64, ``+ id_offset``) and ``scores [Q, k]``.

        Any ``k``: beyond the kernel's ``MAX_K`` per call, each query is
        searched in passes of ``MAX_K`` with the rows already returned masked
        out of a scratch copy of the valid mask, so the passes concatenate
        into the exact (similarity desc, row asc) order."""
        q = torch.as_tensor(queries)
        if q.ndim == 1:
            q = q.unsqueeze(0)
        if q.shape[-1] != self.dim:
            raise ValueError(f"query dim {q.shape[-1]} != store dim {self.dim}")
        q = q.to(device=self.device, dtype=torch.float32, non_blocking=True).contiguous()
        n_rows = self.max_entries if n_rows is None else int(n_rows)
        if k > MAX_K:
            res = [self._search_wide(q[i : i + 1], k, min_similarity, n_rows, id_offset, capacity)
                   for i in range(q.shape[0])]
            return torch.cat([r[0] for r in res]), torch.cat([r[1] for r in res])
        return cosine_topk(
            self.emb, self.emb16, self.valid, self.stats, q, k, min_similarity, n_rows=n_rows,
            id_offset=id_offset, capacity=capacity, status=self._status, workspace_owner=self,
        )

    def _search_wide(self, q: torch.Tensor, k: int, min_similarity: float, n_rows: int, id_offset: int,
                     capacity: int) -> tuple[torch.Tensor, torch.Tensor]:
        """One query's top-``k`` for ``k > MAX_K`` (see :meth:`search`)."""
        mask = self.valid.clone()
        ids = torch.full((1, k), -1, dtype=torch.int64, device=self.device)
        scores = torch.full((1, k), float("-inf"), dtype=torch.float32, device=self.device)
        got = 0
        while got < k:
            kk = min(MAX_K, k - got)
            i, s = cosine_topk(self.emb, self.emb16, mask, self.stats, q, kk, min_similarity, n_rows=n_rows,
                               id_offset=id_offset, capacity=capacity, status=self._status, workspace_owner=self)
            ids[:, got : got + kk] = i
            scores[:, got : got + kk] = s
            got += kk
            hit = i[i >= 0]
            if hit.numel() < kk:  # fewer rows than asked reach the threshold: none is left
                break
            mask.index_fill_(0, hit - id_offset, 0)
        return ids, scores


def _workspace(owner, nbytes: int, device: torch.device) -> torch.Tensor:
    ws = getattr(owner, "_ws", None) if owner is not None else None
    if ws is None or ws.numel() < nbytes:
        ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=device)
        if owner is not None:
            owner._ws = ws
    return ws


def cosine_topk_async(emb: torch.Tensor, emb16: torch.Tensor, valid: torch.Tensor | None,
                      stats: torch.Tensor, queries: torch.Tensor, k: int, min_similarity: float, *,
                      n_rows: int | None = None, id_offset: int = 0, capacity: int = DEFAULT_CAPACITY,
                      status: torch.Tensor | None = None, workspace_owner=None,
                      out: tuple[torch.Tensor, torch.Tensor] | None = None,
                      rescore_stream: torch.cuda.Stream | None = None):
    """One search attempt, enqueued without synchronising.

    Returns ``(ids, scores, status)``; ``status`` (device int32) must be read
    before the results are trusted: bit 0 = a query overflowed ``capacity``
    (retry larger), values >= 2 = a kernel wait timed out.

    With ``rescore_stream``, the screening runs on the current stream and the
    exact rescoring on ``rescore_stream`` after it (``sb_cosine_screen`` then
    ``sb_cosine_rescore``): the results are ready on ``rescore_stream``, and the
    workspace of ``workspace_owner`` stays in use until that stream has
    finished the rescore, so the caller orders the next use of it.
    """
    for t, name in ((emb, "emb"), (emb16, "emb16"), (queries, "queries"), (stats, "stats")):
        _lib.require_cuda(t, name)
    dev = emb.device
    nq, dim = queries.shape
    n_rows = emb.shape[0] if n_rows is None else n_rows
    dim_pad = emb16.shape[1]
    k = int(k)
    if not 1 <= k <= 32:
        raise ValueError(f"k must be in [1, 32], got {k}")
    ld_q = queries.stride(0) if nq > 1 else dim  # a size-1 dim may carry any stride
    ld_e = emb.stride(0) if emb.shape[0] > 1 else dim
    ld_b = emb16.stride(0) if emb16.shape[0] > 1 else dim_pad
    if queries.stride(1) != 1 or emb.stride(1) != 1 or emb16.stride(1) != 1:
        raise ValueError("queries and embedding rows must be contiguous along the embedding dimension")
    if out is None:
        ids = torch.empty(nq, k, dtype=torch.int64, device=dev)
        scores = torch.empty(nq, k, dtype=torch.float32, device=dev)
    else:
        ids, scores = out
    if status is None:
        status = torch.zeros(1, dtype=torch.int32, device=dev)
    elif rescore_stream is None:
        status.zero_()  # (sb_cosine_screen zeroes it itself)
    lib = _lib.load()
    cap = max(int(capacity), k)
    nbytes = lib.sb_cosine_topk_workspace_bytes(nq, n_rows, dim, dim_pad, cap)
    ws = _workspace(workspace_owner, nbytes, dev)
    if rescore_stream is None:
        _lib.check(
            lib.sb_cosine_topk(
                emb.data_ptr(), ld_e, emb16.data_ptr(), ld_b, _lib.dtype_code(emb16.dtype),
                valid.data_ptr() if valid is not None else None, n_rows, dim, dim_pad, stats.data_ptr(),
                queries.data_ptr(), ld_q, nq, k, float(min_similarity), int(id_offset),
                ids.data_ptr(), scores.data_ptr(), cap, ws.data_ptr(), ws.numel(), status.data_ptr(),
                _lib.stream_ptr(dev),
            ),
            "sb_cosine_topk",
        )
        return ids, scores, status
    _lib.check(
        lib.sb_cosine_screen(
            emb16.data_ptr(), ld_b, _lib.dtype_code(emb16.dtype), valid.data_ptr() if valid is not None else None,
            n_rows, dim, dim_pad, stats.data_ptr(), queries.data_ptr(), ld_q, nq, k, float(min_similarity), cap,
            ws.data_ptr(), ws.numel(), status.data_ptr(), _lib.stream_ptr(dev),
        ),
        "sb_cosine_screen",
    )
    rescore_stream.wait_stream(torch.cuda.current_stream(dev))
    _lib.check(
        lib.sb_cosine_rescore(
            emb.data_ptr(), ld_e, n_rows, dim, dim_pad, nq, k, float(min_similarity), int(id_offset),
            ids.data_ptr(), scores.data_ptr(), cap, ws.data_ptr(), ws.numel(), status.data_ptr(),
            rescore_stream.cuda_stream,
        ),
        "sb_cosine_rescore",
    )
    for t in (ids, scores, status, ws):  # allocated on the current stream, used on the rescore stream
        t.record_stream(rescore_stream)
    return ids, scores, status


def cosine_topk(emb: torch.Tensor, emb16: torch.Tensor, valid: torch.Tensor | None, stats: torch.Tensor,
                queries: torch.Tensor, k: int, min_similarity: float, *, n_rows: int | None = None,
                id_offset: int = 0, capacity: int = DEFAULT_CAPACITY, status: torch.Tensor | None = None,
                workspace_owner=None) -> tuple[torch.Tensor, torch.Tensor]:
    """Functional form of :meth:`DeviceDonorMatrix.search` over raw tensors.

    Synchronises to read the kernel status; retries with a 4x larger
    candidate capacity if screening overflowed it (many near-ties); raises if
    a kernel wait timed out.
    """
    cap = max(int(capacity), int(k))
    while True:
        ids, scores, st_t = cosine_topk_async(
            emb, emb16, valid, stats, queries, k, min_similarity, n_rows=n_rows, id_offset=id_offset,
            capacity=cap, status=status, workspace_owner=workspace_owner)
        st = int(st_t.item())
        if st & ~1:
            raise _lib.NativeLibraryError(f"sb_cosine_topk: kernel wait timed out (code {st})")
        if st & 1 and cap < 16384:
            cap = min(cap * 4, 16384)
            continue
        if st & 1:
            raise _lib.NativeLibraryError("sb_cosine_topk: more than 16384 screening candidates for a query")
        return ids, scores


def merge_topk(ids: torch.Tensor, scores: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Merge per-shard sorted lists ``[n_lists, Q, k]`` into ``[Q, k]`` by
    (score desc, id asc) with ``sb_topk_merge``.  Each list must be contiguous
    (``[Q, k]`` row-major); the lists themselves may be strided (views into
    all-gathered shard records are read in place)."""
    _lib.require_cuda(ids, "ids")
    n_lists, nq, k = ids.shape
    if scores.dtype != torch.float32:
        scores = scores.to(torch.float32)
    if ids.dtype != torch.int64:
        ids = ids.to(torch.int64)

    def lists(t):
        return t if t.stride(2) == 1 and t.stride(1) == k else t.contiguous()

    ids_c, scores_c = lists(ids), lists(scores)
    out_i = torch.empty(nq, k, dtype=torch.int64, device=ids.device)
    out_s = torch.empty(nq, k, dtype=torch.float32, device=ids.device)
    lib = _lib.load()
    _lib.check(
        lib.sb_topk_merge(ids_c.data_ptr(), ids_c.stride(0) if n_lists > 1 else nq * k, scores_c.data_ptr(),
                          scores_c.stride(0) if n_lists > 1 else nq * k, n_lists, nq, k,
                          out_i.data_ptr(), out_s.data_ptr(), _lib.stream_ptr(ids.device)),
        "sb_topk_merge",
    )
    return out_i, out_s
