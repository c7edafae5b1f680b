"""Donor search sharded by rows across the ranks of a process group.

Each rank holds a contiguous slice of the donor rows in its own
:class:`~semblend_b200.search.DeviceDonorMatrix` and searches it exactly
(global row ids = local row + the shard's first row); one
``all_gather_into_tensor`` of a byte record per shard holding its ``[Q, k]``
ids, similarities and kernel status (NCCL over NVLink on GPUs) and a k-way
merge by (similarity desc, row asc) give every rank the global top-k.  The merged result equals a single-device
search over all rows.  The reference searches one process's matrix
(semblend_core/donor_store.py:323-341); this is the multi-GPU form of that
stage.
"""

from __future__ import annotations

from collections.abc import Callable

import torch
import torch.distributed as dist

from . import _lib
from ._lib import NativeLibraryError
from .search import DEFAULT_CAPACITY, MAX_K, DeviceDonorMatrix, _workspace, cosine_topk_async, merge_topk


class _Workspace:
    """Holder of one pipeline slot's search workspace (``_ws``)."""


def _exchange_group(group, cta_policy: int):
    """A new NCCL group over the ranks of ``group`` with the given CTA policy
    (collective: every rank of ``group`` calls it).  Falls back to ``group``
    when this torch build has no communicator options."""
    try:
        from torch.distributed import ProcessGroupNCCL

        opts = ProcessGroupNCCL.Options()
        opts.config.cta_policy = int(cta_policy)
    except (ImportError, AttributeError):
        return group
    ranks = dist.get_process_group_ranks(group) if group is not None else list(range(dist.get_world_size()))
    return dist.new_group(ranks=ranks, backend="nccl", pg_options=opts)


def shard_bounds(n_rows: int, world: int) -> list[tuple[int, int]]:
    """Contiguous, near-equal row ranges ``[(begin, end)]`` for each rank."""
    return [(r * n_rows // world, (r + 1) * n_rows // world) for r in range(world)]


class ShardedDonorMatrix:
    """Row-sharded donor matrix; ``search`` returns the global top-k on every rank.

    ``local_search(queries, k, thr, id_offset, capacity) -> (ids, scores,
    status)`` (status as ``sb_cosine_topk`` sets it: bit 0 = capacity
    overflow, >= 2 = a wait timed out) and ``merge(ids [W, Q, k], scores
    [W, Q, k]) -> (ids, scores)`` default to the GPU kernels; they are
    parameters so the exchange, retry and merge logic can run on CPU process
    groups too.
    """

    def __init__(self, n_rows: int, dim: int, group=None, device=None, shadow_dtype=torch.float16,
                 local_search: Callable | None = None, merge: Callable | None = None,
                 exchange_cta_policy: int | None = 1, overlap_rescore: bool = True):
        self.group = group
        # search_batches: batch i's exact rescoring runs on the exchange stream, beside batch
        # i+1's screening (each slot has its own workspace); False keeps it on the current stream
        self.overlap_rescore = bool(overlap_rescore)
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if (exchange_cta_policy is not None and self.world > 1 and local_search is None
                and dist.get_backend(group) == "nccl"):
            # the exchange gets a communicator of its own whose kernels take as few SMs as NCCL
            # allows (its CTA policy), so they fit beside the next batch's screening kernel
            self.group = _exchange_group(group, exchange_cta_policy)
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

    def _record_bytes(self, nq: int, k: int) -> int:
        # per-rank record: ids int64 [Q, k] | scores fp32 [Q, k] | status int32, padded to 16 bytes
        return (12 * nq * k + 4 + 15) // 16 * 16

    def search_async(self, queries: torch.Tensor, k: int, min_similarity: float,
                     capacity: int = DEFAULT_CAPACITY) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """Global top-``k`` without a host synchronisation: ``(ids, scores, status [W])``.

        Each rank writes its shard's ids, similarities and kernel status into
        one byte record; a single ``all_gather_into_tensor`` exchanges the
        records, so every rank holds every shard's status and makes the same
        retry decision (keeping the ranks' collectives in step).
        """
        nq, kk = queries.shape[0], int(k)
        qk = nq * kk
        rec = self._record_bytes(nq, kk)
        dev = queries.device if self._local_search is not None else self.local.device
        if self.world == 1:
            send = torch.empty(rec, dtype=torch.uint8, device=dev)
        else:
            # exchange buffers are reused across calls: the collective is stream-ordered
            # before the next call's writes, and the merged results are fresh tensors
            key = (nq, kk, str(dev))
            if getattr(self, "_bufs_key", None) != key:
                self._bufs = (torch.empty(rec, dtype=torch.uint8, device=dev),
                              torch.empty(self.world * rec, dtype=torch.uint8, device=dev))
                self._bufs_key = key
            send, recv = self._bufs
        ids_v = send[: 8 * qk].view(torch.int64).view(nq, kk)
        sc_v = send[8 * qk : 12 * qk].view(torch.float32).view(nq, kk)
        st_v = send[12 * qk : 12 * qk + 4].view(torch.int32)
        if self._local_search is not None:
            ids, scores, st = self._local_search(queries, kk, min_similarity, self.row_begin, capacity)
            ids_v.copy_(ids)
            sc_v.copy_(scores)
            st_v.fill_(int(st))
        else:
            m = self.local
            q = queries.to(device=m.device, dtype=torch.float32).contiguous()
            cosine_topk_async(m.emb, m.emb16, m.valid, m.stats, q, kk, min_similarity, n_rows=self.n_local,
                              id_offset=self.row_begin, capacity=capacity, status=st_v, workspace_owner=m,
                              out=(ids_v, sc_v))
        if self.world == 1:
            return ids_v, sc_v, st_v
        dist.all_gather_into_tensor(recv, send, group=self.group)
        table = recv.view(self.world, rec)
        all_ids = table[:, : 8 * qk].view(torch.int64).view(self.world, nq, kk)
        all_sc = table[:, 8 * qk : 12 * qk].view(torch.float32).view(self.world, nq, kk)
        status = table[:, 12 * qk : 12 * qk + 4].view(torch.int32).reshape(self.world)
        ids, scores = self._merge(all_ids, all_sc)
        return ids, scores, status

    def _pipeline(self, nq: int, k: int, min_similarity: float, capacity: int):
        """Buffers of the two in-flight slots of :meth:`search_batches` for one
        batch shape, kept across calls: the query input, the send record
        (ids, similarities, status) and the receive table of each slot."""
        key = (nq, k)
        cache = self.__dict__.setdefault("_pipes", {})
        st = cache.get(key)
        if st is None:
            dev = self.local.device
            rec = self._record_bytes(nq, k)
            st = {"q": [torch.empty(nq, self.dim, dtype=torch.float32, device=dev) for _ in range(2)],
                  "ws": [_Workspace() for _ in range(2)],
                  "send": [torch.empty(rec, dtype=torch.uint8, device=dev) for _ in range(2)],
                  "recv": [torch.empty(self.world * rec, dtype=torch.uint8, device=dev) for _ in range(2)],
                  "rec": rec}
            cache[key] = st
        return st

    def _views(self, send: torch.Tensor, nq: int, k: int):
        qk = nq * k
        return (send[: 8 * qk].view(torch.int64).view(nq, k), send[8 * qk : 12 * qk].view(torch.float32).view(nq, k),
                send[12 * qk : 12 * qk + 4].view(torch.int32))

    def _shard_search(self, q: torch.Tensor, send: torch.Tensor, k: int, min_similarity: float,
                      capacity: int, rescore_stream=None, workspace_owner=None) -> None:
        """The shard's search of ``q`` into a send record (the rescoring on
        ``rescore_stream`` when given, with ``workspace_owner``'s workspace)."""
        m = self.local
        ids_v, sc_v, st_v = self._views(send, q.shape[0], k)
        cosine_topk_async(m.emb, m.emb16, m.valid, m.stats, q, k, min_similarity, n_rows=self.n_local,
                          id_offset=self.row_begin, capacity=capacity, status=st_v,
                          workspace_owner=workspace_owner if workspace_owner is not None else m,
                          out=(ids_v, sc_v), rescore_stream=rescore_stream)

    def search_batches(self, batches, k: int, min_similarity: float, capacity: int = DEFAULT_CAPACITY,
                       on_result=None) -> list[tuple[torch.Tensor, torch.Tensor, torch.Tensor]]:
        """Search a sequence of query batches with two in flight, without a
        host synchronisation: batch i's exact rescoring, all-gather and merge
        run on a second stream while batch i+1 is screened on the current one.  Returns
        ``(ids, scores, status [W])`` per batch, ready on the current stream.
        ``on_result(i, ids, scores)``, if given, is called on the exchange
        stream right after batch i is merged (e.g. to queue its copy to the
        host).  Batches in pinned host memory are copied to the device on a
        third stream, each copy overlapping the previous batch's search.  The
        slots' buffers are kept across calls for each batch shape: keep such
        calls on one stream of the device (two calls of one shape must not run
        concurrently).
        """
        batches = list(batches)
        if self.world == 1 or self._local_search is not None:
            out = []
            for i, q in enumerate(batches):
                r = self.search_async(q, k, min_similarity, capacity=capacity)
                if on_result is not None:
                    on_result(i, r[0], r[1])
                out.append(r)
            return out
        if not batches:
            return []
        m = self.local
        dev = m.device
        cur = torch.cuda.current_stream(dev)
        if getattr(self, "_xstream", None) is None:
            self._xstream = torch.cuda.Stream(dev)
        xs = self._xstream
        kk = int(k)
        nq = batches[0].shape[0]
        if any(b.shape != batches[0].shape for b in batches):
            raise ValueError("search_batches needs batches of one shape")
        st = self._pipeline(nq, kk, min_similarity, capacity)
        rec, qk = st["rec"], nq * kk
        ready = [torch.cuda.Event() for _ in range(2)]
        done = [torch.cuda.Event() for _ in range(2)]
        results = []
        # host batches: copied on a copy stream straight into the slots' query buffers, each copy
        # overlapping the previous batch's search
        host = batches[0].device.type == "cpu"
        if host:
            if getattr(self, "_cstream", None) is None:
                self._cstream = torch.cuda.Stream(dev)
            cs = self._cstream
            cs.wait_stream(cur)  # the slots' buffers may still be read by work queued earlier
            copied = [torch.cuda.Event() for _ in range(2)]
            consumed = [torch.cuda.Event() for _ in range(2)]

            def stage(j):
                with torch.cuda.stream(cs):
                    if j >= 2:
                        cs.wait_event(consumed[j % 2])
                    st["q"][j % 2].copy_(batches[j], non_blocking=True)
                    copied[j % 2].record(cs)

            stage(0)
        fast = self.overlap_rescore and self._merge is merge_topk and kk <= MAX_K
        if fast:
            # The per-batch host work is most of a step's time at 8 GPUs (~0.3 ms of Python
            # against ~0.4 ms of GPU work), so the calls are made straight through the C ABI
            # with their arguments prepared once per slot, and the outputs of all batches
            # are allocated together.
            calls = self._calls(st, nq, kk, float(min_similarity), int(max(capacity, kk)), cur, xs)
            lib = _lib.load()
            screen, rescore, merge = lib.sb_cosine_screen, lib.sb_cosine_rescore, lib.sb_topk_merge
            n = len(batches)
            out_ids = torch.empty(n, nq, kk, dtype=torch.int64, device=dev)
            out_sc = torch.empty(n, nq, kk, dtype=torch.float32, device=dev)
            out_st = torch.empty(n, self.world, dtype=torch.int32, device=dev)
            oi, os_ = out_ids.data_ptr(), out_sc.data_ptr()
        for i, q in enumerate(batches):
            slot = i % 2
            if i >= 2:
                cur.wait_event(done[slot])  # the exchange of batch i - 2 has read this slot
            if host:
                if i + 1 < len(batches):
                    stage(i + 1)
                cur.wait_event(copied[slot])
                q = st["q"][slot]
            else:
                q = q.to(device=dev, dtype=torch.float32).contiguous()
            if fast:
                sa, ra, ma, status_view = calls[slot]
                sa[8], sa[9] = q.data_ptr(), (q.stride(0) if nq > 1 else self.dim)
                rc = screen(*sa)
                if rc:
                    _lib.check(rc, "sb_cosine_screen")
                if host:
                    consumed[slot].record(cur)
                ready[slot].record(cur)
                xs.wait_event(ready[slot])
                rc = rescore(*ra)
                if rc:
                    _lib.check(rc, "sb_cosine_rescore")
                with torch.cuda.stream(xs):
                    dist.all_gather_into_tensor(st["recv"][slot], st["send"][slot], group=self.group)
                    ma[7], ma[8] = oi + 8 * qk * i, os_ + 4 * qk * i
                    rc = merge(*ma)
                    if rc:
                        _lib.check(rc, "sb_topk_merge")
                    out_st[i].copy_(status_view)
                    if on_result is not None:
                        on_result(i, out_ids[i], out_sc[i])
                    done[slot].record(xs)
                continue
            if self.overlap_rescore:
                # screening on the current stream, rescoring on the exchange stream in front of
                # the all-gather, so batch i+1's screening starts as soon as batch i's ends
                self._shard_search(q, st["send"][slot], kk, min_similarity, capacity, rescore_stream=xs,
                                   workspace_owner=st["ws"][slot])
            else:
                self._shard_search(q, st["send"][slot], kk, min_similarity, capacity)
            if host:
                consumed[slot].record(cur)
            ready[slot].record(cur)
            send, recv = st["send"][slot], st["recv"][slot]
            with torch.cuda.stream(xs):
                xs.wait_event(ready[slot])
                dist.all_gather_into_tensor(recv, send, group=self.group)
                table = recv.view(self.world, rec)
                ids, scores = self._merge(table[:, : 8 * qk].view(torch.int64).view(self.world, nq, kk),
                                          table[:, 8 * qk : 12 * qk].view(torch.float32).view(self.world, nq, kk))
                status = table[:, 12 * qk : 12 * qk + 4].view(torch.int32).reshape(self.world).clone()
                if on_result is not None:
                    on_result(i, ids, scores)
                done[slot].record(xs)
            for t in (ids, scores, status):
                t.record_stream(cur)
            results.append((ids, scores, status))
        cur.wait_stream(xs)
        if fast:
            # (allocated on the current stream, written on the exchange stream, which the
            # current stream has just waited for)
            return [(out_ids[i], out_sc[i], out_st[i]) for i in range(len(batches))]
        return results

    def _calls(self, st: dict, nq: int, k: int, thr: float, cap: int, cur, xs) -> list:
        """Per slot: the argument lists of sb_cosine_screen (query pointer and
        pitch filled in per batch), sb_cosine_rescore and sb_topk_merge (output
        pointers filled in per batch), and the status words of the receive
        table; cached per (streams, threshold, capacity)."""
        key = (cur.cuda_stream, xs.cuda_stream, thr, cap)
        if st.get("calls_key") == key:
            return st["calls"]
        m = self.local
        lib = _lib.load()
        dim, dim_pad = self.dim, m.emb16.shape[1]
        ld_e = m.emb.stride(0) if m.emb.shape[0] > 1 else dim
        ld_b = m.emb16.stride(0) if m.emb16.shape[0] > 1 else dim_pad
        nbytes = lib.sb_cosine_topk_workspace_bytes(nq, self.n_local, dim, dim_pad, cap)
        if nbytes < 0:
            raise ValueError("search workspace size out of range")
        qk, rec = nq * k, st["rec"]
        calls = []
        for slot in range(2):
            ws = _workspace(st["ws"][slot], nbytes, m.device)
            send, recv = st["send"][slot], st["recv"][slot]
            sp = send.data_ptr()
            status_ptr = sp + 12 * qk
            sa = [m.emb16.data_ptr(), ld_b, _lib.dtype_code(m.emb16.dtype),
                  m.valid.data_ptr() if m.valid is not None else None, self.n_local, dim, dim_pad,
                  m.stats.data_ptr(), None, None, nq, k, thr, cap, ws.data_ptr(), ws.numel(), status_ptr,
                  cur.cuda_stream]
            ra = [m.emb.data_ptr(), ld_e, self.n_local, dim, dim_pad, nq, k, thr, self.row_begin, sp, sp + 8 * qk,
                  cap, ws.data_ptr(), ws.numel(), status_ptr, xs.cuda_stream]
            rp = recv.data_ptr()
            ma = [rp, rec // 8, rp + 8 * qk, rec // 4, self.world, nq, k, None, None, xs.cuda_stream]
            status_view = recv.view(self.world, rec)[:, 12 * qk : 12 * qk + 4].view(torch.int32).reshape(self.world)
            calls.append((sa, ra, ma, status_view))
        st["calls"], st["calls_key"] = calls, key
        return calls

    def search(self, queries: torch.Tensor, k: int, min_similarity: float,
               capacity: int = DEFAULT_CAPACITY) -> tuple[torch.Tensor, torch.Tensor]:
        """Global top-``k`` (ids, similarities) ``[Q, k]``, identical on every rank.

        Reads every shard's status: retries all ranks together with a 4x
        larger candidate capacity if any shard overflowed it, raises if a
        kernel wait timed out on any shard.
        """
        cap = max(int(capacity), int(k))
        while True:
            ids, scores, status = self.search_async(queries, k, min_similarity, capacity=cap)
            st = 0
            for v in status.reshape(-1).tolist():
                st |= int(v)
            if st & ~1:
                raise NativeLibraryError(f"sharded search: kernel wait timed out (code {st})")
            if st & 1 and cap < 16384:
                cap = min(cap * 4, 16384)
                continue
            if st & 1:
                raise NativeLibraryError("sharded search: more than 16384 screening candidates for a query")
            return ids, scores
