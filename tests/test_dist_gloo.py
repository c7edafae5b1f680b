"""Multi-rank host logic on CPU (gloo, world size 2): row sharding, global ids,
the all-gather of per-shard top-k and the merge reproduce a single search over
all rows; a rank that dies before the collective makes the survivor fail
within the process-group timeout instead of hanging."""

from __future__ import annotations

import datetime
import os
import socket
import traceback

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import search as osearch


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _data(seed=0, n=3001, dim=64, nq=40):
    rng = np.random.default_rng(seed)
    centers = rng.standard_normal((6, dim)).astype(np.float32)
    E = centers[rng.integers(0, 6, n)] + 0.3 * rng.standard_normal((n, dim)).astype(np.float32)
    E /= np.linalg.norm(E, axis=1, keepdims=True)
    Q = centers[rng.integers(0, 6, nq)] + 0.3 * rng.standard_normal((nq, dim)).astype(np.float32)
    return E.astype(np.float32), Q.astype(np.float32)


def _cpu_merge(ids, scores):
    """k-way merge by (score desc, id asc) of [W, Q, k] lists, -1 ids empty."""
    W, Q, k = ids.shape
    ids = ids.permute(1, 0, 2).reshape(Q, W * k)
    sc = scores.permute(1, 0, 2).reshape(Q, W * k).clone()
    sc[ids < 0] = -float("inf")
    out_i = torch.full((Q, k), -1, dtype=torch.int64)
    out_s = torch.full((Q, k), -float("inf"))
    for q in range(Q):
        order = sorted(range(W * k), key=lambda j: (-float(sc[q, j]), int(ids[q, j])))
        picked = [j for j in order if ids[q, j] >= 0][:k]
        out_i[q, : len(picked)] = ids[q, picked]
        out_s[q, : len(picked)] = sc[q, picked]
    return out_i, out_s


def _worker(rank, world, port, mode, result_path):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=8))
        from semblend_b200.sharded_search import ShardedDonorMatrix, shard_bounds

        E, Q = _data()
        a, b = shard_bounds(E.shape[0], world)[rank]

        calls = []

        def local_search(queries, k, thr, offset, capacity):
            calls.append(capacity)
            ids, sc = osearch.topk_batch(E[a:b], np.ones(b - a, bool), queries.numpy(), thr, k)
            ids = np.where(ids >= 0, ids + offset, -1)
            status = 0
            if mode == "overflow" and rank == 1 and capacity < 1000:
                status = 1  # this shard had more screening candidates than the capacity
            if mode == "timeout" and rank == 0:
                status = 2  # a kernel wait gave up on this shard
            return torch.from_numpy(ids), torch.from_numpy(sc), status

        m = ShardedDonorMatrix(E.shape[0], E.shape[1], local_search=local_search, merge=_cpu_merge)
        assert (m.row_begin, m.row_end) == (a, b)
        if mode == "die" and rank == 1:
            os._exit(3)  # leaves without joining the collective
        if mode == "timeout":  # every rank sees the failing shard's status and raises
            from semblend_b200._lib import NativeLibraryError

            try:
                m.search(torch.from_numpy(Q), 5, 0.5, capacity=64)
            except NativeLibraryError:
                if rank == 0:
                    torch.save({"raised": True}, result_path)
                dist.destroy_process_group()
                return
            raise AssertionError("no error for a timed-out shard")
        ids, sc = m.search(torch.from_numpy(Q), 5, 0.5, capacity=64)
        if mode == "overflow":  # both ranks retried together: 64 -> 256 -> 1024
            assert calls == [64, 256, 1024], calls
        batched = m.search_batches([torch.from_numpy(Q)] * 2, 5, 0.5)
        for bi, bs, bst in batched:
            assert torch.equal(bi, ids) and torch.equal(bs, sc) and int(bst.abs().sum()) == 0
        if rank == 0:
            torch.save({"ids": ids, "scores": sc}, result_path)
        dist.destroy_process_group()
    except Exception:
        if rank == 0:
            torch.save({"error": traceback.format_exc()}, result_path)
        os._exit(1)


def _run(mode, tmp_path):
    port = _free_port()
    path = str(tmp_path / f"{mode}.pt")
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, path)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
            pytest.fail("rank did not finish")
    return torch.load(path), [p.exitcode for p in procs]


def test_sharded_search_equals_single_search(tmp_path):
    res, codes = _run("ok", tmp_path)
    assert codes == [0, 0], res.get("error")
    E, Q = _data()
    want_i, want_s = osearch.topk_batch(E, np.ones(E.shape[0], bool), Q, 0.5, 5)
    got_i, got_s = res["ids"].numpy(), res["scores"].numpy()
    np.testing.assert_allclose(got_s, want_s, atol=1e-6)
    diff = got_i != want_i
    assert np.all(np.abs(got_s[diff] - want_s[diff]) <= 1e-6)  # ids differ only on ties


def test_capacity_overflow_on_one_shard_retries_on_every_rank(tmp_path):
    res, codes = _run("overflow", tmp_path)
    assert codes == [0, 0], res.get("error")
    E, Q = _data()
    want_i, want_s = osearch.topk_batch(E, np.ones(E.shape[0], bool), Q, 0.5, 5)
    np.testing.assert_allclose(res["scores"].numpy(), want_s, atol=1e-6)


def test_timed_out_shard_raises_on_every_rank(tmp_path):
    res, codes = _run("timeout", tmp_path)
    assert codes == [0, 0], res.get("error")
    assert res.get("raised") is True


def test_dead_rank_surfaces_as_an_error_not_a_hang(tmp_path):
    res, codes = _run("die", tmp_path)
    assert codes[1] == 3
    assert codes[0] == 1 and "error" in res
