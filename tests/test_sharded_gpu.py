"""Row-sharded search over NCCL on two GPUs (skipped with fewer): the pipelined
batches and the one-batch search equal a single-GPU search of all rows."""

from __future__ import annotations

import datetime
import os
import socket
import traceback

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _data(dev, n=50000, dim=384, nq=300):
    g = torch.Generator(device=dev).manual_seed(4)
    centers = torch.randn(32, dim, generator=g, device=dev)
    E = centers[torch.randint(0, 32, (n,), generator=g, device=dev)] + 0.3 * torch.randn(n, dim, generator=g,
                                                                                      device=dev)
    E = E / E.norm(dim=1, keepdim=True)
    Q = centers[torch.randint(0, 32, (nq,), generator=g, device=dev)] + 0.3 * torch.randn(nq, dim, generator=g,
                                                                                        device=dev)
    return E, Q


def _worker(rank, world, port, path):
    try:
        import torch.distributed as dist

        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=dev)
        from semblend_b200.sharded_search import ShardedDonorMatrix

        E, Q = _data(dev)
        m = ShardedDonorMatrix(E.shape[0], E.shape[1], device=dev)
        m.write_range(0, E)
        ids, sc = m.search(Q, 8, 0.6)
        # batches alternate two query sets (the second reversed): the replayed shard search must take
        # each batch's own queries
        Qr = Q.flip(0).contiguous()
        res = m.search_batches([Q, Qr, Q], 8, 0.6)
        hq, hqr = Q.cpu().pin_memory(), Qr.cpu().pin_memory()
        res_h = m.search_batches([hqr, hq, hqr, hq], 8, 0.6)
        torch.cuda.synchronize(dev)
        out = {"ids": ids.cpu(), "scores": sc.cpu(),
               "batched": [(a.cpu(), b.cpu(), c.cpu()) for a, b, c in res + res_h]}
        if rank == 0:
            torch.save(out, path)
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        if rank == 0:
            torch.save({"error": traceback.format_exc()}, path)
        os._exit(1)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_sharded_search_equals_single_search(tmp_path):
    from semblend_b200.search import DeviceDonorMatrix

    path = str(tmp_path / "res.pt")
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, path)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        if p.is_alive():
            p.kill()
            pytest.fail("rank did not finish")
    res = torch.load(path)
    assert "error" not in res, res.get("error")
    dev = torch.device("cuda", 0)
    E, Q = _data(dev)
    full = DeviceDonorMatrix(E.shape[0], E.shape[1], dev)
    full.write_range(0, E)
    want_i, want_s = full.search(Q, 8, 0.6)
    assert torch.equal(res["ids"], want_i.cpu()) and torch.equal(res["scores"], want_s.cpu())
    wi, ws = want_i.cpu(), want_s.cpu()
    order = [False, True, False, True, False, True, False]  # reversed query sets in res + res_h
    assert len(res["batched"]) == len(order)
    for (ids, sc, st), rev in zip(res["batched"], order):
        assert torch.equal(ids, wi.flip(0) if rev else wi) and torch.equal(sc, ws.flip(0) if rev else ws)
        assert int(st.abs().sum()) == 0
