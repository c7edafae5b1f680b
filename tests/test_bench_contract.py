"""The reference arm of ``bench.py`` (the oracle port of the reference's CPU
inject, timed on the host cores) prints one JSON line with the keys the
benchmark contract names, on the same metric and workload as the GPU arm.
Runs without a GPU."""

from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parents[1]


def test_reference_arm_line():
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1", "--warmup", "1"],
                       capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
                "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["metric"] == "RoPE-corrected KV inject GB/s" and d["unit"] == "GB/s"
    assert d["higher_is_better"] is True and d["value"] > 0 and d["steps"] == 1
    assert d["config"]["workload"].startswith("c2")
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def _bench():
    sys.path.insert(0, str(ROOT))
    import bench

    return bench


def test_c2_partition_covers_every_unit_once():
    """The strong-scaled c2 split gives every (layer, KV head) unit to exactly
    one rank, as rectangles one launch covers (heads first)."""
    b = _bench()
    for world in (1, 2, 3, 4, 5, 6, 7, 8, 16):
        seen = {}
        for rank in range(world):
            h0, h1, l0, l1 = b.c2_partition(world, rank)
            assert 0 <= h0 < h1 <= 4 and 0 <= l0 < l1 <= 28
            for h in range(h0, h1):
                for layer in range(l0, l1):
                    assert (layer, h) not in seen, (world, rank, layer, h)
                    seen[(layer, h)] = rank
        assert len(seen) == 112, world
    assert b.c2_partition(2, 1) == (2, 4, 0, 28)
    assert b.c2_partition(4, 3) == (3, 4, 0, 28)
    h0, h1, l0, l1 = b.c2_partition(8, 5)
    assert (h1 - h0) * (l1 - l0) == 14


def test_cpu_baseline_applies_every_pair():
    """Each CPU sample slice has its own valid block table: every pair is
    applied and counted (a slice with skipped pairs raises)."""
    b = _bench()
    cs = b.CpuInjectSlices()
    for r in range(b.N_REQ):
        sec, nbytes = cs.run()
        n = cs.plans[r][0].shape[0]
        assert sec > 0 and nbytes == b.algorithmic_bytes(n, 1, 4, 128, 2, b.SEQ // b.BLOCK)


def test_c1_inputs_match_the_config():
    """16 permuted 256-token chunks (deltas multiples of 256 within
    [-3840, 3840]), 256 of 1024 blocks, every pair lands inside the table, and
    the oracle applies all 4096 pairs."""
    from oracle import rope as orope

    b = _bench()
    donor, cache, bt, d, t = b.make_c1_inputs(b.SEED + 1)
    assert donor.shape == (2, 4, 4096, 128) and donor.dtype == torch.float32
    assert cache.shape == (1024, 2, 4, 16, 128)
    assert bt.shape == (256,) and len(set(bt.tolist())) == 256 and int(bt.max()) < 1024
    assert sorted(t.tolist()) == list(range(4096)) and sorted(d.tolist()) == list(range(4096))
    delta = (t - d).numpy()
    assert (delta % 256 == 0).all() and abs(delta).max() <= 3840
    _, applied = orope.rope_correct_scatter_paged(cache, donor, bt, d, t, 1e6, "neox", return_applied=True)
    assert applied == 4096
