"""Benchmark of the B200 donor-reuse hot path (one JSON line on rank 0).

Workload (``configs[1]`` of the baseline): RoPE-corrected donor-KV inject for
8 requests × 16384-token donors, 28 layers × 4 KV heads × 128 dims, bf16, 85 %
of tokens reused through 256-token chunks shifted by per-chunk deltas
U[-4096, 4096] (clamped so donor rows exist), 15 % recompute positions left
untouched, paged cache with block size 16 and a seeded random block table.
One step = one launch injecting every layer, head and request.

Metric: GB/s of algorithmic bytes (K and V rows read and written, positions and
block tables read once).  Multi-GPU: one process per GPU and the SAME step split
across them (strong scaling, no collective on the inject path): with N | 4 each
rank owns 4/N of the KV heads for all 28 layers, with N = 8 each rank owns one
KV head for 14 of the layers (the 112 (layer, head) units, 14 per rank);
value = the whole step's bytes ÷ the slowest rank's time.

Output: rank 0 prints ONE JSON line on stdout (the c2 headline, whose last key
``components_summary`` condenses every component); each component's full line
goes to stderr first, one JSON object per line.  A failed parity check of any
component makes the exit status non-zero after the line is printed.

``--impl reference`` times the CPU restatement of the reference's inject
(``oracle/``) on the host cores: each step one (request, layer) slice of c2.

Usage: python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

# c2 geometry
N_REQ, SEQ, N_LAYERS, N_KV_HEADS, HEAD_DIM, BLOCK = 8, 16384, 28, 4, 128, 16
CHUNK, MAX_DELTA, RECOMPUTE_FRAC, ROPE_THETA = 256, 4096, 0.15, 1e6
SEED = 20261201


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


# ---------------------------------------------------------------------------
# Workload generation (seeded, host side: pair lists and block tables)
# ---------------------------------------------------------------------------
def make_request_plan(rng: np.random.Generator, seq: int = SEQ):
    """Donor/target positions of one request: 256-token chunks shifted by a
    per-chunk delta, 15 % of target positions marked for recompute."""
    n_chunks = seq // CHUNK
    tgt_all, don_all = [], []
    for c in range(n_chunks):
        t0 = c * CHUNK
        delta = int(rng.integers(-MAX_DELTA, MAX_DELTA + 1))
        delta = min(max(delta, t0 - (seq - CHUNK)), t0)  # donor chunk inside [0, seq)
        t = np.arange(t0, t0 + CHUNK)
        tgt_all.append(t)
        don_all.append(t - delta)
    tgt = np.concatenate(tgt_all)
    don = np.concatenate(don_all)
    recompute = rng.permutation(seq)[: int(round(RECOMPUTE_FRAC * seq))]
    keep = np.ones(seq, bool)
    keep[recompute] = False
    return don[keep].astype(np.int32), tgt[keep].astype(np.int32), np.sort(recompute)


def make_block_tables(rng: np.random.Generator, n_req: int, seq: int, pool: int):
    per = seq // BLOCK
    perm = rng.permutation(pool)[: n_req * per]
    return [perm[r * per : (r + 1) * per].astype(np.int32) for r in range(n_req)]


def algorithmic_bytes(n_pairs: int, n_layers: int, n_heads: int, head_dim: int, elt: int, n_blocks: int) -> int:
    """K and V rows read once and written once, positions (2 × int32) and
    block-table entries (int32) read once."""
    return n_pairs * n_layers * n_heads * head_dim * elt * 4 + 8 * n_pairs + 4 * n_blocks


def c2_partition(world: int, rank: int, n_layers: int = N_LAYERS, n_heads: int = N_KV_HEADS):
    """The rank's share of the c2 step as (head_lo, head_hi, layer_lo, layer_hi).

    The (layer, KV head) units are split into gcd(world, heads) head groups
    times world / gcd layer groups, so every share is a rectangle one launch
    covers: N = 2 / 4 split the heads (all layers), N = 8 gives one head x 14
    layers.  Layer groups differ by at most one layer when they do not divide."""
    import math

    hg = math.gcd(world, n_heads)
    lg = world // hg
    hi_, li = rank % hg, rank // hg
    h0, h1 = hi_ * n_heads // hg, (hi_ + 1) * n_heads // hg
    l0, l1 = li * n_layers // lg, (li + 1) * n_layers // lg
    return h0, h1, l0, l1


def ulp_report(got: torch.Tensor, want: torch.Tensor, style: str) -> tuple[int, float]:
    """(largest per-element ulp distance, largest error in ulps of the element's
    RoPE-pair magnitude) between two bf16 / fp16 tensors of K rows."""
    mant = {torch.bfloat16: 7, torch.float16: 10}[got.dtype]

    def ordered(x):
        i = x.contiguous().view(torch.int16).to(torch.int64)
        return torch.where(i < 0, -(i & 0x7FFF), i)

    elem = int((ordered(got) - ordered(want)).abs().max()) if got.numel() else 0
    g, w = got.float(), want.float()
    d = w.shape[-1]
    if style == "neox":
        a, b = w[..., : d // 2], w[..., d // 2:]
        n = torch.sqrt(a * a + b * b)
        n = torch.cat([n, n], dim=-1)
    else:
        n = torch.sqrt(w[..., 0::2] ** 2 + w[..., 1::2] ** 2)
        n = torch.stack([n, n], dim=-1).reshape(w.shape)
    ulp = torch.exp2(torch.floor(torch.log2(n.clamp_min(1e-30))) - mant)
    pair = float(((g - w).abs() / ulp).max()) if got.numel() else 0.0
    return elem, pair


def inject_cu_digest() -> str:
    """Digest of the inject kernel's sources, to tell whether a committed DRAM
    traffic profile was captured on this build."""
    import hashlib

    h = hashlib.sha256()
    for name in ("inject.cu", "common.cuh"):
        h.update((ROOT / "semblend_b200" / "csrc" / name).read_bytes())
    return h.hexdigest()[:16]


def committed_traffic(name: str) -> tuple[int | None, str]:
    """DRAM bytes per launch from ``profiles/<name>.json`` when it was captured
    on the current inject sources, else (None, why)."""
    tf = ROOT / "profiles" / f"{name}.json"
    if not tf.exists():
        return None, "no profile"
    prof = json.loads(tf.read_text())
    if prof.get("inject_src_sha16") != inject_cu_digest():
        return None, f"profiles/{name}.json was captured on other inject sources"
    return prof.get("bytes_per_launch"), f"profiles/{name}.json (ncu, same inject sources)"


# ---------------------------------------------------------------------------
# Clock sampling during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self._t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", str(self.gpu_index)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None
            return
        self._t = threading.Thread(target=self._read, daemon=True)
        self._t.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self._t.join(timeout=2)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# Distributed plumbing
# ---------------------------------------------------------------------------
def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return world, rank, local


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def min_over_ranks(x: float, world: int) -> float:
    return -max_over_ranks(-float(x), world)


# ---------------------------------------------------------------------------
# Our implementation
# ---------------------------------------------------------------------------
def run_ours(args, world, rank, local) -> dict | None:
    """The c2 headline: one inject launch per step over the rank's share of the
    step (all of it at N = 1), timed on the device, then the same step end to
    end through ``inject_donors`` with host buffers, then a seeded sample of
    (request, layer) slices checked against the CPU oracle."""
    from semblend_b200 import _lib
    from semblend_b200 import rope_correction as rc

    dev = torch.device("cuda", local)
    n_req, n_layers = args.requests, args.layers
    h0, h1, l0, l1 = c2_partition(world, rank, n_layers, N_KV_HEADS)
    my_heads, my_layers = h1 - h0, l1 - l0
    rng = np.random.default_rng(SEED)  # the same step (pairs, block tables) on every rank
    pool = int(n_req * (SEQ // BLOCK) * 1.25)
    plans = [make_request_plan(rng) for _ in range(n_req)]
    tables = make_block_tables(rng, n_req, SEQ, pool)
    n_pairs = sum(p[0].shape[0] for p in plans)

    gen = torch.Generator(device=dev).manual_seed(SEED + rank)
    cache = torch.empty(my_layers, pool, 2, my_heads, BLOCK, HEAD_DIM, dtype=torch.bfloat16, device=dev)
    cache.normal_(generator=gen)
    donors = []
    for _ in range(n_req):
        dk = torch.empty(my_layers, 2, my_heads, SEQ, HEAD_DIM, dtype=torch.bfloat16, device=dev)
        dk.normal_(generator=gen)
        donors.append(dk)

    # the slices the oracle checks afterwards: their cache blocks before any write
    crng = np.random.default_rng(SEED + 100 + rank)
    checks = [(int(crng.integers(n_req)), int(crng.integers(my_layers))) for _ in range(args.check_slices)]
    before = {(r, l): cache[l][torch.from_numpy(tables[r].astype(np.int64)).to(dev)].cpu() for r, l in checks}

    # host-side (pinned) step inputs: positions and block tables
    host_pos = [torch.from_numpy(np.stack([d, t])).pin_memory() for d, t, _ in plans]
    host_bt = [torch.from_numpy(b).pin_memory() for b in tables]
    dev_pos = [h.to(dev) for h in host_pos]
    dev_bt = [h.to(dev) for h in host_bt]
    injections = [rc.DonorInjection(donors[r], dev_bt[r], dev_pos[r][0], dev_pos[r][1]) for r in range(n_req)]
    err = _lib.err_counter(dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        rc.inject_donors(cache, injections, rope_base=ROPE_THETA, rotary_style="neox")

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)

    # --- device-resident timed region ---
    clocks = ClockSampler(local)
    clocks.start()
    barrier(world)
    torch.cuda.synchronize(dev)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    with _lib.KernelTimer(args.steps) as kt:  # events on the launch stream around each inject_kernel
        t0.record(stream)
        for _ in range(args.steps):
            step()
        t1.record(stream)
        torch.cuda.synchronize(dev)
    barrier(world)
    clk = clocks.stop()
    total_ms = max_over_ranks(t0.elapsed_time(t1), world)
    kernel_ms_max = max_over_ranks(kt.mean_ms, world)

    # --- A/B: the same launches with the source rows staged through 1-D bulk copies ---
    for _ in range(2):
        rc.inject_donors(cache, injections, rope_base=ROPE_THETA, rotary_style="neox", staging="bulk")
    torch.cuda.synchronize(dev)
    with _lib.KernelTimer(args.steps) as kt_bulk:
        for _ in range(args.steps):
            rc.inject_donors(cache, injections, rope_base=ROPE_THETA, rotary_style="neox", staging="bulk")
        torch.cuda.synchronize(dev)
    bulk_ms_max = max_over_ranks(kt_bulk.mean_ms, world)

    # --- end to end through the public API with host buffers ---
    h2d = sum(h.numel() * h.element_size() for h in host_pos) + sum(h.numel() * h.element_size() for h in host_bt)
    status = torch.empty(1, dtype=torch.int64).pin_memory()

    def e2e_step():
        for r in range(n_req):
            dev_pos[r].copy_(host_pos[r], non_blocking=True)
            dev_bt[r].copy_(host_bt[r], non_blocking=True)
        rc.inject_donors(cache, injections, rope_base=ROPE_THETA, rotary_style="neox")
        status.copy_(err, non_blocking=True)

    for _ in range(max(3, args.warmup // 2)):
        e2e_step()
    torch.cuda.synchronize(dev)
    barrier(world)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), world)
    skipped = int(status.item())

    # --- parity: sampled (request, layer) slices of the final cache against the oracle ---
    chk = check_c2_slices(cache, donors, tables, plans, before, dev)
    ok_all = min_over_ranks(int(chk["matches_oracle"]) and skipped == 0, world)

    elt = 2
    n_blocks = n_req * (SEQ // BLOCK)
    step_bytes = algorithmic_bytes(n_pairs, n_layers, N_KV_HEADS, HEAD_DIM, elt, n_blocks)
    rank_bytes = algorithmic_bytes(n_pairs, my_layers, my_heads, HEAD_DIM, elt, n_blocks)
    ms_per_step = total_ms / args.steps
    value = step_bytes / (ms_per_step * 1e-3) / 1e9
    e2e_value = step_bytes / (e2e_ms / args.steps * 1e-3) / 1e9
    pk = peaks()
    achieved = rank_bytes / (kernel_ms_max * 1e-3) / 1e9
    del cache, donors
    torch.cuda.empty_cache()
    if rank != 0:
        return None
    traffic, traffic_src = (committed_traffic("inject_c2_traffic") if world == 1
                            else (None, "profiled at N = 1 only"))
    cfg = inject_config(n_req, n_layers, world, n_pairs)
    cfg["rank0_share"] = {"kv_heads": [h0, h1], "layers": [l0, l1]}
    return {
        "metric": "RoPE-corrected KV inject GB/s",
        "value": round(value, 2),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) K/V, seeded chunk deltas, recompute set and block tables)",
        "config": cfg,
        "matches_oracle": bool(ok_all),
        "oracle_check": chk,
        "roofline": {
            "bound": "hbm",
            "achieved": round(achieved, 1),
            "peak": pk["hbm_gbs"],
            "unit": "GB/s",
            "frac": round(achieved / pk["hbm_gbs"], 4),
            "peak_source": pk["source"],
            "traffic": traffic,
            "traffic_source": traffic_src,
            "algorithmic_bytes_per_launch": rank_bytes,
            "kernel": "inject_kernel<bf16, 8> (slowest rank; CUDA events on the launch stream)",
            "kernel_ms": round(kernel_ms_max, 4),
            "staging_ab": {"bulk_staged_kernel_ms": round(bulk_ms_max, 4),
                           "bulk_staged_frac": round(rank_bytes / (bulk_ms_max * 1e-3) / 1e9 / pk["hbm_gbs"], 4),
                           "note": "inject_bulk_kernel (SB_INJECT_BULK_STAGED: source rows through 1-D "
                                   "cp.async.bulk into a 3-stage shared-memory ring) on the same step; the "
                                   "direct path above is the default"},
        },
        "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": 8, "api": "semblend_b200.rope_correction.inject_donors",
                "skipped_pairs": skipped},
        "gpu_launches": args.steps,
        "clocks": clk,
    }


def check_c2_slices(cache, donors, tables, plans, before, dev) -> dict:
    """Compare (request, layer) slices of the injected cache with the oracle
    run on the same slice's donor rows and pre-inject blocks: V rows and rows
    no pair targets bit-exact, K rows within 1 bf16 ulp at the magnitude of
    their RoPE pair; every pair of the slice must be applied."""
    from oracle import rope as orope

    worst_elem, worst_pair, ok, applied_all = 0, 0.0, True, True
    for (r, l), blk in before.items():
        d, t, _ = plans[r]
        bt = torch.from_numpy(tables[r].astype(np.int64))
        got = cache[l][bt.to(dev)].cpu()
        want, applied = orope.rope_correct_scatter_paged(
            blk, donors[r][l].cpu(), torch.arange(bt.shape[0], dtype=torch.int32), torch.from_numpy(d),
            torch.from_numpy(t), ROPE_THETA, "neox", return_applied=True)
        applied_all &= applied == d.shape[0]
        ok &= torch.equal(got[:, 1].view(torch.int16), want[:, 1].view(torch.int16))
        hit = torch.zeros(bt.shape[0] * BLOCK, dtype=torch.bool)
        hit[torch.from_numpy(t.astype(np.int64))] = True
        hit = hit.view(-1, BLOCK)
        gk = got[:, 0].permute(0, 2, 1, 3)  # [blocks, bs, H, D]
        wk = want[:, 0].permute(0, 2, 1, 3)
        ok &= torch.equal(gk[~hit].contiguous().view(torch.int16), wk[~hit].contiguous().view(torch.int16))
        e, p = ulp_report(gk[hit], wk[hit], "neox")
        worst_elem, worst_pair = max(worst_elem, e), max(worst_pair, p)
    ok = bool(ok and applied_all and worst_pair <= 1.0)
    return {"matches_oracle": ok, "slices": [list(k) for k in before], "all_pairs_applied": bool(applied_all),
            "k_max_ulp_elem": worst_elem, "k_max_ulp_pair_scale": round(worst_pair, 4),
            "bar": "V and untouched rows bit-exact; K <= 1 bf16 ulp at its RoPE pair's magnitude"}


# ---------------------------------------------------------------------------
# Component: single-layer fp32 inject (configs[0], c1)
# ---------------------------------------------------------------------------
C1_TOKENS, C1_CHUNKS, C1_POOL, C1_BLOCKS = 4096, 16, 1024, 256


def make_c1_inputs(seed: int = SEED):
    """c1: donor K/V fp32 N(0,1) [2, 4 heads, 4096, 128]; 16 chunks of 256
    tokens moved by a seeded permutation (donor chunk i -> target chunk pi(i));
    paged cache [1024, 2, 4, 16, 128] fp32 whose block table is the first 256
    entries of a seeded shuffle of the 1024 blocks.  Returns (donor, cache,
    block_table int32, donor_positions int32, target_positions int32), on the CPU."""
    rng = np.random.default_rng(seed)
    g = torch.Generator().manual_seed(seed)
    donor = torch.randn(2, N_KV_HEADS, C1_TOKENS, HEAD_DIM, generator=g)
    cache = torch.randn(C1_POOL, 2, N_KV_HEADS, BLOCK, HEAD_DIM, generator=g)
    bt = rng.permutation(C1_POOL)[:C1_BLOCKS].astype(np.int32)
    pi = rng.permutation(C1_CHUNKS)
    j = np.arange(CHUNK)
    d = np.concatenate([i * CHUNK + j for i in range(C1_CHUNKS)]).astype(np.int32)
    t = np.concatenate([pi[i] * CHUNK + j for i in range(C1_CHUNKS)]).astype(np.int32)
    return donor, cache, torch.from_numpy(bt), torch.from_numpy(d), torch.from_numpy(t)


def run_c1(args, local: int) -> dict:
    """c1 through ``rope_correct_scatter_paged``: one call = one launch moving
    33.6 MB.  Timed as a CUDA graph of 64 calls cycling over 8 replicas of the
    inputs (640 MiB allocated, 256 MiB touched between two uses of a replica:
    more than L2), since one call is a few microseconds and launch overhead
    would otherwise dominate; the kernel's own time from library events on
    eager launches; e2e through the same API with positions and block table
    copied from pinned host memory and the skipped-pair count read back."""
    from oracle import rope as orope
    from semblend_b200 import _lib
    from semblend_b200 import rope_correction as rc

    dev = torch.device("cuda", local)
    donor_h, cache_h, bt_h, d_h, t_h = make_c1_inputs(SEED + 1)
    reps = 8
    donors = [donor_h.to(dev) for _ in range(reps)]
    caches = [cache_h.to(dev) for _ in range(reps)]
    bt, dp, tp = bt_h.to(dev), d_h.to(dev), t_h.to(dev)

    def call(i, b=bt, d=dp, t=tp):
        rc.rope_correct_scatter_paged(caches[i], donors[i], b, d, t, rope_base=ROPE_THETA, rotary_style="neox")

    for i in range(reps):
        call(i)
    torch.cuda.synchronize(dev)
    # parity of the whole c1 output against the oracle (fp32 bar: 1e-5 relative at the RoPE pair's magnitude)
    want, applied = orope.rope_correct_scatter_paged(cache_h, donor_h, bt_h, d_h, t_h, ROPE_THETA, "neox",
                                                     return_applied=True)
    got = caches[0].cpu()
    v_ok = torch.equal(got[:, 1].view(torch.int32), want[:, 1].view(torch.int32))
    gk, wk = got[:, 0], want[:, 0]
    diff = (gk - wk).abs()
    a, b_ = wk[..., : HEAD_DIM // 2], wk[..., HEAD_DIM // 2:]
    n = torch.sqrt(a * a + b_ * b_)
    rel = float((diff / torch.cat([n, n], dim=-1).clamp_min(1e-30)).max())
    ok = bool(v_ok and rel <= 1e-5 and applied == C1_TOKENS)

    stream = torch.cuda.current_stream(dev)
    calls = 64
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for c in range(calls):
            call(c % reps)
    for _ in range(max(args.warmup, 3)):
        graph.replay()
    torch.cuda.synchronize(dev)
    replays = max(5, min(args.steps, 50))
    clocks = ClockSampler(local)
    clocks.start()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(replays):
        graph.replay()
    t1.record(stream)
    torch.cuda.synchronize(dev)
    clk = clocks.stop()
    ms_call = t0.elapsed_time(t1) / (replays * calls)
    with _lib.KernelTimer(4 * reps) as kt:
        for r in range(4):
            for i in range(reps):
                call(i)
        torch.cuda.synchronize(dev)

    # end to end: positions and block table from pinned host memory, skipped count back
    hd, ht, hb = d_h.pin_memory(), t_h.pin_memory(), bt_h.pin_memory()
    bd, btd, bb = torch.empty_like(dp), torch.empty_like(tp), torch.empty_like(bt)
    err = _lib.err_counter(dev)
    hs = torch.empty(1, dtype=torch.int64).pin_memory()

    def e2e(i):
        bd.copy_(hd, non_blocking=True)
        btd.copy_(ht, non_blocking=True)
        bb.copy_(hb, non_blocking=True)
        call(i, bb, bd, btd)
        hs.copy_(err, non_blocking=True)

    for i in range(reps):
        e2e(i)
    torch.cuda.synchronize(dev)
    n_e2e = 8 * reps
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for c in range(n_e2e):
        e2e(c % reps)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = e0.elapsed_time(e1) / n_e2e
    skipped = int(hs.item())

    # the reference's CPU path (oracle port) on the same c1 call, ~3 s of CPU work
    torch.set_num_threads(os.cpu_count() or 1)
    cpu_s, n_cpu = 0.0, 0
    while cpu_s < 3.0:
        c0 = time.perf_counter()
        orope.rope_correct_scatter_paged(cache_h, donor_h, bt_h, d_h, t_h, ROPE_THETA, "neox", inplace=True)
        cpu_s += time.perf_counter() - c0
        n_cpu += 1
    nbytes = algorithmic_bytes(C1_TOKENS, 1, N_KV_HEADS, HEAD_DIM, 4, C1_BLOCKS)
    pk = peaks()
    # a launch of a few microseconds is timed from the graph (kernel + the gap to the next
    # launch, an upper bound on the kernel's time); events around one eager launch add their own
    # overhead and are reported beside it
    ach = nbytes / (ms_call * 1e-3) / 1e9
    deltas = (t_h - d_h).numpy()
    return {
        "component": "c1_inject",
        "metric": "RoPE-corrected KV inject GB/s", "value": round(nbytes / (ms_call * 1e-3) / 1e9, 2), "unit": "GB/s",
        "higher_is_better": True, "ms_per_step": round(ms_call, 5), "steps": replays * calls, "dtype": "f32",
        "config": {"workload": "c1: one layer, donor K/V fp32 [4096 tok, 4 KV heads, 128], 16 chunks x 256 "
                               "permuted (seeded), block 16, block table = 256 of 1024 blocks (seeded shuffle), "
                               "neox RoPE theta 1e6; one step = one rope_correct_scatter_paged call",
                   "realised_deltas": [int(deltas.min()), int(deltas.max())],
                   "timing": f"CUDA graph of {calls} calls over {reps} input replicas (640 MiB; inputs larger "
                             "than L2 between reuses)", "seed": SEED + 1},
        "matches_oracle": ok,
        "oracle_check": {"v_bit_exact": bool(v_ok), "k_max_rel_err_pair_scale": rel, "pairs_applied": applied,
                         "bar": "V bit-exact, K within 1e-5 relative at its RoPE pair's magnitude"},
        "roofline": {"bound": "hbm", "kernel": "inject_kernel<float, 4>", "achieved": round(ach, 1),
                     "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": round(ach / pk["hbm_gbs"], 4),
                     "kernel_ms": round(ms_call, 5), "kernel_time": "per call inside the CUDA graph (kernel + "
                     "launch gap)", "eager_event_ms": round(kt.mean_ms, 5),
                     "algorithmic_bytes_per_launch": nbytes, "traffic": None, "peak_source": pk["source"]},
        "e2e": {"value": round(nbytes / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                "h2d_bytes_per_step": int(hd.numel() * 4 + ht.numel() * 4 + hb.numel() * 4),
                "d2h_bytes_per_step": 8, "api": "semblend_b200.rope_correction.rope_correct_scatter_paged",
                "skipped_pairs": skipped},
        "cpu_baseline": {"value": round(nbytes * n_cpu / cpu_s / 1e9, 4), "unit": "GB/s",
                         "cores": torch.get_num_threads(), "kind": "port",
                         "sample": f"the whole c1 call {n_cpu} times through oracle.rope.rope_correct_scatter_paged "
                                   f"(in place), {cpu_s:.1f} s"},
        "gpu_launches": replays * calls,
        "clocks": clk,
    }

# ---------------------------------------------------------------------------
# Component: donor search (configs[2], c3)
# ---------------------------------------------------------------------------
S_ROWS, S_DIM, S_QUERIES, S_K, S_THR, S_CENTERS = 1 << 20, 384, 4096, 8, 0.60, 256


def make_search_inputs(dev: torch.device, seed: int, n_rows: int = S_ROWS, n_q: int = S_QUERIES):
    """256 isotropic Gaussian clusters (centres N(0,1), sigma 0.3), rows
    L2-normalised; queries 70 % from the clusters, 30 % uniform on the sphere."""
    g = torch.Generator(device=dev).manual_seed(seed)
    centers = torch.randn(S_CENTERS, S_DIM, generator=g, device=dev)
    lab = torch.randint(0, S_CENTERS, (n_rows,), generator=g, device=dev)
    emb = torch.empty(n_rows, S_DIM, device=dev)
    for a in range(0, n_rows, 1 << 18):  # chunked to bound temporaries
        b = min(a + (1 << 18), n_rows)
        x = centers[lab[a:b]] + 0.3 * torch.randn(b - a, S_DIM, generator=g, device=dev)
        emb[a:b] = x / x.norm(dim=1, keepdim=True)
    nc = int(round(0.7 * n_q))
    qc = centers[torch.randint(0, S_CENTERS, (nc,), generator=g, device=dev)]
    qc = qc + 0.3 * torch.randn(nc, S_DIM, generator=g, device=dev)
    qu = torch.randn(n_q - nc, S_DIM, generator=g, device=dev)
    queries = torch.cat([qc, qu])
    return emb, queries


def run_search(args, local: int) -> dict:
    from oracle import search as osearch
    from semblend_b200 import _lib
    from semblend_b200.search import DeviceDonorMatrix, cosine_topk_async

    dev = torch.device("cuda", local)
    n_rows = args.search_rows
    emb, queries = make_search_inputs(dev, SEED + 3, n_rows=n_rows)
    m = DeviceDonorMatrix(n_rows, S_DIM, dev)
    m.write_range(0, emb)
    out = (torch.empty(S_QUERIES, S_K, dtype=torch.int64, device=dev),
           torch.empty(S_QUERIES, S_K, dtype=torch.float32, device=dev))
    status = torch.zeros(1, dtype=torch.int32, device=dev)

    def step(q):
        return cosine_topk_async(m.emb, m.emb16, m.valid, m.stats, q, S_K, S_THR, status=status,
                                 workspace_owner=m, out=out)

    for _ in range(args.warmup):
        step(queries)
    torch.cuda.synchronize(dev)
    assert int(status.item()) == 0, f"search status {int(status.item())}"
    steps = max(5, args.steps // 10)
    stream = torch.cuda.current_stream(dev)
    # eager launches: the screening kernel's own time (library-recorded events)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with _lib.KernelTimer(steps) as kt:
        t0.record(stream)
        for _ in range(steps):
            step(queries)
        t1.record(stream)
        torch.cuda.synchronize(dev)
    eager_ms = t0.elapsed_time(t1) / steps
    # the step as one CUDA graph (query preparation, screening, rescoring), as a serving loop runs it
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step(queries)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize(dev)
    clocks = ClockSampler(local)
    clocks.start()
    t0.record(stream)
    for _ in range(steps):
        graph.replay()
    t1.record(stream)
    torch.cuda.synchronize(dev)
    clk = clocks.stop()
    st = int(status.item())
    ms = t0.elapsed_time(t1) / steps

    # end to end: pinned host queries in, ids + scores out
    hq = queries.cpu().pin_memory()
    dq = torch.empty_like(queries)
    hi = torch.empty(S_QUERIES, S_K, dtype=torch.int64).pin_memory()
    hs = torch.empty(S_QUERIES, S_K, dtype=torch.float32).pin_memory()
    graph_e2e = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph_e2e):
        step(dq)

    def e2e_step():
        dq.copy_(hq, non_blocking=True)
        graph_e2e.replay()
        i, s = out
        hi.copy_(i, non_blocking=True)
        hs.copy_(s, non_blocking=True)

    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = e0.elapsed_time(e1) / steps

    # cross-check a query sample against the oracle, and time the oracle there
    ids_g, sc_g = out[0].cpu().numpy(), out[1].cpu().numpy()
    n_sample = 32 if n_rows == S_ROWS else 64
    sample = np.random.default_rng(SEED).choice(S_QUERIES, n_sample, replace=False)
    E = m.emb.cpu().numpy()
    valid = np.ones(n_rows, bool)
    Qs = queries.cpu().numpy()[sample]
    torch.set_num_threads(os.cpu_count() or 1)
    c0 = time.perf_counter()
    ids_o, sc_o = osearch.topk_batch(E, valid, Qs, S_THR, S_K)
    cpu_s = (time.perf_counter() - c0) / len(sample)
    # a stronger CPU bound: one fp32 GEMM per 256-query block instead of per-query matvecs
    qb = queries.cpu().numpy()[:512]
    c0 = time.perf_counter()
    osearch.topk_batch_gemm(E, valid, qb, S_THR, S_K)
    cpu_gemm_s = (time.perf_counter() - c0) / qb.shape[0]
    agree = int(sum(
        np.array_equal(ids_o[j][ids_o[j] >= 0], ids_g[q][ids_g[q] >= 0])
        or np.allclose(sc_o[j][: (ids_o[j] >= 0).sum()], sc_g[q][: (ids_o[j] >= 0).sum()], atol=1e-6)
        for j, q in enumerate(sample)))
    flops = 2.0 * n_rows * S_QUERIES * S_DIM
    pk = peaks()
    achieved = flops / (kt.mean_ms * 1e-3) / 1e12
    hits = float((out[0] >= 0).float().mean().item())
    cand = m._ws[: 4 * S_QUERIES].view(torch.int32).float()  # per-query screening candidates (workspace head)
    return {
        "component": "c3_search",
        "metric": "donor search q/s",
        "value": round(S_QUERIES / (ms * 1e-3), 1),
        "unit": "q/s",
        "ms_per_step": round(ms, 4),
        "steps": steps,
        "matches_oracle": bool(agree == len(sample) and st == 0),
        "config": {"workload": f"c3{'' if n_rows == S_ROWS else ' (reduced)'}: {n_rows:,} x 384 fp32 donors "
                               "(256 clusters, sigma 0.3, L2-normalised), 4096 queries (70% clustered, 30% "
                               "uniform), top-8, threshold 0.60",
                   "fill": round(hits, 4), "status": st, "eager_launch_ms": round(eager_ms, 4),
                   "step": "one CUDA graph per step (query preparation, screening, rescoring)",
                   "candidates_per_query": {"mean": round(float(cand.mean()), 1), "max": int(cand.max())}},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": round(achieved / pk["bf16_tflops"], 4), "peak_source": pk["source"],
                     "kernel": "screen_kernel<8> (fp16 tcgen05, 2*N*Q*d flops)", "kernel_ms": round(kt.mean_ms, 4),
                     "traffic": None},
        "e2e": {"value": round(S_QUERIES / (e2e_ms * 1e-3), 1), "unit": "q/s",
                "h2d_bytes_per_step": hq.numel() * 4, "d2h_bytes_per_step": S_QUERIES * S_K * 12},
        "gpu_launches": steps * 3,
        "clocks": clk,
        "oracle_check": f"{agree}/{len(sample)} sampled queries equivalent (ids exact, or the same scores "
                        "within 1e-6 where ties reorder ids)",
        "cpu_baseline": {"value": round(1.0 / cpu_s, 3), "unit": "q/s", "cores": torch.get_num_threads(),
                         "kind": "port", "sample": f"{len(sample)} queries through oracle.search.topk_batch "
                         f"(the reference's per-query numpy stage) on the full {n_rows:,} x 384 matrix, "
                         f"{cpu_s * len(sample):.1f} s",
                         "batched_gemm_q_per_s": round(1.0 / cpu_gemm_s, 2),
                         "batched_gemm_sample": "512 queries, one fp32 numpy GEMM per 256-query block "
                                                "(oracle.search.topk_batch_gemm)"},
    }


def run_search_sharded(args, world: int, rank: int, local: int) -> dict | None:
    """c3 with the donor rows split across `world` GPUs (strong scaling): each
    rank searches its shard exactly, one NCCL all_gather_into_tensor exchanges
    the per-shard top-8 records, every rank merges."""
    from semblend_b200 import _lib
    from semblend_b200.search import cosine_topk_async
    from semblend_b200.sharded_search import ShardedDonorMatrix

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    n_rows = args.search_rows
    # every rank generates the same matrix and keeps its shard (seeded on the device)
    emb, queries = make_search_inputs(dev, SEED + 3, n_rows=n_rows)
    m = ShardedDonorMatrix(n_rows, S_DIM, device=dev)
    m.write_range(0, emb)
    e_host = emb.cpu().numpy() if rank == 0 else None  # rank 0 checks merged results against the oracle
    del emb
    torch.cuda.empty_cache()

    steps = max(30, args.steps)  # a step is well under a millisecond
    # two query batches in flight: batch i's rescoring, all-gather and merge overlap batch i+1's screening
    m.search_batches([queries] * max(args.warmup, 2), S_K, S_THR)
    torch.cuda.synchronize(dev)
    stream = torch.cuda.current_stream(dev)
    # Clocks come from a separate run of the same loop (~0.3 s): nvidia-smi starting up and
    # polling beside the timed steps stalled rank 0's launching thread (2-3x slower steps at
    # 8 GPUs), which a loop of eager launches per step cannot hide.
    clocks = ClockSampler(local) if rank == 0 else None
    if clocks:
        clocks.start()
        time.sleep(0.5)
    barrier(world)
    m.search_batches([queries] * 600, S_K, S_THR)
    torch.cuda.synchronize(dev)
    barrier(world)
    clk = clocks.stop() if clocks else None
    if clk is not None:
        clk["window"] = "600 further batches of the same loop (not the timed steps)"
    barrier(world)
    torch.cuda.synchronize(dev)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    res = m.search_batches([queries] * steps, S_K, S_THR)
    t1.record(stream)
    torch.cuda.synchronize(dev)
    barrier(world)
    ids, sc, status = res[-1]
    st = 0
    for _, _, s_ in res[-2:]:
        for v in s_.reshape(-1).tolist():
            st |= int(v)
    ms = max_over_ranks(t0.elapsed_time(t1) / steps, world)

    # one batch at a time (exchange not overlapped), for the overhead split
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    s0.record(stream)
    for _ in range(steps):
        m.search_async(queries, S_K, S_THR)
    s1.record(stream)
    torch.cuda.synchronize(dev)
    serial_ms = max_over_ranks(s0.elapsed_time(s1) / steps, world)

    # the shard search alone (no exchange, no merge)
    lm = m.local
    lo = (torch.empty(S_QUERIES, S_K, dtype=torch.int64, device=dev),
          torch.empty(S_QUERIES, S_K, dtype=torch.float32, device=dev))
    lst = torch.zeros(1, dtype=torch.int32, device=dev)
    l0, l1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with _lib.KernelTimer(steps) as kt:  # the screening kernel's own time (eager launches)
        l0.record(stream)
        for _ in range(steps):
            cosine_topk_async(lm.emb, lm.emb16, lm.valid, lm.stats, queries, S_K, S_THR, n_rows=m.n_local,
                              id_offset=m.row_begin, status=lst, workspace_owner=lm, out=lo)
        l1.record(stream)
        torch.cuda.synchronize(dev)
    local_ms = max_over_ranks(l0.elapsed_time(l1) / steps, world)
    kms = max_over_ranks(kt.mean_ms, world)

    # end to end: pinned host query batches in (copied on a copy stream), merged ids +
    # scores of every batch back to pinned host memory (every rank)
    hq = [queries.cpu().pin_memory() for _ in range(2)]
    hi = [torch.empty(S_QUERIES, S_K, dtype=torch.int64).pin_memory() for _ in range(2)]
    hs = [torch.empty(S_QUERIES, S_K, dtype=torch.float32).pin_memory() for _ in range(2)]

    def to_host(i, ids_, sc_):
        hi[i % 2].copy_(ids_, non_blocking=True)
        hs[i % 2].copy_(sc_, non_blocking=True)

    m.search_batches([hq[i % 2] for i in range(3)], S_K, S_THR, on_result=to_host)
    torch.cuda.synchronize(dev)
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    m.search_batches([hq[i % 2] for i in range(steps)], S_K, S_THR, on_result=to_host)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / steps, world)
    fill = float((ids >= 0).float().mean().item())
    if rank != 0:
        return None
    # the merged result of 8 sampled queries against the oracle (the reference's per-query stage)
    from oracle import search as osearch

    sample = np.random.default_rng(SEED).choice(S_QUERIES, 8, replace=False)
    ids_o, sc_o = osearch.topk_batch(e_host, np.ones(n_rows, bool), queries.cpu().numpy()[sample], S_THR, S_K)
    ids_g, sc_g = ids.cpu().numpy()[sample], sc.cpu().numpy()[sample]
    agree = int(sum(
        np.array_equal(ids_o[j][ids_o[j] >= 0], ids_g[j][ids_g[j] >= 0])
        or np.allclose(sc_o[j][: (ids_o[j] >= 0).sum()], sc_g[j][: (ids_o[j] >= 0).sum()], atol=1e-6)
        for j in range(len(sample))))
    pk = peaks()
    flops_rank = 2.0 * (m.row_end - m.row_begin) * S_QUERIES * S_DIM
    achieved = flops_rank / (kms * 1e-3) / 1e12
    return {
        "component": "c3_search_sharded",
        "matches_oracle": bool(agree == len(sample) and st == 0),
        "oracle_check": f"{agree}/{len(sample)} sampled queries of the merged result equivalent to the oracle's",
        "metric": "donor search q/s",
        "value": round(S_QUERIES / (ms * 1e-3), 1),
        "unit": "q/s",
        "n_gpus": world,
        "scaling": "strong",
        "ms_per_step": round(ms, 4),
        "steps": steps,
        "config": {"workload": f"c3: {n_rows:,} x 384 donors split over {world} GPUs, 4096 queries, top-8, "
                               "threshold 0.60; per-shard exact top-8, one NCCL all_gather_into_tensor of "
                               "the shard records, k-way merge on every rank; two query batches in flight "
                               "(batch i's exact rescoring, exchange and merge run on a second stream beside "
                               "batch i+1's screening; the exchange on its own NCCL group with the efficiency "
                               "CTA policy)",
                   "one_batch_at_a_time_ms": round(serial_ms, 4),
                   "fill": round(fill, 4), "status": st,
                   "shard_search_ms": round(local_ms, 4),
                   "exchange_and_merge_ms_serial": round(serial_ms - local_ms, 4)},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": pk["bf16_tflops"],
                     "unit": "TFLOP/s", "frac": round(achieved / pk["bf16_tflops"], 4),
                     "peak_source": pk["source"], "kernel": "screen_kernel<8> on the slowest rank's shard",
                     "kernel_ms": round(kms, 4), "traffic": None},
        "e2e": {"value": round(S_QUERIES / (e2e_ms * 1e-3), 1), "unit": "q/s",
                "h2d_bytes_per_step": hq[0].numel() * 4, "d2h_bytes_per_step": S_QUERIES * S_K * 12},
        "gpu_launches": steps * (4 if world == 1 else 5),
        "clocks": clk,
    }


# ---------------------------------------------------------------------------
# Component: partial-prefill attention (configs[3], c4)
# ---------------------------------------------------------------------------
A_B, A_HQ, A_HKV, A_S, A_D, A_SPANS, A_TAIL, A_FRAC = 4, 28, 4, 32768, 128, 64, 512, 0.10


def make_attention_mask(rng: np.random.Generator, S: int) -> np.ndarray:
    """64 seeded contiguous recompute spans plus the final 512 tokens, 10 % of
    positions in total."""
    mask = np.zeros(S, bool)
    tail = min(A_TAIL, S // 4)
    mask[S - tail:] = True
    budget = int(A_FRAC * S) - tail
    starts = np.sort(rng.choice(S - tail, A_SPANS, replace=False))
    lens = 1 + rng.multinomial(max(budget - A_SPANS, 0), np.ones(A_SPANS) / A_SPANS)
    for a, ln in zip(starts, lens):
        mask[a : min(a + ln, S - tail)] = True
    return mask


def attention_flops(masks: np.ndarray, n_q_heads: int, head_dim: int) -> float:
    """4 * D * Hq * sum over compute rows of (p + 1): causal, inclusive, no padding."""
    total = 0.0
    for m in masks:
        pos = np.nonzero(m)[0].astype(np.float64)
        total += float((pos + 1).sum())
    return 4.0 * head_dim * n_q_heads * total


def run_attention(args, local: int) -> dict:
    from oracle import attention as oatt
    from semblend_b200 import _lib
    from semblend_b200 import triton_kernels as tk

    dev = torch.device("cuda", local)
    B, S = args.attn_batch, args.attn_seq
    rng = np.random.default_rng(SEED + 5)
    masks = np.stack([make_attention_mask(rng, S) for _ in range(B)])
    g = torch.Generator(device=dev).manual_seed(SEED + 5)
    scale = 1.0 / np.sqrt(A_D)
    q = (torch.randn(B, A_HQ, S, A_D, generator=g, device=dev) * scale).to(torch.bfloat16)
    k = (torch.randn(B, A_HKV, S, A_D, generator=g, device=dev) * scale).to(torch.bfloat16)
    v = (torch.randn(B, A_HKV, S, A_D, generator=g, device=dev) * scale).to(torch.bfloat16)
    mask_d = torch.from_numpy(masks).to(dev)
    rows, counts = tk.mask_to_rows(mask_d)
    out = torch.zeros_like(q)
    status = torch.zeros(1, dtype=torch.int32, device=dev)

    def step():
        tk.gqa_partial_attention(q, k, v, rows, counts, out, max_rows=S, status=status)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    steps = max(5, args.steps // 10)
    stream = torch.cuda.current_stream(dev)
    clocks = ClockSampler(local)
    clocks.start()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with _lib.KernelTimer(steps) as kt:
        t0.record(stream)
        for _ in range(steps):
            step()
        t1.record(stream)
        torch.cuda.synchronize(dev)
    clk = clocks.stop()
    st = int(status.item())
    ms = t0.elapsed_time(t1) / steps
    flops = attention_flops(masks, A_HQ, A_D)

    # end to end through the reference API: the step's compute mask from pinned
    # host memory in, per-batch row counts and the kernel status out
    hmask = torch.from_numpy(masks).pin_memory()
    dmask = torch.empty_like(mask_d)
    hres = torch.empty(B + 1, dtype=torch.int32).pin_memory()

    def e2e_step():
        dmask.copy_(hmask, non_blocking=True)
        o = tk.partial_prefill_attention(q, k, v, dmask)
        r, c = tk.mask_to_rows(dmask)
        hres[:B].copy_(c, non_blocking=True)
        return o

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = e0.elapsed_time(e1) / steps

    # CPU port on a seeded sample of rows of batch element 0 (GQA-expanded),
    # also used to cross-check the GPU rows
    pos0 = np.nonzero(masks[0])[0]
    order = np.random.default_rng(SEED).permutation(pos0)
    qc, kc, vc = q[0].float().cpu(), k[0].float().cpu(), v[0].float().cpu()
    kk, vv = oatt.expand_kv_heads(kc, A_HQ), oatt.expand_kv_heads(vc, A_HQ)
    torch.set_num_threads(os.cpu_count() or 1)
    done, wants, cpu_s = [], [], 0.0
    for c in range(0, order.shape[0], 64):  # ~8 s of CPU work in seeded 64-row batches
        rows_c = np.sort(order[c : c + 64])
        c0 = time.perf_counter()
        wants.append(oatt.partial_prefill_attention_blocked(qc, kk, vv, torch.from_numpy(rows_c), block=8))
        cpu_s += time.perf_counter() - c0
        done.append(rows_c)
        if cpu_s >= 8.0:
            break
    sample = np.concatenate(done)
    want = torch.cat(wants, dim=1)
    got = out[0][:, torch.from_numpy(sample).to(dev), :].float().cpu()
    max_err = float((got - want).abs().max())
    cpu_flops = 4.0 * A_D * A_HQ * float((sample + 1).sum())
    pk = peaks()
    achieved = flops / (kt.mean_ms * 1e-3) / 1e12
    return {
        "component": "c4_attention",
        "matches_oracle": bool(max_err <= 2e-2 and st == 0),
        "metric": "partial-prefill attention TFLOP/s",
        "value": round(flops / (ms * 1e-3) / 1e12, 2),
        "unit": "TFLOP/s",
        "ms_per_step": round(ms, 4),
        "steps": steps,
        "config": {"workload": f"c4{'' if (B, S) == (A_B, A_S) else ' (reduced)'}: batch {B}, 28 q heads / 4 KV "
                               f"heads, head_dim 128, bf16, S={S}, compute rows = 64 seeded spans + final 512 "
                               f"(10%), fp32 softmax", "compute_rows": int(masks.sum()),
                   "flops_per_step": flops, "status": st},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": round(achieved / pk["bf16_tflops"], 4), "peak_source": pk["source"],
                     "kernel": "attn_tc_kernel<bf16> (tcgen05, 4*D*Hq*sum(p+1) flops)",
                     "kernel_ms": round(kt.mean_ms, 4), "traffic": None},
        "e2e": {"value": round(flops / (e2e_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
                "h2d_bytes_per_step": int(hmask.numel()), "d2h_bytes_per_step": 4 * B,
                "api": "semblend_b200.triton_kernels.partial_prefill_attention"},
        "gpu_launches": steps,
        "clocks": clk,
        "oracle_check": f"max |gpu - fp32 oracle| = {max_err:.2e} over {sample.shape[0]} sampled rows x 28 heads "
                        "(bar 2e-2)",
        "cpu_baseline": {"value": round(cpu_flops / cpu_s / 1e12, 6), "unit": "TFLOP/s",
                         "cores": torch.get_num_threads(), "kind": "port",
                         "sample": f"{sample.shape[0]} seeded rows of batch element 0 through "
                                   f"oracle.attention (fp32, GQA-expanded), {cpu_s:.1f} s; TFLOP/s by the same "
                                   "flop formula"},
    }


def run_attention_sharded(args, world: int, rank: int, local: int) -> dict | None:
    """c4 split over `world` GPUs by (batch element, KV head) units with no
    collective (strong scaling): heads first (N | 4: 4/N KV heads and their 28/4
    query heads each, every batch element), then batch elements (N = 8: one KV
    head x 2 batch elements).  Every rank builds the same inputs and runs its
    share in one launch; value = the step's flops over the slowest rank's time."""
    from oracle import attention as oatt
    from semblend_b200 import _lib
    from semblend_b200 import triton_kernels as tk

    dev = torch.device("cuda", local)
    B, S = args.attn_batch, args.attn_seq
    h0, h1, b0, b1 = c2_partition(world, rank, n_layers=B, n_heads=A_HKV)
    g = A_HQ // A_HKV
    rng = np.random.default_rng(SEED + 5)
    masks = np.stack([make_attention_mask(rng, S) for _ in range(B)])
    gen = torch.Generator(device=dev).manual_seed(SEED + 5)
    scale = 1.0 / np.sqrt(A_D)
    q = (torch.randn(B, A_HQ, S, A_D, generator=gen, device=dev) * scale).to(torch.bfloat16)
    k = (torch.randn(B, A_HKV, S, A_D, generator=gen, device=dev) * scale).to(torch.bfloat16)
    v = (torch.randn(B, A_HKV, S, A_D, generator=gen, device=dev) * scale).to(torch.bfloat16)
    rows, counts = tk.mask_to_rows(torch.from_numpy(masks).to(dev))
    out = torch.zeros_like(q)
    qs, ks, vs, os_ = (q[b0:b1, g * h0:g * h1], k[b0:b1, h0:h1], v[b0:b1, h0:h1], out[b0:b1, g * h0:g * h1])
    rs, cs = rows[b0:b1], counts[b0:b1]
    status = torch.zeros(1, dtype=torch.int32, device=dev)

    def step():
        tk.gqa_partial_attention(qs, ks, vs, rs, cs, os_, max_rows=S, status=status)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    steps = max(5, args.steps // 10)
    stream = torch.cuda.current_stream(dev)
    barrier(world)
    torch.cuda.synchronize(dev)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with _lib.KernelTimer(steps) as kt:
        t0.record(stream)
        for _ in range(steps):
            step()
        t1.record(stream)
        torch.cuda.synchronize(dev)
    barrier(world)
    ms = max_over_ranks(t0.elapsed_time(t1) / steps, world)
    kms = max_over_ranks(kt.mean_ms, world)
    st = int(status.item())
    kms_rank0 = kt.mean_ms
    # end to end: the rank's compute masks from pinned host memory in, its row counts out
    hmask = torch.from_numpy(masks[b0:b1].copy()).pin_memory()
    dmask = torch.empty(hmask.shape, dtype=torch.bool, device=dev)
    hcnt = torch.empty(b1 - b0, dtype=torch.int32).pin_memory()

    def e2e_step():
        dmask.copy_(hmask, non_blocking=True)
        r_, c_ = tk.mask_to_rows(dmask)
        tk.gqa_partial_attention(qs, ks, vs, r_, c_, os_, max_rows=S, status=status)
        hcnt.copy_(c_, non_blocking=True)

    e2e_step()
    torch.cuda.synchronize(dev)
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / steps, world)
    # parity: 64 seeded rows of the rank's first batch element, its query heads, against the fp32 oracle
    pos = np.nonzero(masks[b0])[0]
    sample = np.sort(np.random.default_rng(SEED + rank).choice(pos, 64, replace=False))
    qc = q[b0, g * h0:g * h1].float().cpu()
    kk = oatt.expand_kv_heads(k[b0, h0:h1].float().cpu(), g * (h1 - h0))
    vv = oatt.expand_kv_heads(v[b0, h0:h1].float().cpu(), g * (h1 - h0))
    want = oatt.partial_prefill_attention_blocked(qc, kk, vv, torch.from_numpy(sample), block=8)
    got = out[b0, g * h0:g * h1][:, torch.from_numpy(sample).to(dev), :].float().cpu()
    err = float((got - want).abs().max())
    ok = min_over_ranks(int(err <= 2e-2 and st == 0), world)
    flops = attention_flops(masks, A_HQ, A_D)
    rank_flops = attention_flops(masks[b0:b1], g * (h1 - h0), A_D)
    del q, k, v, out
    torch.cuda.empty_cache()
    if rank != 0:
        return None
    pk = peaks()
    ach = rank_flops / (kms_rank0 * 1e-3) / 1e12
    return {
        "component": "c4_attention_sharded",
        "metric": "partial-prefill attention TFLOP/s", "value": round(flops / (ms * 1e-3) / 1e12, 2),
        "unit": "TFLOP/s", "n_gpus": world, "scaling": "strong", "ms_per_step": round(ms, 4), "steps": steps,
        "matches_oracle": bool(ok),
        "config": {"workload": f"c4 split over {world} GPUs by (batch element, KV head): rank 0 owns KV heads "
                               f"[{h0}, {h1}) x batch [{b0}, {b1}); no collective",
                   "flops_per_step": flops, "slowest_rank_kernel_ms": round(kms, 4)},
        "roofline": {"bound": "tensor", "achieved": round(ach, 1), "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": round(ach / pk["bf16_tflops"], 4), "peak_source": pk["source"],
                     "kernel": "attn_tc_kernel<bf16> on rank 0's share", "kernel_ms": round(kms_rank0, 4),
                     "traffic": None},
        "oracle_check": f"rank 0: max |gpu - fp32 oracle| = {err:.2e} over 64 rows x {g * (h1 - h0)} heads "
                        "(bar 2e-2); every rank checked",
        "e2e": {"value": round(flops / (e2e_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
                "h2d_bytes_per_step": int(hmask.numel()), "d2h_bytes_per_step": 4 * (b1 - b0),
                "api": "semblend_b200.triton_kernels.gqa_partial_attention (rank's mask in, its row counts out)"},
        "gpu_launches": steps,
    }

# ---------------------------------------------------------------------------
# Component: end-to-end reuse step on the Llama-3-70B geometry (configs[4], c5)
# ---------------------------------------------------------------------------
C5_L, C5_HQ, C5_HKV, C5_D, C5_THETA = 80, 64, 8, 128, 5e5
C5_REQ, C5_POOL, C5_SEARCH_ROWS, C5_TP = 64, 64, 262144, 8


def c5_lengths(rng: np.random.Generator, n: int) -> np.ndarray:
    """Lognormal context lengths, median 8K, clipped to [4K, 32K], whole 256-token chunks."""
    x = np.exp(rng.normal(np.log(8192.0), 0.5, n))
    return (np.clip(x, 4096, 32768) // CHUNK * CHUNK).astype(np.int64)


def c5_plan(rng: np.random.Generator, req_len: np.ndarray, donor_len: np.ndarray):
    """Per request: 2-4 donors from the pool, each 256-token chunk either
    recomputed (10-20 % of the request, always its last chunk) or copied from a
    random chunk of one of its donors.  Returns per-request lists of
    (donor index, donor positions, target positions) and the recompute masks."""
    reqs, masks = [], []
    for L in req_len:
        n_chunks = L // CHUNK
        donors = rng.choice(len(donor_len), int(rng.integers(2, 5)), replace=False)
        frac = rng.uniform(0.10, 0.20)
        n_re = max(1, int(round(frac * n_chunks)))
        recompute = set(rng.choice(n_chunks - 1, n_re - 1, replace=False).tolist()) | {n_chunks - 1}
        per_donor = {int(d): ([], []) for d in donors}
        mask = np.zeros(L, bool)
        for c in range(n_chunks):
            t = np.arange(c * CHUNK, (c + 1) * CHUNK)
            if c in recompute:
                mask[t] = True
                continue
            d = int(rng.choice(donors))
            dc = int(rng.integers(0, donor_len[d] // CHUNK))
            per_donor[d][0].append(np.arange(dc * CHUNK, (dc + 1) * CHUNK))
            per_donor[d][1].append(t)
        entries = [(d, np.concatenate(dp).astype(np.int32), np.concatenate(tp).astype(np.int32))
                   for d, (dp, tp) in per_donor.items() if dp]
        reqs.append(entries)
        masks.append(mask)
    return reqs, masks


def c5_cpu_and_check(m, queries, plan, pool, tables, nblk, cache, q, k, v, out, masks, hq, hkv, dev,
                     inj_bytes, attn_flops) -> tuple[dict, dict]:
    """The reference's CPU path (oracle ports) on bounded samples of the c5
    step, each scaled to the whole step by its own work formula, and a parity
    check of the GPU step on samples of each part.  Returns (cpu_baseline,
    oracle_check)."""
    from oracle import attention as oatt
    from oracle import rope as orope
    from oracle import search as osearch

    torch.set_num_threads(os.cpu_count() or 1)
    # search: 4 queries through the reference's per-query stage over the 262,144 rows
    E = m.emb.cpu().numpy()
    valid = np.ones(E.shape[0], bool)
    Qs = queries[:4].cpu().numpy()
    c0 = time.perf_counter()
    osearch.topk_batch(E, valid, Qs, S_THR, S_K)
    search_s = (time.perf_counter() - c0) / 4 * queries.shape[0]
    # inject: request 0's donors at layer 0 (every pair), K/V of the target rows against the GPU cache
    r, layer = 0, 0
    bt = torch.from_numpy(tables[r].astype(np.int64))
    got = cache[layer][bt.to(dev)].cpu()
    work = got.clone()
    inj_s, inj_b, applied_all, v_ok, worst_pair = 0.0, 0, True, True, 0.0
    for d, dp, tp in plan[r]:
        c0 = time.perf_counter()
        _, applied = orope.rope_correct_scatter_paged(
            work, pool[d][layer].cpu(), torch.arange(bt.shape[0], dtype=torch.int32), torch.from_numpy(dp),
            torch.from_numpy(tp), C5_THETA, "neox", return_applied=True, inplace=True)
        inj_s += time.perf_counter() - c0
        applied_all &= applied == dp.shape[0]
        inj_b += algorithmic_bytes(applied, 1, hkv, C5_D, 2, 0)
    inj_b += 4 * int(nblk[r])
    v_ok = torch.equal(got[:, 1].view(torch.int16), work[:, 1].view(torch.int16))
    _, worst_pair = ulp_report(got[:, 0], work[:, 0], "neox")
    inj_s_step = inj_s * inj_bytes / inj_b
    # attention: 32 seeded compute rows of request 0 (GQA-expanded fp32 port)
    pos = np.nonzero(masks[0])[0]
    rows = np.sort(np.random.default_rng(SEED).choice(pos, min(32, pos.shape[0]), replace=False))
    qc, kc, vc = q[0].float().cpu(), k[0].float().cpu(), v[0].float().cpu()
    kk, vv = oatt.expand_kv_heads(kc, hq), oatt.expand_kv_heads(vc, hq)
    c0 = time.perf_counter()
    want = oatt.partial_prefill_attention_blocked(qc, kk, vv, torch.from_numpy(rows), block=8)
    att_s = time.perf_counter() - c0
    att_err = float((out[0][:, torch.from_numpy(rows).to(dev), :].float().cpu() - want).abs().max())
    att_flops_sample = 4.0 * C5_D * hq * float((rows + 1).sum())
    att_s_step = att_s * attn_flops / att_flops_sample
    step_s = search_s + inj_s_step + att_s_step
    ok = bool(applied_all and v_ok and worst_pair <= 1.0 and att_err <= 2e-2)
    cpu = {"value": round(step_s * 1e3, 1), "unit": "ms", "cores": torch.get_num_threads(), "kind": "port",
           "sample": f"oracle ports on samples scaled by each part's work formula: search 4 queries x "
                     f"{C5_SEARCH_ROWS:,} rows (x16 -> {search_s:.1f} s), inject request 0 at layer 0 "
                     f"({inj_s:.2f} s for {inj_b / 1e6:.1f} MB -> {inj_s_step:.1f} s), attention 32 rows of "
                     f"request 0 ({att_s:.2f} s -> {att_s_step:.1f} s)",
           "parts_s": {"search": round(search_s, 2), "inject": round(inj_s_step, 2), "attention": round(att_s_step, 2)}}
    chk = {"inject_request0_layer0": {"v_bit_exact": bool(v_ok), "k_max_ulp_pair_scale": round(worst_pair, 4),
                                      "all_pairs_applied": bool(applied_all)},
           "attention_32_rows_max_abs_err": att_err, "matches_oracle": ok}
    return cpu, chk

def run_c5(args, world: int, rank: int, local: int) -> dict | None:
    """One TP-8 rank's slice of the c5 step (1 KV head, 8 query heads): the
    donor search (64 queries over 262,144 x 384), the fused inject of all 80
    layers and every request's donors (one launch), and partial-prefill
    attention for each of the 80 layers (one launch each).  Ranks beyond the
    first take the next KV heads (weak scaling up to 8)."""
    from semblend_b200 import _lib
    from semblend_b200 import rope_correction as rc
    from semblend_b200 import triton_kernels as tk
    from semblend_b200.search import DeviceDonorMatrix, cosine_topk_async

    dev = torch.device("cuda", local)
    n_req, n_pool = args.c5_requests, args.c5_pool
    rng = np.random.default_rng(SEED + 7)  # the same workload on every rank
    req_len, donor_len = c5_lengths(rng, n_req), c5_lengths(rng, n_pool)
    plan, masks_l = c5_plan(rng, req_len, donor_len)
    s_max = int(req_len.max())
    hq, hkv = C5_HQ // C5_TP, C5_HKV // C5_TP
    gen = torch.Generator(device=dev).manual_seed(SEED + 7 + rank)

    # paged target cache [L, blocks, 2, hkv, 16, D] and the donor pool [L, 2, hkv, len, D]
    nblk = (req_len // BLOCK).astype(np.int64)
    pool_blocks = int(nblk.sum() * 1.1)
    perm = rng.permutation(pool_blocks)
    offs = np.concatenate([[0], np.cumsum(nblk)])
    tables = [perm[offs[r] : offs[r + 1]].astype(np.int32) for r in range(n_req)]
    cache = torch.empty(C5_L, pool_blocks, 2, hkv, BLOCK, C5_D, dtype=torch.bfloat16, device=dev)
    cache.normal_(generator=gen)
    pool = []
    for Ld in donor_len:
        t = torch.empty(C5_L, 2, hkv, int(Ld), C5_D, dtype=torch.bfloat16, device=dev)
        t.normal_(generator=gen)
        pool.append(t)
    host_bt = [torch.from_numpy(b).pin_memory() for b in tables]
    dev_bt = [h.to(dev) for h in host_bt]
    host_pos, dev_pos, inj = [], [], []
    n_pairs = 0
    for r, entries in enumerate(plan):
        for d, dp, tp in entries:
            h = torch.from_numpy(np.stack([dp, tp])).pin_memory()
            dpos = h.to(dev)
            host_pos.append(h)
            dev_pos.append(dpos)
            inj.append(rc.DonorInjection(pool[d], dev_bt[r], dpos[0], dpos[1]))
            n_pairs += dp.shape[0]

    # donor search: 262,144 x 384 clustered rows, one query per request
    emb, _ = make_search_inputs(dev, SEED + 8, n_rows=C5_SEARCH_ROWS, n_q=16)
    m = DeviceDonorMatrix(C5_SEARCH_ROWS, S_DIM, dev)
    m.write_range(0, emb)
    del emb
    qg = torch.Generator(device=dev).manual_seed(SEED + 9)
    queries = m.emb[torch.randint(0, C5_SEARCH_ROWS, (n_req,), generator=qg, device=dev)] + \
        0.05 * torch.randn(n_req, S_DIM, generator=qg, device=dev)
    s_out = (torch.empty(n_req, S_K, dtype=torch.int64, device=dev),
             torch.empty(n_req, S_K, dtype=torch.float32, device=dev))
    s_status = torch.zeros(1, dtype=torch.int32, device=dev)

    # attention operands of one layer (the 80 layers reuse them: same shapes, same cost)
    scale = 1.0 / np.sqrt(C5_D)
    q = (torch.randn(n_req, hq, s_max, C5_D, generator=gen, device=dev) * scale).to(torch.bfloat16)
    k = (torch.randn(n_req, hkv, s_max, C5_D, generator=gen, device=dev) * scale).to(torch.bfloat16)
    v = (torch.randn(n_req, hkv, s_max, C5_D, generator=gen, device=dev) * scale).to(torch.bfloat16)
    masks = np.zeros((n_req, s_max), bool)
    for r, mk in enumerate(masks_l):
        masks[r, : mk.shape[0]] = mk
    mask_d = torch.from_numpy(masks).to(dev)
    rows, counts = tk.mask_to_rows(mask_d)
    out = torch.zeros_like(q)
    a_status = torch.zeros(1, dtype=torch.int32, device=dev)
    err = _lib.err_counter(dev)
    stream = torch.cuda.current_stream(dev)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]

    def step(record: bool):
        if record:
            ev[0].record(stream)
        cosine_topk_async(m.emb, m.emb16, m.valid, m.stats, queries, S_K, S_THR, status=s_status,
                          workspace_owner=m, out=s_out)
        if record:
            ev[1].record(stream)
        rc.inject_donors(cache, inj, rope_base=C5_THETA, rotary_style="neox")
        if record:
            ev[2].record(stream)
        for _ in range(C5_L):
            tk.gqa_partial_attention(q, k, v, rows, counts, out, max_rows=s_max, status=a_status)
        if record:
            ev[3].record(stream)

    for _ in range(2):
        step(False)
    torch.cuda.synchronize(dev)
    steps = max(3, min(args.steps // 50, 6))
    parts = np.zeros(3)
    clocks = ClockSampler(local) if rank == 0 else None
    if clocks:
        clocks.start()
    barrier(world)
    torch.cuda.synchronize(dev)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(steps):
        step(True)
        torch.cuda.synchronize(dev)
        parts += [ev[0].elapsed_time(ev[1]), ev[1].elapsed_time(ev[2]), ev[2].elapsed_time(ev[3])]
    t1.record(stream)
    torch.cuda.synchronize(dev)
    barrier(world)
    clk = clocks.stop() if clocks else None
    step_ms = max_over_ranks(t0.elapsed_time(t1) / steps, world)
    parts = [max_over_ranks(x / steps, world) for x in parts]
    st_s, st_a, skipped = int(s_status.item()), int(a_status.item()), _lib.skipped_pairs(dev, reset=True)
    # each part's kernels alone, timed by library events on the launch stream (the in-step
    # brackets above also hold host work such as building the inject's 186 descriptors)
    kern = []
    for fn, n_launch in ((lambda: cosine_topk_async(m.emb, m.emb16, m.valid, m.stats, queries, S_K, S_THR,
                                                    status=s_status, workspace_owner=m, out=s_out), 1),
                         (lambda: rc.inject_donors(cache, inj, rope_base=C5_THETA, rotary_style="neox"), 1),
                         (lambda: rc.inject_donors(cache, inj, rope_base=C5_THETA, rotary_style="neox",
                                                   staging="bulk"), 1),
                         (lambda: tk.gqa_partial_attention(q, k, v, rows, counts, out, max_rows=s_max,
                                                           status=a_status), C5_L)):
        with _lib.KernelTimer(steps * n_launch) as kt:
            for _ in range(steps * n_launch):
                fn()
            torch.cuda.synchronize(dev)
        kern.append(max_over_ranks(kt.total_ms / steps, world))
    kern = [kern[0], kern[1], kern[3], kern[2]]  # screen, inject (direct), attention, inject (bulk-staged)

    # end to end: this step's pair lists, block tables, queries and masks from pinned host
    # memory; search ids and the skipped-pair count back to the host
    hq_host = queries.cpu().pin_memory()
    hmask = torch.from_numpy(masks).pin_memory()
    hres = torch.empty(n_req, S_K, dtype=torch.int64).pin_memory()
    hskip = torch.empty(1, dtype=torch.int64).pin_memory()
    h2d = (sum(h.numel() * h.element_size() for h in host_pos) + sum(h.numel() * 4 for h in host_bt)
           + hq_host.numel() * 4 + hmask.numel())

    def e2e_step():
        queries.copy_(hq_host, non_blocking=True)
        for h, d_ in zip(host_pos, dev_pos):
            d_.copy_(h, non_blocking=True)
        for h, d_ in zip(host_bt, dev_bt):
            d_.copy_(h, non_blocking=True)
        mask_d.copy_(hmask, non_blocking=True)
        r_, c_ = tk.mask_to_rows(mask_d)
        cosine_topk_async(m.emb, m.emb16, m.valid, m.stats, queries, S_K, S_THR, status=s_status,
                          workspace_owner=m, out=s_out)
        rc.inject_donors(cache, inj, rope_base=C5_THETA, rotary_style="neox")
        for _ in range(C5_L):
            tk.gqa_partial_attention(q, k, v, r_, c_, out, max_rows=s_max, status=a_status)
        hres.copy_(s_out[0], non_blocking=True)
        hskip.copy_(err, non_blocking=True)

    e2e_step()
    torch.cuda.synchronize(dev)
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / steps, world)

    inj_bytes = algorithmic_bytes(n_pairs, C5_L, hkv, C5_D, 2, int(nblk.sum()))
    attn_flops = C5_L * attention_flops(masks, hq, C5_D)
    search_flops = 2.0 * C5_SEARCH_ROWS * n_req * S_DIM
    cpu, chk = (None, None)
    if rank == 0:
        cpu, chk = c5_cpu_and_check(m, queries, plan, pool, tables, nblk, cache, q, k, v, out, masks, hq, hkv,
                                    dev, inj_bytes, attn_flops)
    del cache, pool, q, k, v, out
    torch.cuda.empty_cache()
    if rank != 0:
        return None
    pk = peaks()
    tokens = int(req_len.sum())
    att_tf = attn_flops / (kern[2] * 1e-3) / 1e12
    return {
        "component": "c5_step",
        "matches_oracle": chk["matches_oracle"] and st_s == 0 and st_a == 0 and skipped == 0,
        "oracle_check": chk,
        "cpu_baseline": cpu,
        "metric": "c5 reuse step ms (search + inject + 80-layer partial attention), one TP-8 rank",
        "value": round(step_ms, 3),
        "unit": "ms",
        "higher_is_better": False,
        "n_gpus": world,
        "scaling": "weak (each rank one of the 8 TP ranks' KV heads; 8 GPUs run the whole TP-8 step)",
        "steps": steps,
        "config": {"workload": f"c5{'' if (n_req, n_pool) == (C5_REQ, C5_POOL) else ' (reduced)'}: Llama-3-70B geometry (80 L, 64 q / 8 KV heads, D 128, theta 5e5, bf16), "
                               f"TP 8 -> {hq} q heads / {hkv} KV head per rank; {n_req} requests, lognormal "
                               f"lengths (median 8K, 4K-32K; {tokens:,} tokens), 2-4 donors each from a pool of "
                               f"{n_pool} at 256-token chunks, 10-20% recompute (last chunk always); search "
                               f"{C5_SEARCH_ROWS:,} x 384, 64 queries, top-8",
                   "pairs": n_pairs, "descriptors": len(inj), "compute_rows": int(masks.sum()),
                   "attention_operands": "one layer's dense Q/K/V reused by the 80 layer launches",
                   "status": {"search": st_s, "attention": st_a, "skipped_pairs": skipped}},
        "components_ms": {"search": round(parts[0], 4), "inject": round(parts[1], 4),
                          "attention_80_layers": round(parts[2], 3),
                          "note": "in-step event brackets around each part's API calls (host work included)"},
        "kernel_ms": {"screen": round(kern[0], 4), "inject": round(kern[1], 4), "attention_80_layers": round(kern[2], 3),
                      "inject_bulk_staged": round(kern[3], 4),
                      "note": "each part's dominant kernels alone, library events on the launch stream"},
        "roofline": {
            "search": {"bound": "tensor", "achieved": round(search_flops / (kern[0] * 1e-3) / 1e12, 1),
                       "unit": "TFLOP/s", "frac": round(search_flops / (kern[0] * 1e-3) / 1e12 / pk["bf16_tflops"], 4),
                       "note": "64 queries: one query tile, latency-bound"},
            "inject": {"bound": "hbm", "achieved": round(inj_bytes / (kern[1] * 1e-3) / 1e9, 1), "unit": "GB/s",
                       "peak": pk["hbm_gbs"], "frac": round(inj_bytes / (kern[1] * 1e-3) / 1e9 / pk["hbm_gbs"], 4),
                       "algorithmic_bytes": inj_bytes},
            "attention": {"bound": "tensor", "achieved": round(att_tf, 1), "unit": "TFLOP/s",
                          "peak": pk["bf16_tflops_sustained"], "frac": round(att_tf / pk["bf16_tflops_sustained"], 4),
                          "frac_of_burst": round(att_tf / pk["bf16_tflops"], 4), "flops": attn_flops,
                          "note": "80 launches inside a ~0.2 s step: measured against the sustained bf16 peak"},
            "peak_source": pk["source"]},
        "e2e": {"value": round(e2e_ms, 3), "unit": "ms", "h2d_bytes_per_step": int(h2d),
                "d2h_bytes_per_step": n_req * S_K * 8 + 8},
        "gpu_launches": steps * (3 + 1 + C5_L),
        "clocks": clk,
    }


# ---------------------------------------------------------------------------
# Component: masked QKV projection (the projection step of partial prefill, c4 geometry)
# ---------------------------------------------------------------------------
P_HIDDEN = A_HQ * A_D  # 3584: Qwen2-7B's hidden size (28 heads x 128)


def run_projection(args, local: int) -> dict:
    """masked_qkv_projection over c4's batch: per sequence hidden [32768, 3584]
    bf16 times W [3 * 3584, 3584] plus bias at the ~10 % compute rows (the
    reference's shapes: one weight row per q/k/v feature), reuse rows zero."""
    from semblend_b200 import _lib
    from semblend_b200 import triton_kernels as tk

    dev = torch.device("cuda", local)
    B, S, hid, nout = args.attn_batch, args.attn_seq, P_HIDDEN, 3 * P_HIDDEN
    rng = np.random.default_rng(SEED + 5)
    masks = np.stack([make_attention_mask(rng, S) for _ in range(B)])  # the attention component's rows
    g = torch.Generator(device=dev).manual_seed(SEED + 13)
    x = [torch.randn(S, hid, generator=g, device=dev).to(torch.bfloat16) for _ in range(B)]
    w = (torch.randn(nout, hid, generator=g, device=dev) / np.sqrt(hid)).to(torch.bfloat16)
    bias = (0.1 * torch.randn(nout, generator=g, device=dev)).to(torch.bfloat16)
    mk = [torch.from_numpy(m).to(dev) for m in masks]
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    rows = masks.sum(axis=1)
    flops = 2.0 * float(rows.sum()) * hid * nout

    def step(ms_):
        return [tk.masked_qkv_projection(x[b], w, ms_[b], bias, status=status) for b in range(B)]

    for _ in range(max(args.warmup, 3)):
        out = step(mk)
    torch.cuda.synchronize(dev)
    # parity spot check: 64 compute rows and 64 reuse rows of sequence 0 against fp32
    r_c = np.nonzero(masks[0])[0][:: max(1, rows[0] // 64)][:64]
    r_r = np.nonzero(~masks[0])[0][:64]
    ref = x[0][r_c].float() @ w.float().T + bias.float()
    err = float((out[0][r_c].float() - ref).abs().max().item())
    zero_ok = bool((out[0][r_r] == 0).all().item())
    steps = max(5, min(args.steps // 10, 30))
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with _lib.KernelTimer(steps * B) as kt:
        e0.record(stream)
        for _ in range(steps):
            step(mk)
        e1.record(stream)
        torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / steps
    kms = kt.mean_ms * B  # the GEMM launches of one step

    # end to end: each step's compute masks copied from pinned host memory, the status read back
    hm = [torch.from_numpy(m).pin_memory() for m in masks]
    hs = torch.zeros(1, dtype=torch.int32).pin_memory()
    torch.cuda.synchronize(dev)
    c0 = time.perf_counter()
    for _ in range(steps):
        dm = [h.to(dev, non_blocking=True) for h in hm]
        step(dm)
        hs.copy_(status, non_blocking=True)
        torch.cuda.synchronize(dev)
    e2e_ms = (time.perf_counter() - c0) * 1e3 / steps

    # the reference's CPU algorithm (every row multiplied, reuse rows zeroed afterwards,
    # triton_kernels.py:451-522), on a 256-row sample in fp32, scaled to all S rows
    torch.set_num_threads(os.cpu_count() or 1)
    xs = x[0][:256].float().cpu()
    wc, bc = w.float().cpu(), bias.float().cpu()
    c0 = time.perf_counter()
    n_rep = 0
    while time.perf_counter() - c0 < 3.0:
        torch.addmm(bc, xs, wc.T)
        n_rep += 1
    cpu_row_s = (time.perf_counter() - c0) / (n_rep * 256)
    cpu_step_s = cpu_row_s * S * B
    pk = peaks()
    ach = flops / (kms * 1e-3) / 1e12
    return {
        "component": "projection",
        "matches_oracle": bool(zero_ok and err <= 2e-2 * max(1.0, float(ref.abs().max())) and int(status.item()) == 0),
        "metric": "masked QKV projection TFLOP/s", "value": round(flops / (ms * 1e-3) / 1e12, 1), "unit": "TFLOP/s",
        "higher_is_better": True, "ms_per_step": round(ms, 4), "steps": steps, "dtype": "bf16",
        "config": {"workload": f"c4 projection: {B} sequences x {S} tokens, hidden {hid} -> {nout} (q, k, v rows of "
                               f"W), bias, bf16, the attention component's compute rows ({int(rows.sum())} of "
                               f"{B * S}); TFLOP/s by 2 x compute rows x {hid} x {nout}",
                   "max_abs_err_vs_fp32": err, "reuse_rows_zero": zero_ok, "status": int(status.item()),
                   "step_includes": "zero-filled output, mask to rows, row gather, GEMM + bias + scatter"},
        "roofline": {"bound": "tensor", "kernel": "gemm_rows_kernel<bf16> (tcgen05, 128 x 256 tiles)",
                     "achieved": round(ach, 1), "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": round(ach / pk["bf16_tflops"], 4), "kernel_ms": round(kms, 4), "traffic": None,
                     "peak_source": pk["source"]},
        "cpu_baseline": {"value": round(flops / cpu_step_s / 1e12, 5), "unit": "TFLOP/s",
                         "cores": torch.get_num_threads(), "kind": "port",
                         "sample": f"torch.addmm over a 256-row fp32 sample ({n_rep} repeats, 3 s), scaled to all "
                                   f"{B * S} rows as the reference multiplies every row; TFLOP/s by compute-row "
                                   "flops"},
        "e2e": {"value": round(flops / (e2e_ms * 1e-3) / 1e12, 1), "unit": "TFLOP/s",
                "h2d_bytes_per_step": int(sum(h.numel() for h in hm)), "d2h_bytes_per_step": 4},
        "gpu_launches": steps * B * 3,
    }


# ---------------------------------------------------------------------------
# Chunk-hash alignment (the step before the inject: which donor chunk feeds which target chunk)
# ---------------------------------------------------------------------------
AL_VOCAB = 128256  # Llama-3 vocabulary: token ids are int64 in [0, AL_VOCAB)


def alignment_inputs(rng: np.random.Generator):
    """c2 geometry: 8 requests, a 16384-token donor and a 16384-token target
    each; 85 % of the target's 256-token chunks are donor chunks in shuffled
    order, the rest fresh tokens (recompute)."""
    n_chunks = SEQ // CHUNK
    donors, targets = [], []
    for _ in range(N_REQ):
        d = rng.integers(0, AL_VOCAB, SEQ)
        src = rng.permutation(n_chunks)
        fresh = rng.random(n_chunks) < RECOMPUTE_FRAC
        t = np.concatenate([rng.integers(0, AL_VOCAB, CHUNK) if fresh[i] else d[src[i] * CHUNK : (src[i] + 1) * CHUNK]
                            for i in range(n_chunks)])
        donors.append(d)
        targets.append(t)
    return np.stack(donors), np.stack(targets)


def run_alignment(args, local: int) -> dict:
    """Chunk-hash alignment of the c2 requests on the device (SHA-256 of every
    256-token chunk, greedy matching with the context gate, position pairs for
    the inject), against the reference's CPU algorithm (the oracle port)."""
    from oracle import alignment as oal
    from semblend_b200 import _lib
    from semblend_b200.alignment import chunk_alignment, chunk_alignment_batch

    dev = torch.device("cuda", local)
    rng = np.random.default_rng(SEED + 11)
    donors, targets = alignment_inputs(rng)
    hd = torch.from_numpy(donors).pin_memory()
    ht = torch.from_numpy(targets).pin_memory()
    dd, dt = hd.to(dev), ht.to(dev)
    stream = torch.cuda.current_stream(dev)

    def step(d, t):  # every request of the step in one batch: 1 hashing + 2 matching launches
        return chunk_alignment_batch(list(d), list(t), CHUNK, context_gate=True, device=dev)

    def step_each(d, t):  # one chunk_alignment call per request
        return [chunk_alignment(d[r], t[r], CHUNK, context_gate=True, device=dev) for r in range(N_REQ)]

    for _ in range(max(args.warmup, 3)):
        res = step(dd, dt)
        res_each = step_each(dd, dt)
    torch.cuda.synchronize(dev)
    got = [int(a.n_pairs.item()) for a in res]
    same = got == [int(a.n_pairs.item()) for a in res_each] and all(
        torch.equal(a.match, b.match) for a, b in zip(res, res_each))
    steps = max(10, min(args.steps, 200))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with _lib.KernelTimer(steps) as kt:
        e0.record(stream)
        for _ in range(steps):
            step(dd, dt)
        e1.record(stream)
        torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / steps
    e0.record(stream)
    for _ in range(steps):
        step_each(dd, dt)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    each_ms = e0.elapsed_time(e1) / steps

    # end to end: token ids from pinned host memory, the pair counts back (the pairs stay on the device)
    hn = torch.empty(N_REQ, dtype=torch.int64).pin_memory()
    bd, bt = torch.empty_like(dd), torch.empty_like(dt)
    torch.cuda.synchronize(dev)
    c0 = time.perf_counter()
    e0.record(stream)
    for _ in range(steps):
        bd.copy_(hd, non_blocking=True)
        bt.copy_(ht, non_blocking=True)
        r = step(bd, bt)
        hn.copy_(torch.cat([a.n_pairs for a in r]), non_blocking=True)
        torch.cuda.synchronize(dev)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = (time.perf_counter() - c0) * 1e3 / steps

    # the reference's CPU algorithm (oracle port: hashlib SHA-256 + greedy matching), bounded sample
    want = [int((oal.chunk_matches(donors[r].tolist(), targets[r].tolist(), CHUNK, True) >= 0).sum()) * CHUNK
            for r in range(2)]
    ok = got[:2] == want and hn.tolist() == got and same
    cpu_s, n_cpu = 0.0, 0
    while cpu_s < 3.0:
        r = n_cpu % N_REQ
        c0 = time.perf_counter()
        oal.chunk_matches(donors[r].tolist(), targets[r].tolist(), CHUNK, True)
        cpu_s += time.perf_counter() - c0
        n_cpu += 1
    tok = N_REQ * SEQ
    pk = peaks()
    sha_bytes = N_REQ * 2 * (SEQ * 8 + (SEQ // CHUNK) * 16)  # donors + targets: int64 ids read, digests written
    sha_ms = kt.mean_ms
    ach = sha_bytes / (sha_ms * 1e-3) / 1e9
    return {
        "component": "alignment",
        "matches_oracle": bool(ok),
        "metric": "chunk alignment tokens/s", "value": round(tok / (ms * 1e-3), 1), "unit": "tokens/s",
        "higher_is_better": True, "ms_per_step": round(ms, 4), "steps": steps, "dtype": "int64",
        "config": {"workload": f"c2 alignment: {N_REQ} targets x {SEQ} tokens against one {SEQ}-token donor each, "
                               f"256-token chunks, {int(round((1 - RECOMPUTE_FRAC) * 100))}% donor chunks shuffled, "
                               "context gate on; the step's requests in one chunk_alignment_batch call (digests "
                               "of donors and targets, matching, pair arrays on the device)",
                   "pairs_per_step": int(sum(got)), "matches_oracle": ok, "seed": SEED + 11,
                   "one_call_per_request_ms": round(each_ms, 4)},
        "roofline": {"bound": "hbm", "kernel": "chunk_sha256_kernel<int64_t>", "achieved": round(ach, 2),
                     "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": round(ach / pk["hbm_gbs"], 6),
                     "kernel_ms": round(sha_ms, 5), "traffic": None, "peak_source": pk["source"],
                     "note": "latency-bound: one thread per 256-token chunk (1,024 per launch), 17 dependent "
                             "SHA-256 compressions each"},
        "cpu_baseline": {"value": round(n_cpu * SEQ / cpu_s, 1), "unit": "tokens/s", "cores": 1, "kind": "port",
                         "sample": f"{n_cpu} requests through oracle.alignment.chunk_matches (hashlib SHA-256 + "
                                   f"greedy matching + gate), {cpu_s:.1f} s of CPU work"},
        "e2e": {"value": round(tok / (e2e_ms * 1e-3), 1), "unit": "tokens/s",
                "h2d_bytes_per_step": int(hd.numel() * 8 + ht.numel() * 8), "d2h_bytes_per_step": N_REQ * 8},
        "gpu_launches": steps * 3,
    }


# ---------------------------------------------------------------------------
# CPU baseline (oracle port of the reference's inject) — bounded sample
# ---------------------------------------------------------------------------
def inject_config(n_req: int, n_layers: int, world: int, n_pairs: int | None) -> dict:
    """The c2 workload description shared by both arms' JSON lines."""
    return {
        "workload": f"c2{'' if (n_req, n_layers) == (N_REQ, N_LAYERS) else ' (reduced)'}: {n_req} req x 16384 "
                    f"tok donors, {n_layers} L x 4 KV heads x 128, bf16, 85% reuse via 256-tok "
                    "chunks (delta U[-4096,4096]), 15% recompute untouched, block 16, neox RoPE theta 1e6",
        "pairs_per_step": n_pairs,
        "parallelism": (f"tp{world}: the step's (layer, KV head) units split over {world} rank(s) "
                        "(heads first: N | 4 -> 4/N heads x all layers, N = 8 -> 1 head x 14 layers); "
                        "strong scaling, no collective"),
        "l2": "inputs larger than L2 (7.3 GB donors + 9.2 GB cache for the whole step)",
        "seed": SEED,
    }


class CpuInjectSlices:
    """The reference's CPU inject (oracle port of rope_correction.py:285-328)
    over (request, layer) slices of c2, on the host cores (all threads).

    Every request has its own 1024-entry block table (a seeded shuffle of its
    own 1024 cache blocks), so every pair of every slice lands in range; each
    call reports how many pairs it applied and bytes are counted for those
    only, after checking that all of the slice's pairs were applied."""

    def __init__(self, seed: int = SEED):
        torch.set_num_threads(os.cpu_count() or 1)
        rng = np.random.default_rng(seed)
        self.plans = [make_request_plan(rng)[:2] for _ in range(N_REQ)]
        per = SEQ // BLOCK
        self.tables = [torch.from_numpy(rng.permutation(per).astype(np.int32)) for _ in range(N_REQ)]
        g = torch.Generator().manual_seed(seed)
        self.donor = torch.randn(2, N_KV_HEADS, SEQ, HEAD_DIM, generator=g).to(torch.bfloat16)
        self.caches = [torch.randn(per, 2, N_KV_HEADS, BLOCK, HEAD_DIM, generator=g).to(torch.bfloat16)
                       for _ in range(N_REQ)]
        self.pos = [(torch.from_numpy(d), torch.from_numpy(t)) for d, t in self.plans]
        self.n = 0

    def run(self) -> tuple[float, int]:
        """One slice (the next request round robin): (seconds, bytes)."""
        from oracle import rope as orope

        r = self.n % N_REQ
        self.n += 1
        d, t = self.pos[r]
        c0 = time.perf_counter()
        _, applied = orope.rope_correct_scatter_paged(self.caches[r], self.donor, self.tables[r], d, t,
                                                      ROPE_THETA, "neox", return_applied=True, inplace=True)
        sec = time.perf_counter() - c0
        if applied != d.shape[0]:
            raise RuntimeError(f"CPU inject applied {applied} of {d.shape[0]} pairs")
        return sec, algorithmic_bytes(applied, 1, N_KV_HEADS, HEAD_DIM, 2, SEQ // BLOCK)

    @staticmethod
    def describe(n: int, sec: float) -> str:
        return (f"{n} (request, layer) slices of c2 (~13.9K pairs x 4 KV heads x 128 bf16 each, every pair "
                f"applied, each request its own block table) through oracle.rope.rope_correct_scatter_paged "
                f"in place, {sec:.1f} s of CPU work; GB/s by algorithmic bytes")


def cpu_baseline(budget_s: float = 8.0) -> dict:
    """The CPU inject on slices of c2 until `budget_s` seconds of CPU work."""
    cs = CpuInjectSlices()
    cs.run()  # warm-up
    nbytes, sec, n = 0, 0.0, 0
    while sec < budget_s and n < N_REQ * N_LAYERS:
        s, b = cs.run()
        sec += s
        nbytes += b
        n += 1
    return {"value": round(nbytes / sec / 1e9, 4), "unit": "GB/s", "cores": torch.get_num_threads(),
            "kind": "port", "sample": CpuInjectSlices.describe(n, sec), "seconds": round(sec, 3)}


def run_reference(args, world, rank) -> dict | None:
    """The reference arm: W warm-up then K timed steps, each step one
    (request, layer) slice of c2 through the reference's CPU inject (oracle
    port) on all host threads; rank 0 only."""
    if rank != 0:
        return None
    rng = np.random.default_rng(SEED)
    ref_pairs = sum(make_request_plan(rng)[0].shape[0] for _ in range(N_REQ))
    cs = CpuInjectSlices()
    for _ in range(args.warmup):
        cs.run()
    nbytes, sec = 0, 0.0
    for _ in range(args.steps):
        s, b = cs.run()
        sec += s
        nbytes += b
    value = round(nbytes / sec / 1e9, 4)
    cb = {"value": value, "unit": "GB/s", "cores": torch.get_num_threads(), "kind": "port",
          "sample": CpuInjectSlices.describe(args.steps, sec), "seconds": round(sec, 3)}
    return {
        "impl": "reference",
        "metric": "RoPE-corrected KV inject GB/s",
        "value": value,
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(sec / args.steps * 1e3, 3),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded)",
        "config": inject_config(N_REQ, N_LAYERS, world, ref_pairs),
        "cpu_baseline": cb,
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def summarize(comp: dict) -> dict:
    """The few numbers of a component line that must survive a truncated log."""
    rl = comp.get("roofline") or {}
    if "frac" not in rl:  # c5: one roofline per part
        frac = {k: v.get("frac") for k, v in rl.items() if isinstance(v, dict)}
    else:
        frac = rl.get("frac")
    e2e = comp.get("e2e") or {}
    cpu = comp.get("cpu_baseline") or {}
    out = {"value": comp.get("value"), "unit": comp.get("unit"), "frac": frac, "e2e": e2e.get("value"),
           "cpu": cpu.get("value"), "ok": comp.get("matches_oracle")}
    if comp.get("n_gpus", 1) > 1:
        out["n_gpus"] = comp["n_gpus"]
    return out


def emit_component(comp: dict | None, summary: dict, name: str) -> None:
    """Full component line on stderr (one JSON object per line), condensed copy
    in the headline's summary."""
    if comp is None:
        return
    print(json.dumps(comp), file=sys.stderr, flush=True)
    summary[name] = summarize(comp)


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-components", action="store_true", help="only the c2 headline")
    ap.add_argument("--only", choices=["all", "c1", "search", "attention", "c5", "alignment", "projection"],
                    default="all", help="print only that component's line (on stdout)")
    ap.add_argument("--attn-batch", type=int, default=A_B, help="attention batch (c4: 4)")
    ap.add_argument("--attn-seq", type=int, default=A_S, help="attention context (c4: 32768)")
    ap.add_argument("--search-rows", type=int, default=S_ROWS, help="donor rows of the search (c3: 1048576)")
    ap.add_argument("--requests", type=int, default=N_REQ, help="requests per step (c2: 8)")
    ap.add_argument("--layers", type=int, default=N_LAYERS, help="layers (c2: 28)")
    ap.add_argument("--c5-requests", type=int, default=C5_REQ, help="c5 requests (64)")
    ap.add_argument("--c5-pool", type=int, default=C5_POOL, help="c5 donor pool (64)")
    ap.add_argument("--check-slices", type=int, default=3, help="(request, layer) slices of c2 checked per rank")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        line = run_reference(args, world, rank)
        if line is not None:
            print(json.dumps(line), flush=True)
        return 0
    world, rank, local = dist_setup(args.gpus)
    failed = []
    if args.only != "all":
        if args.only == "search" and world > 1:
            res = run_search_sharded(args, world, rank, local)
        elif args.only == "attention" and world > 1:
            res = run_attention_sharded(args, world, rank, local)
        elif args.only == "c5":
            res = run_c5(args, world, rank, local)
        elif rank != 0:
            res = None
        else:
            res = {"c1": run_c1, "search": run_search, "attention": run_attention, "alignment": run_alignment,
                   "projection": run_projection}[args.only](args, local)
        if res is not None:
            print(json.dumps(res), flush=True)
            if res.get("matches_oracle") is False:
                failed.append(args.only)
    else:
        line = run_ours(args, world, rank, local)
        summary: dict = {}
        if line is not None and world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline()
        if not args.no_components:
            if world == 1:
                for name, fn in (("c1", run_c1), ("c3_search", run_search), ("c4_attention", run_attention),
                                 ("projection", run_projection), ("alignment", run_alignment)):
                    emit_component(fn(args, local), summary, name)
            emit_component(run_c5(args, world, rank, local), summary, "c5_step")
            if world > 1:
                emit_component(run_search_sharded(args, world, rank, local), summary, "c3_search_sharded")
                emit_component(run_attention_sharded(args, world, rank, local), summary, "c4_attention_sharded")
        if line is not None:
            failed += [k for k, v in summary.items() if v.get("ok") is False]
            if not line["matches_oracle"]:
                failed.append("c2_inject")
            if summary:
                line["components_summary"] = summary
            print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()
    if failed:
        print(f"bench: parity check failed for {', '.join(failed)}", file=sys.stderr, flush=True)
        return 1
    return 0


if __name__ == "__main__":
    sys.exit(main())
