"""Chunk-hash alignment on the GPU against the reference's goldens and the CPU
oracle: SHA-256 digests bit-exact, chunk matches and position pairs exact."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import alignment as oal
from oracle import rope as orope
from semblend_b200 import alignment as al
from semblend_b200 import rope_correction as rc
from tests.helpers import assert_rope_close, load_golden

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _digests_u32(d: torch.Tensor) -> np.ndarray:
    return d.cpu().numpy().view(np.uint32)


def _expected_pairs(match: np.ndarray, chunk: int):
    dp, tp = [], []
    for t, d in enumerate(match.tolist()):
        if d >= 0:
            dp += range(d * chunk, (d + 1) * chunk)
            tp += range(t * chunk, (t + 1) * chunk)
    return np.array(dp, np.int32), np.array(tp, np.int32)


@pytest.mark.parametrize("name", ["align_gate", "align_nogate", "align_small"])
def test_alignment_matches_reference_golden(name):
    g = load_golden(name)
    chunk, gate = int(g["chunk"]), bool(g["gate"])
    donor, target = g["donor"].to(DEV), g["target"].to(DEV)
    assert np.array_equal(_digests_u32(al.chunk_digests(donor, chunk)), g["donor_digests"].numpy())
    assert np.array_equal(_digests_u32(al.chunk_digests(target, chunk)), g["target_digests"].numpy())
    a = al.chunk_alignment(donor, target, chunk, context_gate=gate)
    assert np.array_equal(a.match.cpu().numpy(), g["match"].numpy().astype(np.int32))
    dp, tp = a.pairs()
    want_d, want_t = _expected_pairs(g["match"].numpy(), chunk)
    assert np.array_equal(dp.cpu().numpy(), want_d) and np.array_equal(tp.cpu().numpy(), want_t)
    res = al.compute_chunk_alignment(g["donor"].tolist(), g["target"].tolist(), chunk, gate)
    assert res.reuse_ratio == pytest.approx(float(g["reuse_ratio"]), abs=0)
    assert res.exact_chunks == int(g["exact_chunks"])
    assert len(res.slot_actions) == g["target"].shape[0]
    assert al.estimate_chunk_reuse(donor, target, chunk) == pytest.approx(float(g["estimate"]), abs=0)


@pytest.mark.parametrize("chunk", [1, 7, 13, 14, 15, 16, 100, 256])
@pytest.mark.parametrize("dtype", [torch.int32, torch.int64])
def test_digests_all_tail_lengths_vs_hashlib(chunk, dtype):
    """Chunks whose byte length leaves every possible tail in the last SHA-256 block."""
    rng = np.random.default_rng(chunk)
    toks = rng.integers(0, 2**31 - 1, chunk * 9 + 3)
    got = _digests_u32(al.chunk_digests(torch.from_numpy(toks).to(dtype).to(DEV), chunk))
    assert np.array_equal(got, oal.digests(toks.tolist(), chunk))


@pytest.mark.parametrize("gate", [False, True])
@pytest.mark.parametrize("chunk", [16, 64, 256])
def test_alignment_vs_oracle_with_repeats(gate, chunk):
    rng = np.random.default_rng(chunk + gate)
    base = [rng.integers(0, 1000, chunk) for _ in range(12)]  # few distinct chunks: many repeats
    donor = np.concatenate([base[i] for i in rng.integers(0, 12, 40)])
    target = np.concatenate([base[i] for i in rng.integers(0, 14, 50) if i < 12] +
                            [rng.integers(0, 1000, chunk - 1)])
    a = al.chunk_alignment(torch.from_numpy(donor).to(DEV), torch.from_numpy(target).to(DEV), chunk, gate)
    want = oal.chunk_matches(donor.tolist(), target.tolist(), chunk, gate)
    assert np.array_equal(a.match.cpu().numpy(), want.astype(np.int32))
    dp, tp = a.pairs()
    wd, wt = _expected_pairs(want, chunk)
    assert np.array_equal(dp.cpu().numpy(), wd) and np.array_equal(tp.cpu().numpy(), wt)
    n = int(a.n_pairs.item())
    assert (a.donor_positions[n:] == -1).all() and (a.target_positions[n:] == -1).all()


def test_alignment_many_chunks():
    """Thousands of chunks: matched chunks out of order, repeats and unmatched
    chunks spread over every pair-writing CTA."""
    rng = np.random.default_rng(11)
    chunk, nd = 16, 3000
    donor = rng.integers(0, 1 << 30, chunk * nd)
    donor[chunk * 100 : chunk * 110] = np.tile(donor[: chunk], 10)  # ten copies of chunk 0
    picks = np.concatenate([rng.permutation(nd)[:2500], np.zeros(12, np.int64)])
    rng.shuffle(picks)
    parts = [donor[i * chunk : (i + 1) * chunk] for i in picks]
    for j in rng.choice(len(parts), 400, replace=False):  # unmatched chunks
        parts[j] = rng.integers(0, 1 << 30, chunk)
    target = np.concatenate(parts + [rng.integers(0, 1 << 30, 7)])
    for gate in (False, True):
        a = al.chunk_alignment(torch.from_numpy(donor).to(DEV), torch.from_numpy(target).to(DEV), chunk, gate)
        want = oal.chunk_matches(donor.tolist(), target.tolist(), chunk, gate)
        assert np.array_equal(a.match.cpu().numpy(), want.astype(np.int32))
        wd, wt = _expected_pairs(want, chunk)
        n = int(a.n_pairs.item())
        assert n == wd.shape[0]
        assert np.array_equal(a.donor_positions[:n].cpu().numpy(), wd)
        assert np.array_equal(a.target_positions[:n].cpu().numpy(), wt)
        assert (a.donor_positions[n:] == -1).all() and (a.target_positions[n:] == -1).all()


@pytest.mark.parametrize("gate", [False, True])
def test_alignment_batch_vs_oracle(gate):
    """Pairs of mixed sizes in one batch: each result equals the oracle's and
    the single-pair call's (empty donor, target shorter than a chunk, partial
    chunks, repeats, int32 beside int64 ids)."""
    rng = np.random.default_rng(21 + gate)
    chunk = 32
    base = [rng.integers(0, 5000, chunk) for _ in range(10)]

    def seq(n_chunks, tail):
        s = [base[i] for i in rng.integers(0, 12, n_chunks) if i < 10]
        s.append(rng.integers(0, 5000, tail))
        return np.concatenate(s)

    donors = [seq(40, 5), np.zeros(0, np.int64), seq(3, 0), seq(70, 31), seq(1, 0), seq(25, 3)]
    targets = [seq(50, 7), seq(6, 0), rng.integers(0, 5000, 20), seq(90, 0), seq(2, 1), seq(30, 16)]
    dt = [torch.from_numpy(d).to(DEV) for d in donors]
    tt = [torch.from_numpy(t).to(DEV) for t in targets]
    tt[5] = tt[5].to(torch.int32)
    res = al.chunk_alignment_batch(dt, tt, chunk, gate)
    assert len(res) == len(targets)
    for r, a in enumerate(res):
        want = oal.chunk_matches(donors[r].tolist(), targets[r].tolist(), chunk, gate)
        assert np.array_equal(a.match.cpu().numpy(), want.astype(np.int32)), r
        wd, wt = _expected_pairs(want, chunk)
        dp, tp = a.pairs()
        assert np.array_equal(dp.cpu().numpy(), wd) and np.array_equal(tp.cpu().numpy(), wt), r
        n = int(a.n_pairs.item())
        assert (a.donor_positions[n:] == -1).all() and (a.target_positions[n:] == -1).all()
        one = al.chunk_alignment(dt[r], tt[r], chunk, gate)
        assert torch.equal(one.match, a.match) and int(one.n_pairs.item()) == n
    assert al.chunk_alignment_batch([], [], chunk) == []


@pytest.mark.parametrize("name", ["align_gate", "align_nogate", "align_small", "reuse_fallback", "reuse_short"])
def test_estimate_reuse_ratio_matches_reference_golden(name):
    g = load_golden(name)
    chunk = int(g["chunk"])
    got = al.estimate_reuse_ratio(g["donor"].to(DEV), g["target"].to(DEV), chunk)
    assert got == float(g["estimate"])


def test_token_overlap_vs_oracle():
    """Repeated ids, int32 beside int64, the id -1 (the table's empty marker),
    large ids and empty sides."""
    rng = np.random.default_rng(5)
    for n_d, n_t, vocab in ((5000, 3000, 50), (20000, 20000, 1 << 40), (1, 1000, 3), (0, 10, 5), (10, 0, 5)):
        d = rng.integers(-1, vocab, n_d)
        t = rng.integers(-1, vocab, n_t)
        want = oal.token_overlap(d.tolist(), t.tolist())
        got = int(al.token_overlap(torch.from_numpy(d).to(DEV), torch.from_numpy(t).to(DEV)).item())
        assert got == want, (n_d, n_t, vocab)
    d = rng.integers(-1, 40, 3000)
    t = rng.integers(-1, 40, 2000)
    got = int(al.token_overlap(torch.from_numpy(d).to(DEV, torch.int32), torch.from_numpy(t).to(DEV)).item())
    assert got == oal.token_overlap(d.tolist(), t.tolist())


def test_alignment_edge_cases():
    t = torch.arange(300, dtype=torch.int64, device=DEV)
    a = al.chunk_alignment(torch.empty(0, dtype=torch.int64, device=DEV), t, 256, True)  # empty donor
    assert a.match.tolist() == [-1, -1] and int(a.n_pairs.item()) == 0
    a = al.chunk_alignment(t, t[:100], 256, False)  # target shorter than a chunk
    assert a.match.tolist() == [-1] and int(a.n_pairs.item()) == 0
    a = al.chunk_alignment(t, t, 256, True)  # a single matched chunk has no neighbour: gated out
    assert a.match.tolist() == [-1, -1]
    a = al.chunk_alignment(t, t, 256, False)
    assert a.match.tolist() == [0, -1] and int(a.n_pairs.item()) == 256


def test_alignment_pairs_drive_the_inject_without_the_host():
    """Device alignment -> inject of the matched chunks, against the oracle."""
    rng = np.random.default_rng(7)
    chunk, H, D, bs = 64, 2, 128, 16
    donor_t = rng.integers(0, 50000, chunk * 10)
    order = [3, 4, 5, 9, 0, 1]
    target_t = np.concatenate([donor_t[i * chunk : (i + 1) * chunk] for i in order] + [rng.integers(0, 50000, 40)])
    a = al.chunk_alignment(torch.from_numpy(donor_t).to(DEV), torch.from_numpy(target_t).to(DEV), chunk, True)
    g = torch.Generator().manual_seed(8)
    donor_kv = torch.randn(2, H, donor_t.shape[0], D, generator=g).to(torch.bfloat16)
    nb = (target_t.shape[0] + bs - 1) // bs + 4
    cache = torch.randn(nb, 2, H, bs, D, generator=g).to(torch.bfloat16)
    bt = torch.randperm(nb, generator=g)[: (target_t.shape[0] + bs - 1) // bs].to(torch.int32)
    dp, tp = a.pairs()
    c = cache.to(DEV)
    rc.rope_correct_scatter_paged(c, donor_kv.to(DEV), bt.to(DEV), dp, tp, rope_base=1e6, rotary_style="neox")
    want_d, want_t = _expected_pairs(oal.chunk_matches(donor_t.tolist(), target_t.tolist(), chunk, True), chunk)
    want = orope.rope_correct_scatter_paged(cache, donor_kv, bt, torch.from_numpy(want_d), torch.from_numpy(want_t),
                                            1e6, "neox")
    got = c.cpu()
    assert torch.equal(got[:, 1], want[:, 1])
    assert_rope_close(got[:, 0].contiguous(), want[:, 0].contiguous(), "neox")
