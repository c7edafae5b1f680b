"""GPU parity of the tensor-core cosine top-k search against the CPU oracle
(the reference's per-query numpy stage) and the DonorStore golden fixture.

Bar: returned rows equal the oracle's except where similarities tie within
1e-6; every similarity within 1e-6 of the oracle's fp32 value.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import search as osearch
from semblend_b200 import donor_store as ds
from semblend_b200.search import DeviceDonorMatrix, merge_topk
from tests.helpers import load_golden

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
TOL = 1e-6


def tol(x):
    """1e-6, relative for similarities above 1 (only unnormalised rows reach them)."""
    return TOL * np.maximum(1.0, np.abs(x))


def exact_scores(E: np.ndarray, q: np.ndarray, ids: np.ndarray) -> np.ndarray:
    qn = osearch.normalize_query(q)
    return np.array([float(E[i] @ qn) if i >= 0 else -np.inf for i in ids], dtype=np.float64)


def assert_topk_equivalent(E, valid, Q, thr, ids_g, s_g, k):
    ids_o, s_o = osearch.topk_batch(E, valid, Q, thr, k)
    for qi in range(Q.shape[0]):
        go, gg = ids_o[qi], ids_g[qi]
        so, sg = s_o[qi].astype(np.float64), s_g[qi].astype(np.float64)
        no, ng = int((go >= 0).sum()), int((gg >= 0).sum())
        if no != ng:
            # only a similarity within TOL of the threshold may flip membership
            extra = so[ng:no] if no > ng else sg[no:ng]
            assert np.all(np.abs(extra - thr) <= tol(thr)), (qi, no, ng, extra)
        n = min(no, ng)
        assert np.all(np.abs(so[:n] - sg[:n]) <= tol(so[:n])), (qi, so[:n], sg[:n])
        assert len(set(gg[:ng].tolist())) == ng, "duplicate ids"
        if ng:
            assert np.all(valid[gg[:ng]]), "invalid row returned"
            ex = exact_scores(E, Q[qi], gg[:ng])
            assert np.all(np.abs(ex - sg[:ng]) <= tol(ex))
        for r in range(n):
            if go[r] != gg[r]:
                assert abs(so[r] - sg[r]) <= tol(so[r]), (qi, r)


def clustered(n, dim, n_centers, seed, sigma=0.3):
    rng = np.random.default_rng(seed)
    centers = rng.standard_normal((n_centers, dim)).astype(np.float32)
    lab = rng.integers(0, n_centers, n)
    E = centers[lab] + sigma * rng.standard_normal((n, dim)).astype(np.float32)
    E /= np.linalg.norm(E, axis=1, keepdims=True)
    return E.astype(np.float32), centers, rng


def queries_for(centers, rng, nq, dim, frac_cluster=0.7, sigma=0.3):
    nc = int(round(frac_cluster * nq))
    lab = rng.integers(0, centers.shape[0], nc)
    Qc = centers[lab] + sigma * rng.standard_normal((nc, dim)).astype(np.float32)
    Qu = rng.standard_normal((nq - nc, dim)).astype(np.float32)
    Q = np.concatenate([Qc, Qu]) * rng.uniform(0.5, 3.0, (nq, 1)).astype(np.float32)  # un-normalised
    return Q.astype(np.float32)


def build(E, valid=None):
    m = DeviceDonorMatrix(E.shape[0], E.shape[1], DEV)
    m.write_range(0, torch.from_numpy(E).to(DEV))
    if valid is not None:
        m.invalidate(np.where(~valid)[0])
    return m


@pytest.mark.parametrize("k", [1, 5, 8, 10, 16, 32])
def test_clustered_vs_oracle(k):
    E, centers, rng = clustered(20000, 384, 64, seed=k)
    Q = queries_for(centers, rng, 300, 384)
    m = build(E)
    ids, s = m.search(Q, k, 0.6)
    valid = np.ones(E.shape[0], bool)
    assert_topk_equivalent(E, valid, Q, 0.6, ids.cpu().numpy(), s.cpu().numpy(), k)


def test_valid_mask_ragged_sizes():
    E, centers, rng = clustered(9999, 384, 16, seed=3)
    valid = rng.random(9999) > 0.3
    Q = queries_for(centers, rng, 129, 384)
    m = build(E, valid)
    ids, s = m.search(Q, 8, 0.5)
    assert_topk_equivalent(E, valid, Q, 0.5, ids.cpu().numpy(), s.cpu().numpy(), 8)


@pytest.mark.parametrize("dim", [64, 100, 128, 512])
def test_other_dims(dim):
    E, centers, rng = clustered(3000, dim, 8, seed=dim)
    Q = queries_for(centers, rng, 50, dim)
    m = build(E)
    ids, s = m.search(Q, 8, 0.4)
    assert_topk_equivalent(E, np.ones(3000, bool), Q, 0.4, ids.cpu().numpy(), s.cpu().numpy(), 8)


def test_single_query_and_no_hits():
    E, centers, rng = clustered(1000, 384, 4, seed=5)
    m = build(E)
    ids, s = m.search(rng.standard_normal(384).astype(np.float32), 5, 0.99)
    assert ids.shape == (1, 5) and torch.all(ids == -1) and torch.all(torch.isinf(s))
    zero = np.zeros((2, 384), np.float32)  # norm 0: q / (0 + 1e-8) = 0, all similarities 0
    ids, s = m.search(zero, 3, 0.6)
    assert torch.all(ids == -1)
    ids, s = m.search(zero, 3, -0.5)
    assert torch.equal(ids.cpu(), torch.tensor([[0, 1, 2], [0, 1, 2]]))


def test_many_exact_ties_overflow_and_retry():
    rng = np.random.default_rng(7)
    v = rng.standard_normal(384).astype(np.float32)
    v /= np.linalg.norm(v)
    E = np.repeat(v[None, :], 6000, axis=0)  # 6000 identical rows: more candidates than the default capacity
    m = build(E)
    ids, s = m.search(v[None, :], 8, 0.6)
    assert ids.cpu().tolist() == [list(range(8))]
    assert np.allclose(s.cpu().numpy(), float(E[0] @ osearch.normalize_query(v)), atol=TOL)


def test_empty_store_rows():
    m = DeviceDonorMatrix(100, 384, DEV)  # nothing written: all rows invalid
    ids, _ = m.search(np.ones((3, 384), np.float32), 4, 0.0)
    assert torch.all(ids == -1)


def test_sharded_merge_equals_full_search():
    E, centers, rng = clustered(12000, 384, 32, seed=9)
    Q = queries_for(centers, rng, 200, 384)
    full = build(E)
    ids_f, s_f = full.search(Q, 8, 0.6)
    bounds = [0, 3500, 8000, 12000]
    parts_i, parts_s = [], []
    for a, b in zip(bounds[:-1], bounds[1:]):
        m = build(E[a:b])
        i, s = m.search(Q, 8, 0.6, id_offset=a)
        parts_i.append(i)
        parts_s.append(s)
    mi, ms = merge_topk(torch.stack(parts_i), torch.stack(parts_s))
    assert torch.equal(mi, ids_f)
    assert torch.equal(ms, s_f)


def test_donor_store_golden():
    g = load_golden("donor_store")

    class _A:
        reuse_ratio = 1.0

    store = ds.DonorStore(max_entries=300, embedding_dim=384, min_similarity=0.6, device=DEV,
                          alignment=(lambda *a, **k: 1.0, lambda *a, **k: _A()))
    for i, (rid, emb, none) in enumerate(zip(g["add_ids"].tolist(), g["add_embeddings"].numpy(),
                                             g["add_is_none"].numpy())):
        store.add_donor(ds.DonorNode(request_id=rid, token_ids=[i, i + 1, i + 2],
                                     embedding=None if none else emb, timestamp=0.0))
    assert np.array_equal(store._embeddings, g["embeddings"].numpy())
    assert np.array_equal(store._valid_mask, g["valid"].numpy())
    for qi, q in enumerate(g["queries"].numpy()):
        ms = store.find_donors(q, query_tokens=[-1], top_k=4, min_reuse_ratio=0.0)
        want = [x for x in g["result_ids"][qi].tolist() if x]
        assert [m.donor.request_id for m in ms] == want
        np.testing.assert_allclose([m.similarity for m in ms], g["result_sims"][qi].numpy()[: len(want)], atol=TOL)


def test_donor_store_batch_add_matches_sequential():
    rng = np.random.default_rng(2)
    nodes = [ds.DonorNode(f"r{i % 70}", [i], rng.standard_normal(64).astype(np.float32), 0.0) for i in range(150)]
    a = ds.DonorStore(max_entries=50, embedding_dim=64, device=DEV)
    b = ds.DonorStore(max_entries=50, embedding_dim=64, device=DEV)
    for n in nodes:
        a.add_donor(n)
    b.add_donors(nodes)
    assert np.array_equal(a._embeddings, b._embeddings)
    assert np.array_equal(a._valid_mask, b._valid_mask)
    assert torch.equal(a.device_matrix.valid.cpu().bool(), torch.from_numpy(a._valid_mask))


def test_bf16_shadow_vs_oracle():
    E, centers, rng = clustered(8000, 384, 16, seed=11)
    Q = queries_for(centers, rng, 200, 384)
    m = DeviceDonorMatrix(E.shape[0], 384, DEV, shadow_dtype=torch.bfloat16)
    m.write_range(0, torch.from_numpy(E).to(DEV))
    ids, s = m.search(Q, 8, 0.6)
    assert_topk_equivalent(E, np.ones(8000, bool), Q, 0.6, ids.cpu().numpy(), s.cpu().numpy(), 8)


def test_fp16_overflow_rows_stay_exact():
    rng = np.random.default_rng(12)
    E = rng.standard_normal((3000, 64)).astype(np.float32)
    E[17, 3] = 1e6  # beyond fp16 range: screening must fall back to rescoring everything
    E[18, 5] = -1e6
    Q = rng.standard_normal((5, 64)).astype(np.float32)
    Q[0] = E[17] / np.linalg.norm(E[17])
    m = build(E)
    ids, s = m.search(Q, 4, -1e9)
    assert_topk_equivalent(E, np.ones(3000, bool), Q, -1e9, ids.cpu().numpy(), s.cpu().numpy(), 4)
    assert ids[0, 0].item() == 17


def _merge_reference(ids, scores):
    """k-way merge by (score desc, id asc) of [L, Q, k] lists, -1 ids empty."""
    L, Q, k = ids.shape
    out_i = torch.full((Q, k), -1, dtype=torch.int64)
    out_s = torch.full((Q, k), -float("inf"))
    for q in range(Q):
        ent = [(float(scores[l, q, j]), int(ids[l, q, j])) for l in range(L) for j in range(k) if ids[l, q, j] >= 0]
        ent.sort(key=lambda e: (-e[0], e[1]))
        for r, (s, i) in enumerate(ent[:k]):
            out_i[q, r], out_s[q, r] = i, s
    return out_i, out_s


@pytest.mark.parametrize("n_lists,k", [(1, 8), (5, 8), (16, 3), (3, 16), (2, 32)])
def test_merge_strided_lists_with_ties_and_empties(n_lists, k):
    g = torch.Generator().manual_seed(n_lists * 100 + k)
    Q = 300
    ids = torch.full((n_lists, Q, k), -1, dtype=torch.int64)
    sc = torch.full((n_lists, Q, k), -float("inf"))
    for l in range(n_lists):
        for q in range(Q):
            n = int(torch.randint(0, k + 1, (1,), generator=g))
            s = torch.randint(0, 6, (n,), generator=g).float() / 8  # many ties across lists
            i = torch.randperm(100000, generator=g)[:n] * n_lists + l  # ids unique across lists
            order = sorted(range(n), key=lambda j: (-float(s[j]), int(i[j])))
            ids[l, q, :n] = i[order]
            sc[l, q, :n] = s[order]
    want_i, want_s = _merge_reference(ids, sc)
    # lists as strided views into larger per-list records (as after an all-gather)
    rec_i = torch.zeros(n_lists, Q * k + 40, dtype=torch.int64)
    rec_s = torch.zeros(n_lists, Q * k + 24)
    rec_i[:, : Q * k] = ids.reshape(n_lists, -1)
    rec_s[:, : Q * k] = sc.reshape(n_lists, -1)
    di, ds_ = rec_i.to(DEV), rec_s.to(DEV)
    got_i, got_s = merge_topk(di[:, : Q * k].view(n_lists, Q, k), ds_[:, : Q * k].view(n_lists, Q, k))
    assert torch.equal(got_i.cpu(), want_i)
    assert torch.equal(got_s.cpu(), want_s)


def test_radix_store_matches_reference_loop():
    """SGLang store: LRU keys, eviction, exclusion, strict threshold, ties by
    insertion order — against the reference's loop (restated in the oracle)."""
    from semblend_b200.radix_store import RadixDonorStore

    rng = np.random.default_rng(17)
    dim = 384
    centers = rng.standard_normal((6, dim)).astype(np.float32)
    ref = osearch.RadixStore(max_entries=40, min_similarity=0.6)
    ours = RadixDonorStore(max_entries=40, min_similarity=0.6, embedding_dim=dim, device=DEV)
    keys = []
    for step in range(140):
        if keys and rng.random() < 0.15:  # re-add an existing key (moves to the end)
            toks = keys[int(rng.integers(0, len(keys)))]
            emb = rng.standard_normal(dim).astype(np.float32)
        else:
            toks = tuple(int(x) for x in rng.integers(0, 50000, int(rng.integers(200, 400))))
            c = centers[int(rng.integers(0, 6))]
            emb = (c + 0.3 * rng.standard_normal(dim)).astype(np.float32)
            if rng.random() < 0.1 and keys:  # an exact duplicate embedding: a tie
                emb = ref.entries[keys[-1][:256]][1].copy() if keys[-1][:256] in ref.entries else emb
            keys.append(toks)
        ref.add_donor(toks, emb)
        ours.add_donor(toks, emb)
        assert ours.size == len(ref.entries)
        if step % 7 == 0:
            q = (centers[int(rng.integers(0, 6))] + 0.3 * rng.standard_normal(dim)).astype(np.float32)
            excl = keys[int(rng.integers(0, len(keys)))] if rng.random() < 0.5 else None
            want, want_sim = ref.find_donor(q, excl)
            got = ours.find_donor(q, excl)
            if want is None:
                assert got is None or float(np.dot(got.embedding, q / (np.linalg.norm(q) + 1e-10))) <= 0.6 + 1e-6
            else:
                assert got is not None
                got_sim = float(np.dot(got.embedding, q / (np.linalg.norm(q) + 1e-10)))
                assert got.token_ids == want or abs(got_sim - want_sim) <= 1e-6


def test_radix_store_ties_beyond_the_first_candidates():
    """Twelve exactly tied donors whose slots (recycled after evictions) are not
    in insertion order: the earliest-added one wins, as in the reference's loop."""
    from semblend_b200.radix_store import RadixDonorStore

    rng = np.random.default_rng(23)
    dim = 64
    ref = osearch.RadixStore(max_entries=16, min_similarity=0.5)
    ours = RadixDonorStore(max_entries=16, min_similarity=0.5, embedding_dim=dim, device=DEV)
    tied = rng.standard_normal(dim).astype(np.float32)
    for i in range(16):  # fill the store, then let the tied donors take recycled slots in mixed order
        emb = rng.standard_normal(dim).astype(np.float32)
        ref.add_donor((i,), emb)
        ours.add_donor((i,), emb)
    for j in range(12):
        toks = (1000 + j,)
        if j % 3 == 0:  # touch an old entry so evictions do not follow slot order
            ref.add_donor((13 - j // 3,), tied)
            ours.add_donor((13 - j // 3,), tied)
        ref.add_donor(toks, tied)
        ours.add_donor(toks, tied)
    for ex in (None, (1000,), (1003,)):
        want, _ = ref.find_donor(tied, ex)
        got = ours.find_donor(tied, ex)
        assert want is not None and got is not None and got.token_ids == want, (ex, got.token_ids, want)


def test_radix_store_matches_reference_golden():
    """The reference's own add_donor / find_donor run (goldens made by the
    reference): the same donor found at every lookup, up to similarities equal
    within 1e-6 (ties and the threshold)."""
    from semblend_b200.radix_store import RadixDonorStore
    from tests.test_oracle_golden import radix_replay

    g = load_golden("radix_store")
    dim = g["vec"].shape[1]
    thr = float(g["min_similarity"])
    ours = RadixDonorStore(max_entries=int(g["max_entries"]), min_similarity=thr, embedding_dim=dim, device=DEV)

    def find(q, ex):
        e = ours.find_donor(q, ex)
        if e is None:
            return None, None
        qn = q / (np.linalg.norm(q) + 1e-10)
        return e.token_ids, float(np.dot(e.embedding, qn))

    result, result_sim = g["result"].numpy(), g["result_sim"].numpy()
    for step, got, sim in radix_replay(ours.add_donor, find, g):
        want = result[step]
        if got == want:
            continue
        if want < 0:  # we found one the reference did not: only at the threshold
            assert sim <= thr + 1e-6, step
        elif got < 0:
            assert result_sim[step] <= thr + 1e-6, step
        else:  # a different donor: an exact tie
            assert abs(sim - result_sim[step]) <= 1e-6, step


def test_cagra_factory_is_the_exact_store():
    """make_donor_store(use_cagra=True) answers like DonorStore (the exact search
    replaces cuVS CAGRA); no index rebuild between adds and finds."""
    from semblend_b200.cagra_donor_store import CAGRADonorStore, make_donor_store

    rng = np.random.default_rng(5)

    class _A:
        reuse_ratio = 1.0

    align = (lambda *a, **k: 1.0, lambda *a, **k: _A())
    a = make_donor_store(max_entries=200, embedding_dim=384, min_similarity=0.5, use_cagra=True, device=DEV,
                         alignment=align)
    b = ds.DonorStore(max_entries=200, embedding_dim=384, min_similarity=0.5, device=DEV, alignment=align)
    assert isinstance(a, CAGRADonorStore)
    base = rng.standard_normal(384).astype(np.float32)
    for i in range(150):
        emb = base + 0.3 * rng.standard_normal(384).astype(np.float32)
        node = ds.DonorNode(request_id=f"r{i}", token_ids=[1, 2, 3, 1000 + i], embedding=emb / np.linalg.norm(emb),
                            timestamp=float(i))
        a.add_donor(node)
        b.add_donor(node)
        if i % 25 == 24:
            q = base + 0.3 * rng.standard_normal(384).astype(np.float32)
            ra = a.find_donors(q, [1, 2, 3], top_k=3)
            rb = b.find_donors(q, [1, 2, 3], top_k=3)
            assert ra
            assert [m.donor.request_id for m in ra] == [m.donor.request_id for m in rb]


# ----------------------------------------------------------------------------
# k beyond one kernel call, and the store's candidate widths
# ----------------------------------------------------------------------------
@pytest.mark.parametrize("k", [33, 40, 70, 100])
def test_wide_search_matches_oracle(k):
    """k > 32 runs in passes with the returned rows masked out; the result is
    the oracle's exact top-k (ties within 1e-6 aside), with invalid rows and
    the threshold respected."""
    E, centers, rng = clustered(12000, 384, 12, seed=30 + k)
    valid = rng.random(12000) > 0.1
    Q = queries_for(centers, rng, 12, 384)
    m = build(E, valid)
    before = m.valid.clone()
    ids, s = m.search(Q, k, 0.6)
    assert ids.shape == (12, k) and torch.equal(m.valid, before)  # the store's mask is untouched
    assert_topk_equivalent(E, valid, Q, 0.6, ids.cpu().numpy(), s.cpu().numpy(), k)


class _Aligned:
    reuse_ratio = 1.0


def test_find_donors_top_k_20_fetches_40_candidates():
    """find_donors(top_k=20) scores the 40 most similar donors above the
    threshold (donor_store.py:335-341); the old 32-candidate cap lost the
    ones ranked 33-40.  Donors ranked 1-25 are filtered by their reuse, so
    exactly those ranked 26-40 must come back, best first."""
    rng = np.random.default_rng(40)
    dim = 64
    base = rng.standard_normal(dim).astype(np.float32)
    embs = base + 0.25 * rng.standard_normal((120, dim)).astype(np.float32)
    query = base + 0.05 * rng.standard_normal(dim).astype(np.float32)
    valid = np.ones(120, bool)
    want_ids, want_sims = osearch.cosine_candidates(embs, valid, query, 0.6, 40)
    want_ids, want_sims = osearch.sort_candidates(want_ids, want_sims)
    assert want_ids.shape[0] == 40
    blocked = set(want_ids[:25].tolist())

    def est(donor_tokens, query_tokens, chunk_size=256):
        return 0.0 if donor_tokens[0] in blocked else 1.0

    store = ds.DonorStore(max_entries=200, embedding_dim=dim, min_similarity=0.6, device=DEV,
                          alignment=(est, lambda *a, **k: _Aligned()))
    # each donor shares the query's one token: Jaccard 0.5 passes the pre-filter at min_reuse_ratio 0.5
    store.add_donors([ds.DonorNode(f"d{i}", [i, -1], embs[i], timestamp=-1e9) for i in range(120)])
    ms = store.find_donors(query, query_tokens=[-1], top_k=20, min_reuse_ratio=0.5)
    assert [m.donor.request_id for m in ms] == [f"d{i}" for i in want_ids[25:40]]
    np.testing.assert_allclose([m.similarity for m in ms], want_sims[25:40], atol=TOL)


def _token_cases(rng, chunk):
    """A query and donors that share reordered whole chunks with it, share only
    tokens (the multiset fallback), share nothing, or are shorter than a chunk."""
    q = rng.integers(0, 5000, 8 * chunk)
    chunks = [q[i * chunk:(i + 1) * chunk] for i in range(8)]
    donors = [
        np.concatenate([chunks[3], chunks[4], chunks[5], rng.integers(0, 5000, chunk), chunks[0], chunks[1]]),
        np.concatenate([chunks[6], chunks[7]]),
        rng.permutation(q)[: 5 * chunk],            # same tokens, no whole chunk
        rng.integers(5000, 9000, 6 * chunk),        # nothing in common
        q[: chunk // 2].copy(),                     # shorter than one chunk
        np.concatenate([chunks[2], chunks[2], chunks[2]]),  # a chunk repeated
    ]
    return q, donors


def test_estimate_reuse_ratio_batch_matches_oracle():
    from oracle import alignment as oal
    from semblend_b200.alignment import estimate_reuse_ratio, estimate_reuse_ratio_batch

    rng = np.random.default_rng(41)
    q, donors = _token_cases(rng, 64)
    got = estimate_reuse_ratio_batch([d.tolist() for d in donors], q.tolist(), 64, device=DEV)
    want = [oal.estimate_reuse_ratio(d.tolist(), q.tolist(), 64) for d in donors]
    assert got == pytest.approx(want, abs=0) and 0 < min(w for w in want if w > 0) < max(want)
    assert [estimate_reuse_ratio(d.tolist(), q.tolist(), 64, device=DEV) for d in donors] == got


def test_donor_store_reuse_on_device_matches_oracle():
    """With no alignment override, the store estimates every candidate's reuse
    on the device (one batched call) and aligns the winners on the device;
    the matches equal the oracle's walk of the same steps: cosine top-2k,
    Jaccard pre-filter, estimate_reuse_ratio, sim x reuse order, and the final
    alignment's reuse (gated exact chunks, else the token-set fallback) as the
    last filter."""
    from oracle import alignment as oal

    chunk = 64
    rng = np.random.default_rng(42)
    q, donors = _token_cases(rng, chunk)
    dim = 32
    base = rng.standard_normal(dim).astype(np.float32)
    embs = base + 0.2 * rng.standard_normal((len(donors), dim)).astype(np.float32)
    query = base.copy()
    store = ds.DonorStore(max_entries=16, embedding_dim=dim, min_similarity=0.6, chunk_size=chunk, device=DEV)
    store.add_donors([ds.DonorNode(f"d{i}", d.tolist(), embs[i], timestamp=-1e9) for i, d in enumerate(donors)])
    ms = store.find_donors(query, q.tolist(), top_k=3, min_reuse_ratio=0.2)

    cand, sims = osearch.cosine_candidates(embs, np.ones(len(donors), bool), query, 0.6, 6)
    qset = set(q.tolist())
    scored = []
    for i, s in zip(cand.tolist(), sims.tolist()):
        dset = set(donors[i].tolist())
        if len(qset & dset) / len(qset | dset) < 0.2:
            continue
        r = oal.estimate_reuse_ratio(donors[i].tolist(), q.tolist(), chunk)
        if r >= 0.2:
            scored.append((s * r, s, i))
    scored.sort(key=lambda x: x[0], reverse=True)
    want = []
    for _, s, i in scored[:3]:
        m = oal.chunk_matches(donors[i].tolist(), q.tolist(), chunk, True)
        reuse = (m >= 0).sum() * chunk / len(q)
        if reuse == 0:
            reuse = oal.token_overlap(donors[i].tolist(), q.tolist()) / len(q)
        if reuse >= 0.2:
            want.append((f"d{i}", s))
    assert want, "the case must produce matches"
    assert [m.donor.request_id for m in ms] == [w[0] for w in want]
    np.testing.assert_allclose([m.similarity for m in ms], [w[1] for w in want], atol=TOL)
    for m in ms:
        assert m.alignment.reuse_ratio >= 0.2


def _split_search(m, Q, k, thr, rs, owner, out=None, n_rows=None, id_offset=0):
    from semblend_b200.search import cosine_topk_async

    return cosine_topk_async(m.emb, m.emb16, m.valid, m.stats, Q, k, thr, n_rows=n_rows, id_offset=id_offset,
                             workspace_owner=owner, out=out, rescore_stream=rs)


@pytest.mark.parametrize("k", [1, 8, 17, 32])
def test_screen_then_rescore_on_another_stream_equals_one_call(k):
    """sb_cosine_screen on the current stream + sb_cosine_rescore on a second
    stream give the bits of one sb_cosine_topk call (ragged valid mask,
    id offset, a row count below the matrix size)."""
    from semblend_b200.search import cosine_topk_async

    E, centers, rng = clustered(20011, 384, 32, seed=21)
    valid = rng.random(E.shape[0]) > 0.1
    m = build(E, valid)
    Q = torch.from_numpy(queries_for(centers, rng, 333, 384)).to(DEV)
    ids_f, s_f, st_f = cosine_topk_async(m.emb, m.emb16, m.valid, m.stats, Q, k, 0.55, n_rows=19000, id_offset=7)
    rs = torch.cuda.Stream(DEV)

    class Owner:
        pass

    ids_s, s_s, st_s = _split_search(m, Q, k, 0.55, rs, Owner(), n_rows=19000, id_offset=7)
    torch.cuda.current_stream(DEV).wait_stream(rs)
    assert int(st_f.item()) == 0 and int(st_s.item()) == 0
    assert torch.equal(ids_s, ids_f) and torch.equal(s_s, s_f)
    assert int(ids_s.max().item()) < 19000 + 7


def test_split_search_with_no_rows_fills_empty():
    m = DeviceDonorMatrix(64, 384, DEV)
    rs = torch.cuda.Stream(DEV)
    ids, sc, st = _split_search(m, torch.ones(5, 384, device=DEV), 4, 0.0, rs, None, n_rows=0)
    torch.cuda.current_stream(DEV).wait_stream(rs)
    assert torch.all(ids == -1) and torch.all(sc == -torch.inf) and int(st.item()) == 0


def test_pipelined_split_search_with_two_workspaces():
    """The sharded pipeline's pattern on one GPU: batch i is rescored on a
    second stream while batch i+1 is screened, the two slots alternating their
    workspaces and output buffers; every batch equals its own one-call search."""
    from semblend_b200.search import cosine_topk_async

    E, centers, rng = clustered(30000, 384, 32, seed=23)
    m = build(E)
    Qs = [torch.from_numpy(queries_for(centers, rng, 256, 384)).to(DEV) for _ in range(3)]
    want = [cosine_topk_async(m.emb, m.emb16, m.valid, m.stats, q, 8, 0.6)[:2] for q in Qs]

    class Owner:
        pass

    cur, rs = torch.cuda.current_stream(DEV), torch.cuda.Stream(DEV)
    owners = [Owner(), Owner()]
    outs = [(torch.empty(256, 8, dtype=torch.int64, device=DEV), torch.empty(256, 8, device=DEV)) for _ in range(2)]
    done = [torch.cuda.Event() for _ in range(2)]
    got = []
    for i in range(7):
        slot = i % 2
        if i >= 2:
            cur.wait_event(done[slot])
        ids, sc, st = _split_search(m, Qs[i % 3], 8, 0.6, rs, owners[slot], out=outs[slot])
        with torch.cuda.stream(rs):
            got.append((ids.clone(), sc.clone(), st.clone()))
            done[slot].record(rs)
    cur.wait_stream(rs)
    torch.cuda.synchronize(DEV)
    for i, (ids, sc, st) in enumerate(got):
        assert int(st.item()) == 0
        assert torch.equal(ids, want[i % 3][0]) and torch.equal(sc, want[i % 3][1]), i


@pytest.mark.parametrize("dim,nq", [(64, 260), (100, 383), (384, 4096), (512, 257)])
def test_large_batches_vs_oracle(dim, nq):
    """Batches of several query tiles (each donor chunk shared by concurrent
    CTAs, each starting at its own tile of the chunk), a partial last tile, and
    d = 512 (the largest query tile in shared memory)."""
    E, centers, rng = clustered(9000, dim, 16, seed=dim + nq)
    Q = queries_for(centers, rng, nq, dim)
    m = build(E)
    ids, s = m.search(Q, 8, 0.5)
    assert_topk_equivalent(E, np.ones(E.shape[0], bool), Q, 0.5, ids.cpu().numpy(), s.cpu().numpy(), 8)
