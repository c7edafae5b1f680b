"""Pin the CPU oracle to the reference: every golden fixture (produced by
running SemBlend 0.3.2's own code, tests/golden/make_golden.py) must be
reproduced by the oracle — bit for bit for the RoPE / scatter family."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle import rope as orope
from oracle import search as osearch
from tests.helpers import load_golden


@pytest.mark.parametrize("name", ["rcsp_fp32", "rcsp_bf16", "rcsp_fp16", "rcsp_c1mini"])
def test_rope_correct_scatter_paged_matches_reference(name):
    g = load_golden(name)
    out = orope.rope_correct_scatter_paged(
        g["cache"], g["donor"], g["block_table"], g["d_pos"], g["t_pos"], rope_base=g["rope_base"]
    )
    assert torch.equal(out.view(torch.int8) if out.dtype != torch.float32 else out,
                       g["out"].view(torch.int8) if out.dtype != torch.float32 else g["out"])


def test_scatter_flat_matches_reference():
    g = load_golden("scatter_flat")
    out = orope.scatter_donor_kv(g["target"], g["donor"], g["d_pos"], g["t_pos"])
    assert torch.equal(out, g["out"])


def test_scatter_paged_matches_reference():
    g = load_golden("scatter_paged")
    out = orope.scatter_donor_kv_paged(g["cache"], g["donor"], g["block_table"], g["d_pos"], g["t_pos"])
    assert torch.equal(out, g["out"])


@pytest.mark.parametrize("name", ["rck_3d_fp32", "rck_4d_bf16"])
def test_rope_correct_k_matches_reference(name):
    g = load_golden(name)
    out = orope.rope_correct_k(g["k"], g["d_pos"], g["t_pos"], head_dim=g["head_dim"], rope_base=g["rope_base"])
    assert torch.equal(out.view(torch.int16) if out.dtype == torch.bfloat16 else out,
                       g["out"].view(torch.int16) if out.dtype == torch.bfloat16 else g["out"])


@pytest.mark.parametrize("name", ["permute_fp32", "permute_bf16"])
def test_permute_matches_reference(name):
    g = load_golden(name)
    pairs = [tuple(p) for p in g["pairs"].tolist()]
    out = orope.permute_paged_kv_with_rope(g["cache"], g["block_table"], pairs, rope_base=g["rope_base"])
    assert torch.equal(out.float(), g["out"].float())


def test_nope_matches_reference():
    g = load_golden("nope_fp16")
    pairs = [tuple(p) for p in g["pairs"].tolist()]
    out = orope.nope_permute_paged_kv(g["cache"], g["block_table"], pairs, rope_base=g["rope_base"])
    assert torch.equal(out, g["out"])
    # the fixture's sources and targets are disjoint, so snapshot V semantics agree
    out2 = orope.nope_permute_paged_kv(g["cache"], g["block_table"], pairs, rope_base=g["rope_base"],
                                       v_from_snapshot=True)
    assert torch.equal(out2, g["out"])


@pytest.mark.parametrize("name", ["ropedelta_canon", "ropedelta_vllm"])
def test_apply_rope_delta_matches_reference(name):
    g = load_golden(name)
    out, n = orope.apply_rope_delta_inplace(
        g["cache"], g["block_table"], g["positions"].tolist(), g["delta"], rope_base=g["rope_base"]
    )
    assert n == g["count"]
    assert torch.equal(out.float(), g["out"].float())


def test_neox_is_conjugated_interleaved():
    g = load_golden("rcsp_fp32")
    perm = orope._perm(g["cache"].shape[-1])
    inv = torch.argsort(perm)
    # neox on permuted inputs == permuted interleaved result
    donor_neox = g["donor"][..., inv]
    cache_neox = g["cache"][..., inv]
    out = orope.rope_correct_scatter_paged(cache_neox, donor_neox, g["block_table"], g["d_pos"], g["t_pos"],
                                           rope_base=g["rope_base"], rotary_style="neox")
    assert torch.equal(out, g["out"][..., inv])


@pytest.mark.parametrize("name", ["attn_small", "attn_mid"])
def test_attention_matches_reference(name):
    g = load_golden(name)
    out = oatt.partial_prefill_attention(g["q"], g["k"], g["v"], g["mask"])
    torch.testing.assert_close(out, g["out"], rtol=0, atol=1e-6)
    rows = torch.where(g["mask"])[0]
    blk = oatt.partial_prefill_attention_blocked(g["q"], g["k"], g["v"], rows)
    torch.testing.assert_close(blk, g["out"][:, rows, :], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("name", ["proj_fp32", "proj_fp16"])
def test_projection_matches_reference(name):
    g = load_golden(name)
    out = oatt.masked_qkv_projection(g["h"], g["w"], g["mask"], g.get("b"))
    assert torch.equal(out, g["out"])


def test_store_rows_and_cosine_stage_match_reference():
    g = load_golden("donor_store")
    rows = osearch.StoreRows(300, 384)
    for rid, emb, none in zip(g["add_ids"].tolist(), g["add_embeddings"].numpy(), g["add_is_none"].numpy()):
        rows.add(rid, None if none else emb)
    assert np.array_equal(rows.embeddings, g["embeddings"].numpy())
    assert np.array_equal(rows.valid, g["valid"].numpy())
    assert dict(rows.entries) == dict(zip(g["id_to_idx_keys"].tolist(), g["id_to_idx_vals"].tolist()))
    idx_to_id = {v: k for k, v in rows.entries.items()}
    for qi, q in enumerate(g["queries"].numpy()):
        c, s = osearch.cosine_candidates(rows.embeddings, rows.valid, q, 0.6, 8)
        c, s = osearch.sort_candidates(c, s)
        want = [x for x in g["result_ids"][qi].tolist() if x]
        got = [idx_to_id[int(i)] for i in c[: len(want)]]
        assert got == want
        np.testing.assert_array_equal(s[: len(want)], g["result_sims"][qi].numpy()[: len(want)].astype(np.float32))


@pytest.mark.parametrize("name", ["align_gate", "align_nogate", "align_small"])
def test_alignment_oracle_matches_reference(name):
    from oracle import alignment as oal

    g = load_golden(name)
    donor, target = g["donor"].tolist(), g["target"].tolist()
    chunk, gate = int(g["chunk"]), bool(g["gate"])
    assert np.array_equal(oal.digests(donor, chunk), g["donor_digests"].numpy())
    assert np.array_equal(oal.digests(target, chunk), g["target_digests"].numpy())
    match = oal.chunk_matches(donor, target, chunk, gate)
    assert np.array_equal(match, g["match"].numpy())
    n_match = int((match >= 0).sum())
    assert n_match == int(g["exact_chunks"])
    assert n_match * chunk / len(target) == pytest.approx(float(g["reuse_ratio"]), abs=0)
    est = oal.estimate_chunk_reuse(donor, target, chunk)
    assert est == pytest.approx(float(g["estimate"]), abs=0)


@pytest.mark.parametrize("name", ["align_gate", "align_nogate", "align_small", "reuse_fallback", "reuse_short"])
def test_reuse_ratio_oracle_matches_reference(name):
    """estimate_reuse_ratio: chunk stage, else the token-multiset fallback."""
    from oracle import alignment as oal

    g = load_golden(name)
    donor, target, chunk = g["donor"].tolist(), g["target"].tolist(), int(g["chunk"])
    assert oal.estimate_reuse_ratio(donor, target, chunk) == pytest.approx(float(g["estimate"]), abs=0)
    if name.startswith("reuse"):  # these goldens exercise the fallback: no full chunk in common
        assert not (oal.chunk_matches(donor, target, chunk, False) >= 0).any()


def radix_replay(store_add, store_find, g):
    """Replay the golden add_donor / find_donor run; yields (step, found sequence id or -1,
    similarity of the found donor or None) for every lookup."""
    lens = g["seq_lens"].numpy()
    flat = g["seq_tokens"].numpy()
    offs = np.concatenate([[0], np.cumsum(lens)])
    seqs = [tuple(int(x) for x in flat[offs[i] : offs[i + 1]]) for i in range(len(lens))]
    index = {}
    for i, t in enumerate(seqs):
        index.setdefault(t, i)
    op, seq, vec = g["op"].numpy(), g["seq"].numpy(), g["vec"].numpy()
    for step in range(op.shape[0]):
        if op[step] == 0:
            store_add(seqs[seq[step]], vec[step])
        else:
            ex = seqs[seq[step]] if seq[step] >= 0 else None
            toks, sim = store_find(vec[step], ex)
            yield step, (-1 if toks is None else index[tuple(toks)]), sim


def test_radix_oracle_matches_reference():
    """The SGLang donor store loop (radix_backend.py:144-211), restated in the
    oracle, against the reference run on the same operations."""
    from oracle import search as osearch

    g = load_golden("radix_store")
    ref = osearch.RadixStore(max_entries=int(g["max_entries"]), min_similarity=float(g["min_similarity"]))
    result, result_sim = g["result"].numpy(), g["result_sim"].numpy()
    n = 0
    for step, got, sim in radix_replay(ref.add_donor, ref.find_donor, g):
        assert got == result[step], step
        if got >= 0:
            assert sim == result_sim[step]
        n += 1
    assert n == int((g["op"].numpy() == 1).sum()) and (result[g["op"].numpy() == 1] == -1).any()
