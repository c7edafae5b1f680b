"""Generate golden fixtures by running the reference implementation itself.

Imports the reference package (SemBlend 0.3.2) from the checkout named by
``$SEMBLEND_REFERENCE`` (required: there is no default location, and the GPU
machines have no checkout), runs its
CPU code paths on small seeded inputs and writes ``tests/golden/*.npz`` plus
``plans.json``.  The fixtures are committed; nothing at test time reads the
reference.  Re-run with ``SEMBLEND_REFERENCE=<checkout> python tests/golden/make_golden.py``.

bf16 tensors are stored as their int16 bit patterns with a ``<name>__bf16``
key suffix (numpy has no bfloat16).
"""

from __future__ import annotations

import json
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REF = Path(os.environ["SEMBLEND_REFERENCE"]) if os.environ.get("SEMBLEND_REFERENCE") else None


def _np(t: torch.Tensor) -> tuple[str, np.ndarray]:
    if t.dtype == torch.bfloat16:
        return "__bf16", t.view(torch.int16).numpy().copy()
    return "", t.numpy().copy()


def save(name: str, **tensors) -> None:
    out = {}
    for k, v in tensors.items():
        if isinstance(v, torch.Tensor):
            suf, arr = _np(v)
            out[k + suf] = arr
        else:
            out[k] = np.asarray(v)
    np.savez_compressed(HERE / f"{name}.npz", **out)


def gen(seed: int) -> torch.Generator:
    return torch.Generator().manual_seed(seed)


def main() -> int:
    if REF is None or not (REF / "semblend_core").is_dir():
        print("make_golden: set SEMBLEND_REFERENCE to a SemBlend 0.3.2 checkout (the directory holding "
              "semblend_core/)", file=sys.stderr)
        return 2
    sys.path.insert(0, str(REF))
    import semblend_core.donor_store as ds
    import semblend_core.partial_attention as pa
    import semblend_core.rope_correction as rc
    import semblend_core.triton_kernels as tk

    torch.set_num_threads(1)

    # --- rope_correct_scatter_paged (CPU path, rope_correction.py:285-328) ---
    def rcsp_case(name, seed, dtype, H, D, Sd, nb, bs, n_log, pairs, base):
        g = gen(seed)
        donor = torch.randn(2, H, Sd, D, generator=g).to(dtype)
        cache = torch.randn(nb, 2, H, bs, D, generator=g).to(dtype)
        bt = torch.randperm(nb, generator=g)[:n_log].to(torch.int32)
        d = torch.tensor([p[0] for p in pairs], dtype=torch.int32)
        t = torch.tensor([p[1] for p in pairs], dtype=torch.int32)
        out = rc.rope_correct_scatter_paged(cache.clone(), donor, bt, d, t, rope_base=base)
        save(name, donor=donor, cache=cache, block_table=bt, d_pos=d, t_pos=t, out=out, rope_base=base)

    rng = np.random.default_rng(11)
    tg = rng.permutation(48)[:40]
    pairs = [(int(rng.integers(0, 96)), int(x)) for x in tg]
    rcsp_case("rcsp_fp32", 1, torch.float32, 4, 128, 96, 16, 4, 12, pairs, 1e6)
    rcsp_case("rcsp_bf16", 2, torch.bfloat16, 4, 128, 96, 16, 4, 12, pairs, 1e4)
    rcsp_case("rcsp_fp16", 3, torch.float16, 2, 64, 96, 16, 4, 12, pairs, 1e4)
    # c1-shaped miniature: 4 chunks of 64 tokens in a seeded permutation
    perm = np.random.default_rng(5).permutation(4)
    c1pairs = [(64 * int(perm[c]) + i, 64 * c + i) for c in range(4) for i in range(64)]
    rcsp_case("rcsp_c1mini", 4, torch.float32, 2, 128, 256, 18, 16, 16, c1pairs, 1e6)

    # --- scatter_donor_kv / scatter_donor_kv_paged (triton_kernels.py:185-189, :338-355) ---
    g = gen(6)
    target = torch.randn(2, 2, 4, 16, 32, generator=g).to(torch.float16)
    donor = torch.randn(2, 2, 4, 8, 32, generator=g).to(torch.float16)
    d = torch.tensor([0, 2, 4, 6, 7], dtype=torch.int32)
    t = torch.tensor([1, 3, 7, 12, 15], dtype=torch.int32)
    out = tk.scatter_donor_kv(target.clone(), donor, d, t)
    save("scatter_flat", target=target, donor=donor, d_pos=d, t_pos=t, out=out)

    kv = torch.randn(8, 2, 4, 4, 32, generator=g).to(torch.float16)
    dkv = torch.randn(2, 4, 16, 32, generator=g).to(torch.float16)
    bt = torch.tensor([3, 5, 0, 6], dtype=torch.int32)
    d = torch.tensor([0, 4, 9, 15, 2], dtype=torch.int32)
    t = torch.tensor([1, 5, 14, 8, 3], dtype=torch.int32)
    out = tk.scatter_donor_kv_paged(kv.clone(), dkv, bt, d, t)
    save("scatter_paged", cache=kv, donor=dkv, block_table=bt, d_pos=d, t_pos=t, out=out)

    # --- rope_correct_k (rope_correction.py:362-399) ---
    g = gen(7)
    k3 = torch.randn(4, 40, 128, generator=g)
    d = torch.tensor([0, 5, 9, 33, 17], dtype=torch.int32)
    t = torch.tensor([3, 5, 1, 39, 1000], dtype=torch.int32)
    out = rc.rope_correct_k(k3, d, t, head_dim=128, rope_base=1e6)
    save("rck_3d_fp32", k=k3, d_pos=d, t_pos=t, out=out, rope_base=1e6, head_dim=128)
    k4 = torch.randn(3, 2, 24, 64, generator=g).to(torch.bfloat16)
    d = torch.tensor([2, 4, 6, 20], dtype=torch.int32)
    t = torch.tensor([12, 0, 300, 21], dtype=torch.int32)
    out = rc.rope_correct_k(k4, d, t, head_dim=64, rope_base=1e4)
    save("rck_4d_bf16", k=k4, d_pos=d, t_pos=t, out=out, rope_base=1e4, head_dim=64)

    # --- permute_paged_kv_with_rope (rope_correction.py:427-476), overlapping ---
    for name, seed, dtype in (("permute_fp32", 8, torch.float32), ("permute_bf16", 9, torch.bfloat16)):
        g = gen(seed)
        kv = torch.randn(8, 2, 2, 16, 64, generator=g).to(dtype)
        bt = torch.randperm(8, generator=g)[:6].to(torch.int32)
        # swap chunk [0,32) with [32,64), shift [64,80) to [80,96)
        perm_pairs = [(i, i + 32) for i in range(32)] + [(i + 32, i) for i in range(32)]
        perm_pairs += [(64 + i, 80 + i) for i in range(16)]
        out = kv.clone()
        rc.permute_paged_kv_with_rope(out, bt, perm_pairs, rope_base=1e4)
        save(name, cache=kv, block_table=bt, pairs=np.array(perm_pairs, np.int64), out=out, rope_base=1e4)

    # --- nope_permute_paged_kv (rope_correction.py:620-696, CPU :797-823), disjoint ---
    g = gen(10)
    kv = torch.randn(8, 2, 4, 16, 64, generator=g).to(torch.float16)
    bt = torch.arange(8, dtype=torch.int32)
    nope_pairs = [(i, 64 + ((i * 7) % 48)) for i in range(48)]
    out = kv.clone()
    rc.nope_permute_paged_kv(out, bt, nope_pairs, rope_base=1e4)
    save("nope_fp16", cache=kv, block_table=bt, pairs=np.array(nope_pairs, np.int64), out=out, rope_base=1e4)

    # --- apply_rope_delta_inplace (rope_correction.py:732-783), both layouts ---
    g = gen(12)
    canon = torch.randn(6, 2, 4, 8, 64, generator=g)
    vllm = torch.randn(2, 6, 8, 4, 64, generator=g).to(torch.bfloat16)
    bt = torch.tensor([4, 1, 5, 0], dtype=torch.int32)
    positions = [0, 3, 9, 9, 17, 31, 40, 45]
    for name, cache in (("ropedelta_canon", canon), ("ropedelta_vllm", vllm)):
        out = cache.clone()
        n = rc.apply_rope_delta_inplace(out, bt, positions, delta=37, rope_base=1e4)
        save(name, cache=cache, block_table=bt, positions=np.array(positions), out=out, count=n, delta=37,
             rope_base=1e4)

    # --- partial_prefill_attention CPU branch (triton_kernels.py:717-732) ---
    for name, seed, H, S, D in (("attn_small", 13, 2, 48, 16), ("attn_mid", 14, 4, 96, 64)):
        g = gen(seed)
        q = torch.randn(H, S, D, generator=g)
        k = torch.randn(H, S, D, generator=g)
        v = torch.randn(H, S, D, generator=g)
        mask = torch.rand(S, generator=g) < 0.3
        mask[-1] = True
        out = tk.partial_prefill_attention(q, k, v, mask)
        save(name, q=q, k=k, v=v, mask=mask, out=out)

    # --- masked_qkv_projection CPU branch (triton_kernels.py:512-520) ---
    g = gen(15)
    h = torch.randn(24, 64, generator=g)
    w = torch.randn(96, 64, generator=g) * 0.1
    b = torch.randn(96, generator=g)
    mask = torch.rand(24, generator=g) < 0.5
    save("proj_fp32", h=h, w=w, b=b, mask=mask, out=tk.masked_qkv_projection(h, w, mask, b))
    h16, w16 = h.half(), w.half()
    save("proj_fp16", h=h16, w=w16, mask=mask, out=tk.masked_qkv_projection(h16, w16, mask))

    # --- DonorStore row bookkeeping + cosine stage (donor_store.py:130-168, :299-407) ---
    rng = np.random.default_rng(16)
    dim, max_entries = 384, 300
    centers = rng.standard_normal((8, dim)).astype(np.float32)
    store = ds.DonorStore(max_entries=max_entries, embedding_dim=dim, min_similarity=0.6)
    ids, embs = [], []
    for i in range(400):
        c = centers[i % 8]
        e = (c + 0.3 * rng.standard_normal(dim)).astype(np.float32)
        e /= np.linalg.norm(e)
        if i % 37 == 5:
            e = None
        rid = f"req-{i}"
        if i % 53 == 7 and ids:
            rid = ids[-3]  # duplicate add: LRU refresh only
        ids.append(rid)
        embs.append(np.zeros(dim, np.float32) if e is None else e)
        store.add_donor(ds.DonorNode(request_id=rid, token_ids=[i, i + 1, i + 2], embedding=e, timestamp=0.0))
    # make the token-level stages pass everything through so find_donors ranks by cosine
    ds.estimate_reuse_ratio = lambda *a, **k: 1.0

    class _A:
        reuse_ratio = 1.0

    ds.compute_alignment = lambda *a, **k: _A()
    queries = []
    for j in range(12):
        if j < 8:
            q = centers[j % 8] + 0.3 * rng.standard_normal(dim)
        else:
            q = rng.standard_normal(dim)
        queries.append(q.astype(np.float32) * (1.0 + j))  # un-normalised on purpose
    results = []
    for q in queries:
        ms = store.find_donors(q, query_tokens=[-1], top_k=4, min_reuse_ratio=0.0)
        results.append([(m.donor.request_id, float(m.similarity)) for m in ms])
    save(
        "donor_store",
        add_ids=np.array(ids),
        add_embeddings=np.stack(embs),
        add_is_none=np.array([(i % 37 == 5) for i in range(400)]),
        embeddings=store._embeddings,
        valid=store._valid_mask,
        id_to_idx_keys=np.array(list(store._id_to_idx.keys())),
        id_to_idx_vals=np.array(list(store._id_to_idx.values())),
        queries=np.stack(queries),
        result_ids=np.array([[r[0] for r in res] + [""] * (4 - len(res)) for res in results]),
        result_sims=np.array([[r[1] for r in res] + [np.nan] * (4 - len(res)) for res in results]),
    )

    # --- partial_attention plan functions (partial_attention.py:105-435) ---
    plans = []
    slot_actions = [{"action": "copy_from_donor", "targetPos": i, "donorPos": (i * 3) % 50} for i in range(40)]
    slot_actions += [{"action": "placeholder", "targetPos": i} for i in range(40, 50)]
    hints = [{"recomputeAll": i in (0, 5), "deviationScore": 0.1 * i} for i in range(6)]
    plan = pa.build_attention_plan("d1", 50, 50, list(range(40)), list(range(40, 50)), slot_actions, hints, num_layers=8)
    plans.append({
        "kind": "single", "args": {"donor_id": "d1", "target_len": 50, "donor_len": 50,
                                   "copy_positions": list(range(40)), "placeholder_positions": list(range(40, 50)),
                                   "slot_actions": slot_actions, "layer_hints": hints, "num_layers": 8},
        "num_reuse": plan.num_reuse_positions, "num_partial": plan.num_partial_positions,
        "num_full_layers": plan.num_full_layers, "computation_ratio": plan.computation_ratio,
        "masks": [pa.compute_attention_mask(plan, l).tolist() for l in range(9)],
        "pairs": [pa.compute_donor_kv_indices(plan, l) for l in range(9)],
    })
    md_actions = [{"action": "copy_from_donor", "targetPos": i, "donorPos": i + 7, "donorId": f"d{i % 3}"} for i in range(30)]
    md_actions += [{"action": "recompute", "targetPos": i, "donorPos": None} for i in range(30, 36)]
    plan = pa.build_multi_donor_attention_plan(36, md_actions, [{"recompute_all": True}], num_layers=3)
    plans.append({
        "kind": "multi", "args": {"target_len": 36, "slot_actions": md_actions,
                                  "layer_hints": [{"recompute_all": True}], "num_layers": 3},
        "num_reuse": plan.num_reuse_positions, "num_partial": plan.num_partial_positions,
        "num_full_layers": plan.num_full_layers, "computation_ratio": plan.computation_ratio,
        "donor_len": plan.donor_len, "donor_id": plan.donor_id, "donor_map": [list(x) for x in plan.donor_map],
        "masks": [pa.compute_attention_mask(plan, l).tolist() for l in range(3)],
        "pairs": [pa.compute_donor_kv_indices(plan, l) for l in range(3)],
    })
    (HERE / "plans.json").write_text(json.dumps(plans, indent=0))

    # --- chunk-hash alignment (alignment.py:120-268, :741-787) ---
    import semblend_core.alignment as al

    def align_case(name, seed, chunk, n_donor_chunks, gate):
        rng = np.random.default_rng(seed)
        donor = rng.integers(0, 152064, n_donor_chunks * chunk + chunk // 3).astype(np.int64)
        dch = [donor[i * chunk : (i + 1) * chunk] for i in range(n_donor_chunks)]
        pieces = []
        for i in range(n_donor_chunks + 6):
            r = rng.random()
            if r < 0.55:  # a donor chunk, anywhere
                pieces.append(dch[int(rng.integers(0, n_donor_chunks))])
            elif r < 0.65 and pieces:  # a repeat of an earlier target chunk
                pieces.append(pieces[int(rng.integers(0, len(pieces)))])
            else:  # new content
                pieces.append(rng.integers(0, 152064, chunk))
        target = np.concatenate(pieces + [rng.integers(0, 152064, chunk // 2)])
        dl, tl = donor.tolist(), target.tolist()
        res = al.compute_chunk_alignment(dl, tl, chunk_size=chunk, context_gate=gate)
        n_t = (len(tl) + chunk - 1) // chunk
        match = np.full(n_t, -1, np.int64)
        for a in res.slot_actions:
            if a.action == al.SlotActionType.COPY_FROM_DONOR and a.target_pos % chunk == 0:
                match[a.target_pos // chunk] = a.donor_pos // chunk
        digests = lambda toks: np.array([[int(al._chunk_hash(toks[i * chunk : (i + 1) * chunk])[8 * w : 8 * w + 8], 16)
                                          for w in range(4)] for i in range(len(toks) // chunk)], np.uint32)
        save(name, donor=donor, target=target, chunk=chunk, gate=int(gate), match=match,
             reuse_ratio=res.reuse_ratio, exact_chunks=res.exact_chunks,
             estimate=al.estimate_reuse_ratio(dl, tl, chunk_size=chunk),
             donor_digests=digests(dl), target_digests=digests(tl))

    align_case("align_gate", 31, 256, 24, True)
    align_case("align_nogate", 32, 256, 24, False)
    align_case("align_small", 33, 16, 60, True)

    # estimate_reuse_ratio's token-multiset fallback (:776-785): no full chunk in common
    def reuse_case(name, seed, chunk, n_donor, n_shared, n_new):
        rng = np.random.default_rng(seed)
        donor = rng.integers(0, 300, n_donor).astype(np.int64)  # small vocabulary: repeated ids
        shared = rng.permutation(donor)[:n_shared]
        target = np.concatenate([shared, rng.integers(200, 600, n_new)]).astype(np.int64)
        dl, tl = donor.tolist(), target.tolist()
        save(name, donor=donor, target=target, chunk=chunk,
             estimate=al.estimate_reuse_ratio(dl, tl, chunk_size=chunk))

    reuse_case("reuse_fallback", 41, 64, 5 * 64 + 7, 3 * 64, 2 * 64 + 5)
    reuse_case("reuse_short", 42, 256, 900, 100, 50)

    # --- the SGLang integration's donor store (radix_backend.py:124-211) ---
    import semblend.integration.sglang.radix_backend as rb

    def radix_case(name, seed, n_ops, max_entries, min_sim):
        """A replayable run of add_donor / find_donor: re-added keys, evictions,
        exclusions and exactly tied embeddings; `result` is the id of the found
        donor's token sequence (-1: none), its similarity in `result_sim`."""
        rng = np.random.default_rng(seed)
        dim = 64
        centers = rng.standard_normal((6, dim)).astype(np.float32)
        store = rb._SemBlendDonorStore(max_entries=max_entries, min_similarity=min_sim)
        seqs, ops, seq_id, embs, excl, result, result_sim = [], [], [], [], [], [], []
        for step in range(n_ops):
            if step % 5 == 4:  # a lookup
                q = (centers[int(rng.integers(0, 6))] + 0.3 * rng.standard_normal(dim)).astype(np.float32)
                if rng.random() < 0.25:  # far from every donor: no match above the threshold
                    q = rng.standard_normal(dim).astype(np.float32)
                ex = int(rng.integers(0, len(seqs))) if seqs and rng.random() < 0.4 else -1
                hit = store.find_donor(q, tuple(seqs[ex]) if ex >= 0 else None)
                res = -1 if hit is None else next(i for i, t in enumerate(seqs) if tuple(t) == hit.token_ids)
                sim = float(np.dot(hit.embedding, q / (np.linalg.norm(q) + 1e-10))) if hit is not None else 0.0
                ops.append(1), seq_id.append(ex), embs.append(q), excl.append(ex)
                result.append(res), result_sim.append(sim)
                continue
            if seqs and rng.random() < 0.15:  # re-add an existing sequence: moves it to the end
                sid = int(rng.integers(0, len(seqs)))
                emb = rng.standard_normal(dim).astype(np.float32)
            else:
                toks = [int(x) for x in rng.integers(0, 50000, int(rng.integers(200, 400)))]
                if seqs and rng.random() < 0.1:  # same first 256 ids as an earlier sequence
                    toks = seqs[-1][:256] + toks[:50]
                seqs.append(toks)
                sid = len(seqs) - 1
                emb = (centers[int(rng.integers(0, 6))] + 0.3 * rng.standard_normal(dim)).astype(np.float32)
                if rng.random() < 0.15 and len(embs):  # an exactly tied embedding
                    emb = embs[-1].copy()
            store.add_donor(tuple(seqs[sid]), emb)
            ops.append(0), seq_id.append(sid), embs.append(emb), excl.append(-1)
            result.append(-2), result_sim.append(0.0)
        lens = np.array([len(t) for t in seqs], np.int64)
        flat = np.array([x for t in seqs for x in t], np.int32)
        save(name, op=np.array(ops, np.int64), seq=np.array(seq_id, np.int64), vec=np.stack(embs),
             result=np.array(result, np.int64), result_sim=np.array(result_sim, np.float64),
             seq_lens=lens, seq_tokens=flat, max_entries=max_entries, min_similarity=min_sim)

    radix_case("radix_store", 51, 400, 40, 0.6)
    print("wrote", sorted(p.name for p in HERE.glob("*.npz")), "plans.json")
    return 0


if __name__ == "__main__":
    sys.exit(main())
