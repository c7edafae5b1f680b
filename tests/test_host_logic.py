"""Host-side logic that needs no GPU: partial-attention plans against the
reference's outputs, plan flattening, layout helpers, pair preprocessing and
the module aliasing of ``semblend_b200.compat``."""

from __future__ import annotations

import json
import sys

import numpy as np
import pytest
import torch

from semblend_b200 import _rows, compat
from semblend_b200 import partial_attention as pa
from semblend_b200.rope_correction import _host_pairs, _last_per_target
from tests.helpers import GOLDEN


@pytest.fixture(scope="module")
def plans():
    return json.loads((GOLDEN / "plans.json").read_text())


def _build(entry):
    a = entry["args"]
    if entry["kind"] == "single":
        return pa.build_attention_plan(a["donor_id"], a["target_len"], a["donor_len"], a["copy_positions"],
                                       a["placeholder_positions"], a["slot_actions"], a["layer_hints"],
                                       num_layers=a["num_layers"])
    return pa.build_multi_donor_attention_plan(a["target_len"], a["slot_actions"], a["layer_hints"],
                                               num_layers=a["num_layers"])


def test_plans_match_reference(plans):
    for entry in plans:
        plan = _build(entry)
        assert plan.num_reuse_positions == entry["num_reuse"]
        assert plan.num_partial_positions == entry["num_partial"]
        assert plan.num_full_layers == entry["num_full_layers"]
        assert plan.computation_ratio == pytest.approx(entry["computation_ratio"], abs=0)
        if entry["kind"] == "multi":
            assert plan.donor_len == entry["donor_len"] and plan.donor_id == entry["donor_id"]
            assert [list(x) for x in plan.donor_map] == entry["donor_map"]
        for layer, (m, pairs) in enumerate(zip(entry["masks"], entry["pairs"])):
            assert pa.compute_attention_mask(plan, layer).tolist() == m
            assert [list(p) for p in pa.compute_donor_kv_indices(plan, layer)] == pairs


def test_plan_arrays_agree_with_per_layer_functions(plans):
    for entry in plans:
        plan = _build(entry)
        arr = pa.plan_arrays(plan)
        for layer in range(len(plan.layer_masks)):
            if arr.recompute_layers[layer]:
                assert pa.compute_attention_mask(plan, layer).all()
                assert pa.compute_donor_kv_indices(plan, layer) == []
            else:
                assert np.array_equal(pa.compute_attention_mask(plan, layer), arr.compute_mask)
                got = list(zip(arr.donor_positions.tolist(), arr.target_positions.tolist()))
                assert got == [tuple(p) for p in pa.compute_donor_kv_indices(plan, layer)]


def test_layout_detection_and_geometry():
    assert _rows.detect_layout(torch.empty(2, 100, 16, 4, 128)) == "vllm"
    assert _rows.detect_layout(torch.empty(100, 2, 4, 16, 128)) == "canonical"
    assert _rows.paged_geometry((2, 100, 16, 4, 128), "vllm") == (100, 4, 16, 128)
    assert _rows.paged_geometry((100, 2, 16, 4, 128), "trtllm") == (100, 4, 16, 128)
    with pytest.raises(ValueError):
        _rows.paged_geometry((100, 3, 4, 16, 128), "canonical")
    with pytest.raises(ValueError):
        _rows.resolve_layout(torch.empty(1), "nonsense")


def test_pair_preprocessing():
    pairs = _host_pairs([(1, 5), (2, 6), (3, 5), (4, 7)])
    assert pairs.shape == (4, 2)
    kept = _last_per_target(pairs)
    assert kept.tolist() == [[2, 6], [3, 5], [4, 7]]  # the last pair for target 5 wins, order kept
    assert _host_pairs([]).shape == (0, 2)
    with pytest.raises(ValueError):
        _host_pairs([(1, 2, 3)])


def test_compat_install_aliases_reference_names():
    saved = {k: v for k, v in sys.modules.items() if k.split(".")[0] in compat.PARENTS}
    try:
        done = compat.install()
        from semblend_core.rope_correction import rope_correct_scatter_paged
        from synapse_kv_connector.donor_store import DonorStore

        assert rope_correct_scatter_paged.__module__ == "semblend_b200.rope_correction"
        assert DonorStore.__module__ == "semblend_b200.donor_store"
        assert done["semblend_core.triton_kernels"] == "semblend_b200.triton_kernels"
        from synapse_kv_connector.cagra_donor_store import CAGRADonorStore, make_donor_store

        assert issubclass(CAGRADonorStore, DonorStore) and make_donor_store.__module__ == "semblend_b200.cagra_donor_store"
        compat.uninstall()
        assert "semblend_core.rope_correction" not in sys.modules
        assert "synapse_kv_connector.cagra_donor_store" not in sys.modules
    finally:
        for k in [k for k in sys.modules if k.split(".")[0] in compat.PARENTS]:
            del sys.modules[k]
        sys.modules.update(saved)


def test_reference_callers_bind_the_drop_in():
    """With a reference checkout named by $SEMBLEND_REFERENCE, the reference's
    own callers import on top of ``compat.install()`` and bind the B200
    functions; ``patch_sglang`` swaps the SGLang donor store."""
    from tests.golden.make_golden import REF

    if REF is None or not (REF / "synapse_kv_connector").is_dir():
        pytest.skip("no reference checkout named by SEMBLEND_REFERENCE")
    import importlib

    saved = {k: v for k, v in sys.modules.items() if k.split(".")[0] in compat.PARENTS + ("semblend",)}
    sys.path.insert(0, str(REF))
    try:
        compat.install()
        ap = importlib.import_module("synapse_kv_connector.attention_patch")
        for name in ("partial_prefill_attention", "scatter_donor_kv", "partial_prefill", "compute_attention_mask"):
            assert getattr(ap, name).__module__.startswith("semblend_b200."), name
        for mod in ("synapse_kv_connector.model_runner_hook", "synapse_kv_connector.semblend_connector",
                    "synapse_kv_connector.pipeline", "semblend.integration.trtllm.pytorch_backend"):
            importlib.import_module(mod)  # their hot-path imports resolve through the aliases at call time
        from semblend_b200.radix_store import RadixDonorStore

        assert compat.patch_sglang()
        rb = importlib.import_module("semblend.integration.sglang.radix_backend")
        assert rb._SemBlendDonorStore is RadixDonorStore
        compat.uninstall()
    finally:
        sys.path.remove(str(REF))
        for k in [k for k in sys.modules if k.split(".")[0] in compat.PARENTS + ("semblend",)]:
            del sys.modules[k]
        sys.modules.update(saved)


def test_layer_results_shared_and_invalidated():
    """Partial layers of one plan share one walk of their position list; a
    layer list changed afterwards is walked again (results always equal a
    fresh walk)."""
    acts = [{"action": "copy_from_donor", "targetPos": i, "donorPos": 100 + i} for i in range(8)]
    acts += [{"action": "placeholder", "targetPos": i} for i in range(8, 12)]
    plan = pa.build_attention_plan("d", 12, 200, list(range(8)), list(range(8, 12)), acts,
                                   [{"recomputeAll": False}, {"recomputeAll": True}], num_layers=4)
    want_pairs = [(100 + i, i) for i in range(8)]
    for layer in (0, 2, 3):
        assert pa.compute_donor_kv_indices(plan, layer) == want_pairs
        assert pa.compute_attention_mask(plan, layer).tolist() == [False] * 8 + [True] * 4
    assert pa.compute_donor_kv_indices(plan, 1) == [] and pa.compute_attention_mask(plan, 1).all()
    # returned objects are copies: mutating them does not leak into later calls
    pa.compute_donor_kv_indices(plan, 0).clear()
    pa.compute_attention_mask(plan, 0)[:] = True
    assert pa.compute_donor_kv_indices(plan, 2) == want_pairs
    assert pa.compute_attention_mask(plan, 2).sum() == 4
    # a caller edits one layer's list: that layer is recomputed, the others keep theirs
    plan.layer_masks[3].position_masks[0] = pa.PositionMask(target_pos=0, mode=pa.AttentionMode.PARTIAL)
    assert pa.compute_donor_kv_indices(plan, 3) == want_pairs[1:]
    assert pa.compute_attention_mask(plan, 3).tolist() == [True] + [False] * 7 + [True] * 4
    assert pa.compute_donor_kv_indices(plan, 0) == want_pairs


def test_position_mapping_host_classes():
    """The host PositionMapping / MultiDonorPositionMapping keep the
    reference's fields and properties (pipeline.py:62-80,
    multi_donor_types.py:50-78); the device form needs a CUDA device."""
    from semblend_b200 import _lib
    from semblend_b200.position_mapping import DevicePositionMapping, MultiDonorPositionMapping, PositionMapping

    assert PositionMapping().num_pairs == 0 and not PositionMapping().needs_correction
    pm = PositionMapping([0, 1, 2, 3], [2, 3, 0, 1])
    assert pm.num_pairs == 4 and pm.needs_correction
    md = MultiDonorPositionMapping(("x", "y", "x"), (0, 1, 2), (0, 5, 2))
    assert md.needs_correction and md.num_pairs == 3
    sub = md.for_donor("x")
    assert sub.donor_positions == (0, 2) and sub.target_positions == (0, 2) and not sub.needs_correction
    with pytest.raises(_lib.NativeLibraryError):
        DevicePositionMapping(torch.zeros(2, dtype=torch.int32), torch.zeros(2, dtype=torch.int32), 2)


def test_token_set_alignment_matches_reference():
    """The no-rapidfuzz fallback of compute_alignment restated for the store
    (alignment.py:945-1020) gives the reference's slot actions."""
    from tests.golden.make_golden import REF

    if REF is None or not (REF / "semblend_core").is_dir():
        pytest.skip("no reference checkout named by SEMBLEND_REFERENCE")
    sys.path.insert(0, str(REF))
    try:
        import importlib

        ref = importlib.import_module("semblend_core.alignment")
        from semblend_b200.alignment import _token_set_alignment

        rng = np.random.default_rng(5)
        for n_d, n_t, vocab in ((300, 250, 50), (10, 40, 8), (0, 5, 3), (64, 0, 9)):
            d = rng.integers(0, vocab, n_d).tolist()
            t = rng.integers(0, vocab, n_t).tolist()
            a, b = _token_set_alignment(d, t), ref._token_set_alignment(d, t)
            assert a.reuse_ratio == b.reuse_ratio and a.edit_distance == b.edit_distance
            assert [(x.action, x.target_pos, x.donor_pos) for x in a.slot_actions] == \
                [(str(x.action.value) if hasattr(x.action, "value") else x.action, x.target_pos, x.donor_pos)
                 for x in b.slot_actions]
    finally:
        sys.path.remove(str(REF))
        for k in [k for k in sys.modules if k.split(".")[0] == "semblend_core"]:
            del sys.modules[k]
