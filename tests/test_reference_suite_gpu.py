"""The reference's own hot-path tests, restated, run on the B200 through the
drop-in names.

``compat.install()`` registers this library under the reference's module
names (``synapse_kv_connector.rope_correction`` and friends); every test below
imports the function under test by that name, as the reference's test does,
and feeds it CUDA tensors (the reference's tests pick CUDA when it is
available, synapse_kv_connector/tests/test_triton_kernels.py:37-39).  The
shapes, inputs and assertions follow the test each case cites (file:line in
synapse_kv_connector/tests/); the helpers are written anew.  The reference
checkout is not needed: nothing here imports it.
"""

from __future__ import annotations

import math
import sys

import numpy as np
import pytest
import torch

from semblend_b200 import compat

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


@pytest.fixture(autouse=True, scope="module")
def drop_in():
    saved = {k: v for k, v in sys.modules.items() if k.split(".")[0] in compat.PARENTS}
    compat.install()
    yield
    compat.uninstall()
    for k in [k for k in sys.modules if k.split(".")[0] in compat.PARENTS]:
        del sys.modules[k]
    sys.modules.update(saved)


def rope_at(x: torch.Tensor, positions, head_dim: int, base: float = 10000.0) -> torch.Tensor:
    """Interleaved RoPE of the rows of ``x [..., S, D]`` at ``positions`` (one
    per row), fp32 on the CPU: the from-scratch ground truth the reference's
    tests compare against (test_rope_correction.py:14-31)."""
    inv = 1.0 / (base ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
    out = x.detach().float().cpu().clone()
    for i, p in enumerate(torch.as_tensor(positions).tolist()):
        th = float(p) * inv
        c, s = torch.cos(th), torch.sin(th)
        ev, od = out[..., i, 0::2].clone(), out[..., i, 1::2].clone()
        out[..., i, 0::2] = ev * c - od * s
        out[..., i, 1::2] = ev * s + od * c
    return out.to(x.dtype)


def i32(*v):
    return torch.tensor(v, dtype=torch.int32, device=DEV)


def close(a, b, atol, rtol):
    torch.testing.assert_close(a.detach().float().cpu(), b.detach().float().cpu(), atol=atol, rtol=rtol)


# ----------------------------------------------------------------------------
# test_rope_correction.py
# ----------------------------------------------------------------------------
class TestRoPECorrection:
    def test_identity_no_delta(self):  # :37-47
        from synapse_kv_connector.rope_correction import rope_correct_k

        k = torch.randn(4, 8, 128, dtype=torch.float16, device=DEV)
        p = i32(0, 3, 7)
        close(rope_correct_k(k, p, p, head_dim=128), k, 1e-3, 1e-3)

    def test_exact_correction_single_position(self):  # :49-83
        from synapse_kv_connector.rope_correction import rope_correct_k

        raw = torch.randn(4, 1, 128)
        padded = torch.zeros(4, 11, 128)
        padded[:, 5] = rope_at(raw, [5], 128)[:, 0]
        out = rope_correct_k(padded.to(DEV), i32(5), i32(10), head_dim=128)
        close(out[:, 5], rope_at(raw, [10], 128)[:, 0], 1e-4, 1e-4)

    def test_exact_correction_reorder(self):  # :85-117
        from synapse_kv_connector.rope_correction import rope_correct_k

        raw = torch.randn(4, 4, 64)
        dpos, tpos = [0, 1, 2, 3], [2, 3, 0, 1]
        out = rope_correct_k(rope_at(raw, dpos, 64).to(DEV), i32(*dpos), i32(*tpos), head_dim=64)
        gt = rope_at(raw, tpos, 64)
        for i in range(4):
            close(out[:, i], gt[:, i], 1e-3, 1e-3)

    def test_negative_delta(self):  # :119-144
        from synapse_kv_connector.rope_correction import rope_correct_k

        raw = torch.randn(2, 1, 64)
        padded = torch.zeros(2, 101, 64)
        padded[:, 100] = rope_at(raw, [100], 64)[:, 0]
        out = rope_correct_k(padded.to(DEV), i32(100), i32(50), head_dim=64)
        close(out[:, 100], rope_at(raw, [50], 64)[:, 0], 1e-3, 1e-3)

    def test_large_sequence(self):  # :146-160
        from synapse_kv_connector.rope_correction import rope_correct_k

        k = torch.randn(4, 8192, 128, dtype=torch.float16, device=DEV)
        # distinct donor rows (a row rotated twice in one call is this library's documented deviation)
        d = torch.randperm(8192, device=DEV)[:100].to(torch.int32)
        t = torch.randint(0, 8192, (100,), dtype=torch.int32, device=DEV)
        out = rope_correct_k(k, d, t, head_dim=128)
        assert out.shape == k.shape and out.dtype == k.dtype

    def test_v_unchanged(self):  # :162-191
        from synapse_kv_connector.rope_correction import rope_correct_scatter_paged

        cache = torch.zeros(4, 2, 2, 16, 64, device=DEV)
        donor = torch.randn(2, 2, 32, 64, device=DEV)
        rope_correct_scatter_paged(cache, donor, torch.arange(4, dtype=torch.int32, device=DEV), i32(0, 1, 2),
                                   i32(5, 10, 15))
        for dp, tp in zip([0, 1, 2], [5, 10, 15]):
            close(cache[tp // 16, 1, :, tp % 16], donor[1, :, dp], 1e-6, 1e-6)

    def test_paged_scatter_k_corrected(self):  # :193-233
        from synapse_kv_connector.rope_correction import rope_correct_scatter_paged

        cache = torch.zeros(4, 2, 2, 16, 64, device=DEV)
        raw = torch.randn(2, 1, 64)
        donor = torch.zeros(2, 2, 32, 64)
        donor[0, :, 3] = rope_at(raw, [3], 64)[:, 0]
        donor[1] = torch.randn(2, 32, 64)
        rope_correct_scatter_paged(cache, donor.to(DEV), torch.arange(4, dtype=torch.int32, device=DEV), i32(3),
                                   i32(7))
        close(cache[0, 0, :, 7], rope_at(raw, [7], 64)[:, 0], 1e-3, 1e-3)

    def test_permute_paged_kv(self):  # :235-264
        from synapse_kv_connector.rope_correction import permute_paged_kv_with_rope

        cache = torch.randn(2, 2, 2, 16, 64, device=DEV)
        v0, v1 = cache[0, 1, :, 0].clone(), cache[0, 1, :, 1].clone()
        permute_paged_kv_with_rope(cache, torch.arange(2, dtype=torch.int32, device=DEV), [(0, 1), (1, 0)])
        close(cache[0, 1, :, 1], v0, 1e-6, 1e-6)
        close(cache[0, 1, :, 0], v1, 1e-6, 1e-6)

    def test_rope_correction_is_cheap(self):  # :266-288 (the reference's budget is 5 s on a CPU)
        import time

        from synapse_kv_connector.rope_correction import rope_correct_k

        k = torch.randn(4, 8192, 128, device=DEV)
        d = torch.arange(8192, dtype=torch.int32, device=DEV)
        t = torch.roll(d, 256)
        rope_correct_k(k, d[:10], t[:10], head_dim=128)
        torch.cuda.synchronize()
        t0 = time.monotonic()
        rope_correct_k(k, d, t, head_dim=128)
        torch.cuda.synchronize()
        assert (time.monotonic() - t0) * 1000 < 5000


class TestRoPECorrectionComposition:
    def test_composition_identity(self):  # :294-323
        from synapse_kv_connector.rope_correction import rope_correct_k

        k = torch.randn(2, 10, 64, device=DEV)
        s1 = rope_correct_k(k, i32(3), i32(8), head_dim=64)
        s2 = rope_correct_k(s1, i32(3), i32(3 - (8 - 3)), head_dim=64)
        close(s2[:, 3], k[:, 3], 1e-3, 1e-3)

    @pytest.mark.parametrize("base", [500.0, 10000.0, 1000000.0])
    def test_different_rope_bases(self, base):  # :325-353
        from synapse_kv_connector.rope_correction import rope_correct_k

        raw = torch.randn(2, 1, 32)
        padded = torch.zeros(2, 11, 32)
        padded[:, 0] = rope_at(raw, [0], 32, base)[:, 0]
        out = rope_correct_k(padded.to(DEV), i32(0), i32(10), head_dim=32, rope_base=base)
        close(out[:, 0], rope_at(raw, [10], 32, base)[:, 0], 1e-3, 1e-3)


class TestPositionMapping:
    """test_rope_correction.py:356-449 against this library's PositionMapping
    and its device form (the reference's class lives in its pipeline module)."""

    def test_position_map_needs_correction(self):  # :359-375
        from semblend_b200.position_mapping import DevicePositionMapping, PositionMapping

        assert not PositionMapping([0, 1, 2], [0, 1, 2]).needs_correction
        assert PositionMapping([0, 1, 2], [5, 10, 15]).needs_correction
        assert not DevicePositionMapping.from_host(PositionMapping([0, 1, 2], [0, 1, 2]), DEV).needs_correction
        assert DevicePositionMapping.from_host(PositionMapping([0, 1, 2], [5, 10, 15]), DEV).needs_correction

    def test_position_map_to_rope_correction(self):  # :377-410
        from semblend_b200.position_mapping import DevicePositionMapping, PositionMapping
        from synapse_kv_connector.rope_correction import rope_correct_k

        raw = torch.randn(2, 1, 64)
        padded = torch.zeros(2, 10, 64)
        padded[:, 3] = rope_at(raw, [3], 64)[:, 0]
        pm = DevicePositionMapping.from_host(PositionMapping([3], [7]), DEV)
        out = rope_correct_k(padded.to(DEV), pm.donor_positions, pm.target_positions, head_dim=64)
        close(out[:, 3], rope_at(raw, [7], 64)[:, 0], 1e-3, 1e-3)

    def test_reorder_position_map(self):  # :412-449
        from semblend_b200.position_mapping import DevicePositionMapping, PositionMapping
        from synapse_kv_connector.rope_correction import rope_correct_k

        pm = PositionMapping([0, 1, 2, 3], [2, 3, 0, 1])
        assert pm.needs_correction and pm.num_pairs == 4
        dm = DevicePositionMapping.from_host(pm, DEV)
        assert dm.num_pairs == 4 and dm.to_host() == pm
        raw = torch.randn(2, 4, 32)
        out = rope_correct_k(rope_at(raw, [0, 1, 2, 3], 32).to(DEV), dm.donor_positions, dm.target_positions,
                             head_dim=32)
        gt = rope_at(raw, [2, 3, 0, 1], 32)
        for i in range(4):
            close(out[:, i], gt[:, i], 1e-3, 1e-3)


class TestNoPePermutation:
    @staticmethod
    def cache(H, D, S, bs=16):  # :478-488
        nb = (S + bs - 1) // bs + 2
        return (torch.zeros(nb, 2, H, bs, D, dtype=torch.float16, device=DEV),
                torch.arange((S + bs - 1) // bs, dtype=torch.int32, device=DEV))

    @staticmethod
    def rope1(raw, pos, D, base=10000.0):  # :490-505 on one row per head
        return rope_at(raw.unsqueeze(1), [pos], D, base)[:, 0]

    def test_nope_identity_no_shift(self):  # :492-506
        from synapse_kv_connector.rope_correction import nope_permute_paged_kv

        raw = torch.randn(4, 64)
        k5 = self.rope1(raw, 5, 64)
        kv, bt = self.cache(4, 64, 32)
        kv[0, 0, :, 5] = k5.half().to(DEV)
        nope_permute_paged_kv(kv, bt, permutation=[(5, 5)], rope_base=10000.0)
        close(kv[0, 0, :, 5], k5, 5e-3, 5e-3)

    def test_nope_matches_delta_arbitrary_shift(self):  # :508-547
        from synapse_kv_connector.rope_correction import nope_permute_paged_kv, permute_paged_kv_with_rope

        raw = torch.randn(4, 64)
        ks = self.rope1(raw, 3, 64).half().to(DEV)
        kd, bt = self.cache(4, 64, 64)
        kn, _ = self.cache(4, 64, 64)
        kd[0, 0, :, 3] = ks
        kn[0, 0, :, 3] = ks
        permute_paged_kv_with_rope(kd, bt, permutation=[(3, 17)], rope_base=10000.0)
        nope_permute_paged_kv(kn, bt, permutation=[(3, 17)], rope_base=10000.0)
        close(kn[1, 0, :, 1], kd[1, 0, :, 1], 5e-3, 5e-3)

    def test_nope_matches_fresh_rope_at_target(self):  # :549-575
        from synapse_kv_connector.rope_correction import nope_permute_paged_kv

        raw = torch.randn(4, 128)
        kv, bt = self.cache(4, 128, 64)
        kv[0, 0, :, 7] = self.rope1(raw, 7, 128).half().to(DEV)
        nope_permute_paged_kv(kv, bt, permutation=[(7, 23)], rope_base=10000.0)
        close(kv[1, 0, :, 7], self.rope1(raw, 23, 128), 1e-2, 1e-2)

    def test_nope_v_cache_unchanged(self):  # :577-592
        from synapse_kv_connector.rope_correction import nope_permute_paged_kv

        kv, bt = self.cache(4, 64, 32)
        v = torch.randn(4, 64, dtype=torch.float16, device=DEV)
        kv[0, 1, :, 2] = v
        nope_permute_paged_kv(kv, bt, permutation=[(2, 10)], rope_base=10000.0)
        assert torch.equal(kv[0, 1, :, 10], v)

    @pytest.mark.parametrize("delta", [0, 1, 5, 50, 100, 256, 1000])
    def test_nope_delta_correction_parity(self, delta):  # :594-637
        from synapse_kv_connector.rope_correction import nope_permute_paged_kv, permute_paged_kv_with_rope

        src, tgt = 5, 5 + delta
        raw = torch.randn(8, 128)
        ks = self.rope1(raw, src, 128).half().to(DEV)
        caches = []
        for _ in range(2):
            kv, bt = self.cache(8, 128, max(tgt + 16, 128))
            kv[0, 0, :, src] = ks
            caches.append((kv, bt))
        permute_paged_kv_with_rope(caches[0][0], caches[0][1], [(src, tgt)], rope_base=10000.0)
        nope_permute_paged_kv(caches[1][0], caches[1][1], [(src, tgt)], rope_base=10000.0)
        close(caches[1][0][tgt // 16, 0, :, tgt % 16], caches[0][0][tgt // 16, 0, :, tgt % 16], 5e-3, 5e-3)


# ----------------------------------------------------------------------------
# test_triton_kernels.py
# ----------------------------------------------------------------------------
def kv_flat(L, H, S, D):  # :42-55
    return torch.zeros(L, 2, H, S, D, dtype=torch.float16, device=DEV)


def donor_flat(L, H, S, D):  # :58-71
    return torch.randn(L, 2, H, S, D, dtype=torch.float16, device=DEV)


class TestScatterDonorKv:
    def test_basic_scatter(self):  # :82-107
        from synapse_kv_connector.triton_kernels import scatter_donor_kv

        t, d = kv_flat(2, 4, 16, 32), donor_flat(2, 4, 8, 32)
        out = scatter_donor_kv(t, d, i32(0, 2, 4, 6), i32(1, 3, 7, 12))
        for dp, tp in zip([0, 2, 4, 6], [1, 3, 7, 12]):
            assert torch.equal(out[:, :, :, tp], d[:, :, :, dp])
        for p in [0, 2, 4]:
            assert torch.all(out[:, :, :, p] == 0)

    def test_empty_pairs(self):  # :109-117
        from synapse_kv_connector.triton_kernels import scatter_donor_kv

        e = torch.zeros(0, dtype=torch.int32, device=DEV)
        assert torch.all(scatter_donor_kv(kv_flat(1, 2, 8, 16), donor_flat(1, 2, 4, 16), e, e) == 0)

    def test_single_pair(self):  # :119-135
        from synapse_kv_connector.triton_kernels import scatter_donor_kv

        t, d = kv_flat(1, 1, 4, 8), donor_flat(1, 1, 2, 8)
        scatter_donor_kv(t, d, i32(1), i32(3))
        assert torch.equal(t[0, :, 0, 3], d[0, :, 0, 1])

    def test_full_sequence_scatter(self):  # :137-147
        from synapse_kv_connector.triton_kernels import scatter_donor_kv

        t, d = kv_flat(2, 4, 16, 32), donor_flat(2, 4, 16, 32)
        p = torch.arange(16, dtype=torch.int32, device=DEV)
        scatter_donor_kv(t, d, p, p)
        assert torch.equal(t, d)

    def test_multi_layer_consistency(self):  # :149-171
        from synapse_kv_connector.triton_kernels import scatter_donor_kv

        t, d = kv_flat(8, 4, 32, 64), donor_flat(8, 4, 16, 64)
        scatter_donor_kv(t, d, i32(0, 5, 10), i32(2, 8, 20))
        for layer in range(8):
            for dp, tp in zip([0, 5, 10], [2, 8, 20]):
                assert torch.equal(t[layer, :, :, tp], d[layer, :, :, dp])


class TestScatterDonorKvPaged:
    @staticmethod
    def paged(nb, H, bs, D):  # :179-190
        return torch.zeros(nb, 2, H, bs, D, dtype=torch.float16, device=DEV)

    @staticmethod
    def donor(H, S, D):  # :192-206
        return torch.randn(2, H, S, D, dtype=torch.float16, device=DEV)

    def test_basic_paged_scatter(self):  # :208-240
        from synapse_kv_connector.triton_kernels import scatter_donor_kv_paged

        kv, d = self.paged(8, 2, 4, 16), self.donor(2, 8, 16)
        scatter_donor_kv_paged(kv, d, i32(3, 5), i32(0, 4), i32(1, 5))
        assert torch.equal(kv[3, :, :, 1], d[:, :, 0])
        assert torch.equal(kv[5, :, :, 1], d[:, :, 4])

    def test_empty_pairs(self):  # :242-251
        from synapse_kv_connector.triton_kernels import scatter_donor_kv_paged

        e = torch.zeros(0, dtype=torch.int32, device=DEV)
        assert torch.all(scatter_donor_kv_paged(self.paged(4, 2, 4, 8), self.donor(2, 4, 8), i32(0, 1), e, e) == 0)

    def test_multiple_positions_same_block(self):  # :253-278
        from synapse_kv_connector.triton_kernels import scatter_donor_kv_paged

        kv, d = self.paged(4, 2, 8, 16), self.donor(2, 8, 16)
        scatter_donor_kv_paged(kv, d, i32(2), i32(0, 1, 2), i32(0, 3, 7))
        for dp, tp in zip([0, 1, 2], [0, 3, 7]):
            assert torch.equal(kv[2, :, :, tp % 8], d[:, :, dp])

    def test_out_of_bounds_block_skipped(self):  # :280-303
        from synapse_kv_connector.triton_kernels import scatter_donor_kv_paged

        kv, d = self.paged(4, 1, 4, 8), self.donor(1, 4, 8)
        scatter_donor_kv_paged(kv, d, i32(1), i32(0, 1), i32(2, 8))
        assert torch.equal(kv[1, :, :, 2], d[:, :, 0])


class TestMaskedQkvProjection:
    def test_all_compute(self):  # :313-328
        from synapse_kv_connector.triton_kernels import masked_qkv_projection

        h = torch.randn(8, 32, dtype=torch.float16, device=DEV)
        w = torch.randn(48, 32, dtype=torch.float16, device=DEV)
        out = masked_qkv_projection(h, w, torch.ones(8, dtype=torch.bool, device=DEV))
        close(out, torch.nn.functional.linear(h.float(), w.float()), 1e-2, 1e-2)

    def test_all_reuse(self):  # :330-343
        from synapse_kv_connector.triton_kernels import masked_qkv_projection

        h = torch.randn(8, 32, dtype=torch.float16, device=DEV)
        w = torch.randn(48, 32, dtype=torch.float16, device=DEV)
        assert torch.all(masked_qkv_projection(h, w, torch.zeros(8, dtype=torch.bool, device=DEV)) == 0)

    def test_mixed_mask(self):  # :345-368
        from synapse_kv_connector.triton_kernels import masked_qkv_projection

        h = torch.randn(8, 32, dtype=torch.float16, device=DEV)
        w = torch.randn(48, 32, dtype=torch.float16, device=DEV)
        m = torch.tensor([True, False] * 4, device=DEV)
        out = masked_qkv_projection(h, w, m)
        for i in [1, 3, 5, 7]:
            assert torch.all(out[i] == 0)
        for i in [0, 2, 4, 6]:
            assert not torch.all(out[i] == 0)

    def test_with_bias(self):  # :370-388
        from synapse_kv_connector.triton_kernels import masked_qkv_projection

        h = torch.randn(4, 16, dtype=torch.float16, device=DEV)
        w = torch.randn(24, 16, dtype=torch.float16, device=DEV)
        b = torch.randn(24, dtype=torch.float16, device=DEV)
        out = masked_qkv_projection(h, w, torch.ones(4, dtype=torch.bool, device=DEV), qkv_bias=b)
        close(out, torch.nn.functional.linear(h.float(), w.float(), b.float()), 1e-2, 1e-2)


def causal_row(q, k, v, h, pos, scale):
    s = (q[h, pos:pos + 1].double() @ k[h, :pos + 1].double().T) * scale
    return (torch.softmax(s, dim=-1) @ v[h, :pos + 1].double()).squeeze(0)


class TestPartialPrefillAttention:
    def test_all_compute_matches_standard(self):  # :396-428
        from synapse_kv_connector.triton_kernels import partial_prefill_attention

        q, k, v = (torch.randn(2, 8, 16, device=DEV) for _ in range(3))
        sc = 1.0 / math.sqrt(16)
        out = partial_prefill_attention(q, k, v, torch.ones(8, dtype=torch.bool, device=DEV), sc)
        for h in range(2):
            for p in range(8):
                close(out[h, p], causal_row(q, k, v, h, p, sc), 1e-4, 1e-3)

    def test_reuse_positions_are_zero(self):  # :430-450
        from synapse_kv_connector.triton_kernels import partial_prefill_attention

        q, k, v = (torch.randn(2, 8, 16, device=DEV) for _ in range(3))
        out = partial_prefill_attention(q, k, v, torch.tensor([True, False] * 4, device=DEV))
        for p in [1, 3, 5, 7]:
            assert torch.all(out[:, p] == 0)

    def test_compute_positions_attend_to_full_context(self):  # :452-482
        from synapse_kv_connector.triton_kernels import partial_prefill_attention

        q, k, v = (torch.randn(1, 4, 8, device=DEV) for _ in range(3))
        out = partial_prefill_attention(q, k, v, torch.tensor([False, False, False, True], device=DEV))
        close(out[0, 3], causal_row(q, k, v, 0, 3, 1.0 / math.sqrt(8)), 1e-4, 1e-3)

    def test_empty_compute_mask(self):  # :484-495
        from synapse_kv_connector.triton_kernels import partial_prefill_attention

        q, k, v = (torch.randn(2, 4, 8, device=DEV) for _ in range(3))
        assert torch.all(partial_prefill_attention(q, k, v, torch.zeros(4, dtype=torch.bool, device=DEV)) == 0)


class TestPartialPrefill:
    @staticmethod
    def weights(H, D, hidden):
        return (torch.randn(3 * H * D, hidden, dtype=torch.float16, device=DEV),
                torch.randn(hidden, H * D, dtype=torch.float16, device=DEV))

    def run(self, S, hidden, H, D, L, Sd, dpos, tpos, mask):
        from synapse_kv_connector.triton_kernels import partial_prefill

        wq, wo = self.weights(H, D, hidden)
        donor = donor_flat(L, H, Sd, D)
        res = partial_prefill(hidden_states=torch.randn(S, hidden, dtype=torch.float16, device=DEV),
                              donor_kv=donor, qkv_weight=wq, output_projection=wo, donor_positions=dpos,
                              target_positions=tpos, compute_mask=mask, num_heads=H, head_dim=D)
        return res, donor

    def test_basic_partial_prefill(self):  # :504-561
        from synapse_kv_connector.triton_kernels import PartialPrefillResult

        m = torch.tensor([False] * 4 + [True] * 4, device=DEV)
        r, _ = self.run(8, 32, 4, 8, 2, 8, i32(0, 1, 2, 3), i32(0, 1, 2, 3), m)
        assert isinstance(r, PartialPrefillResult)
        assert r.positions_computed == 4 and r.positions_reused == 4 and abs(r.computation_ratio - 0.5) < 1e-6
        assert r.output.shape == (8, 32) and r.kv_cache.shape == (2, 2, 4, 8, 8)

    def test_full_reuse(self):  # :563-610
        p = torch.arange(4, dtype=torch.int32, device=DEV)
        r, _ = self.run(4, 16, 2, 8, 1, 4, p, p, torch.zeros(4, dtype=torch.bool, device=DEV))
        assert r.positions_computed == 0 and r.positions_reused == 4 and r.computation_ratio == 0.0

    def test_no_reuse(self):  # :612-652
        e = torch.zeros(0, dtype=torch.int32, device=DEV)
        r, _ = self.run(4, 16, 2, 8, 1, 4, e, e, torch.ones(4, dtype=torch.bool, device=DEV))
        assert r.positions_computed == 4 and r.positions_reused == 0 and r.computation_ratio == 1.0

    def test_sparse_reuse_pattern(self):  # :654-717
        dpos, tpos = i32(0, 2, 4, 6, 8), i32(0, 3, 6, 9, 12)
        m = torch.ones(16, dtype=torch.bool, device=DEV)
        m[tpos.long()] = False
        r, donor = self.run(16, 32, 4, 8, 2, 10, dpos, tpos, m)
        assert r.positions_reused == 5 and r.positions_computed == 11
        for dp, tp in zip(dpos.tolist(), tpos.tolist()):
            assert torch.equal(r.kv_cache[:, :, :, tp], donor[:, :, :, dp])

    def test_timing_reported(self):  # :719-763
        p = torch.arange(16, dtype=torch.int32, device=DEV)
        m = torch.ones(64, dtype=torch.bool, device=DEV)
        m[:16] = False
        r, _ = self.run(64, 128, 8, 16, 4, 32, p, p, m)
        assert r.total_time_ms > 0 and r.scatter_time_ms >= 0


# ----------------------------------------------------------------------------
# test_donor_store.py (the embedding store; its SimHash tests are outside the hot path)
# ----------------------------------------------------------------------------
def make_store(n, max_entries=1000, dim=384, seed=0):  # :89-111
    from synapse_kv_connector.donor_store import DonorNode, DonorStore

    rng = np.random.default_rng(seed)
    store = DonorStore(max_entries=max_entries, embedding_dim=dim, min_similarity=0.5, device=DEV)
    for i in range(n):
        e = rng.standard_normal(dim).astype(np.float32)
        store.add_donor(DonorNode(f"req-{i}", list(range(i * 10, i * 10 + 100)), e / np.linalg.norm(e), float(i)))
    return store


class TestDonorStore:
    def test_donor_store_empty(self):  # :115-122
        assert make_store(0).find_donor(query_embedding=np.zeros(384, np.float32), query_tokens=[1, 2, 3]) is None

    def test_donor_store_add_and_find(self):  # :125-158
        from synapse_kv_connector.donor_store import DonorNode

        store = make_store(0)
        e = np.random.default_rng(1).standard_normal(384).astype(np.float32)
        e /= np.linalg.norm(e)
        store.add_donor(DonorNode("donor-1", list(range(100)), e.copy(), 1.0))
        q = list(range(100))
        q[50] = 999
        r = store.find_donor(query_embedding=e, query_tokens=q, min_reuse_ratio=0.5)
        assert r is not None and r.donor.request_id == "donor-1" and r.similarity > 0.9
        assert r.alignment.reuse_ratio >= 0.3

    def test_donor_store_lru_eviction(self):  # :161-164
        assert make_store(100, max_entries=50).size == 50

    def test_donor_store_duplicate_add(self):  # :167-180
        from synapse_kv_connector.donor_store import DonorNode

        store = make_store(0)
        node = DonorNode("dup", [1, 2, 3], np.zeros(384, np.float32), 1.0)
        store.add_donor(node)
        store.add_donor(node)
        assert store.size == 1

    def test_donor_store_no_self_match(self):  # :183-205
        from synapse_kv_connector.donor_store import DonorNode

        store = make_store(0)
        e = np.random.default_rng(2).standard_normal(384).astype(np.float32)
        e /= np.linalg.norm(e)
        store.add_donor(DonorNode("self", list(range(100)), e.copy(), 1.0))
        assert store.find_donor(query_embedding=e, query_tokens=list(range(100))) is None

    def test_donor_store_1k_entries(self):  # :208-221
        import time

        store = make_store(1000)
        e = np.random.default_rng(3).standard_normal(384).astype(np.float32)
        t0 = time.monotonic()
        store.find_donor(query_embedding=e / np.linalg.norm(e), query_tokens=list(range(50)))
        assert (time.monotonic() - t0) * 1000 < 500

    def test_donor_store_no_embedding_fallback(self):  # :224-246
        from synapse_kv_connector.donor_store import DonorNode

        store = make_store(0)
        store.add_donor(DonorNode("no-emb", list(range(100)), None, 1.0))
        q = list(range(100))
        q[50] = 999
        assert store.find_donor(query_embedding=None, query_tokens=q) is None
