"""The product has no CPU path: every public entry point given host tensors (or
run without a CUDA device) raises NativeLibraryError instead of computing on
the CPU.  Runs without a GPU."""

from __future__ import annotations

import pytest
import torch

from semblend_b200 import _lib
from semblend_b200 import alignment as al
from semblend_b200 import rope_correction as rc
from semblend_b200 import search as se
from semblend_b200 import triton_kernels as tk

H, D, BS, NB, S = 2, 64, 16, 8, 64


def _inputs():
    g = torch.Generator().manual_seed(0)
    cache = torch.zeros(NB, 2, H, BS, D)
    donor = torch.randn(2, H, S, D, generator=g)
    bt = torch.arange(4, dtype=torch.int32)
    pos = torch.arange(10, dtype=torch.int32)
    q = torch.randn(H, S, D, generator=g)
    mask = torch.zeros(S, dtype=torch.bool)
    mask[-5:] = True
    return cache, donor, bt, pos, q, mask


def _host_tensor_calls():
    cache, donor, bt, pos, q, mask = _inputs()
    return {
        "rope_correct_scatter_paged": lambda: rc.rope_correct_scatter_paged(cache, donor, bt, pos, pos),
        "rope_correct_k": lambda: rc.rope_correct_k(donor[0], pos, pos),
        "inject_donors": lambda: rc.inject_donors(cache[None], [rc.DonorInjection(donor[None], bt, pos, pos)]),
        "scatter_donor_kv": lambda: tk.scatter_donor_kv(torch.zeros(1, 2, H, S, D), donor[None].clone(), pos, pos),
        "scatter_donor_kv_paged": lambda: tk.scatter_donor_kv_paged(cache, donor, bt, pos, pos),
        "masked_qkv_projection": lambda: tk.masked_qkv_projection(torch.randn(S, 32), torch.randn(96, 32), mask),
        "partial_prefill_attention": lambda: tk.partial_prefill_attention(q, q, q, mask),
        "gqa_partial_attention": lambda: tk.gqa_partial_attention(
            q[None], q[None], q[None], torch.zeros(1, 5, dtype=torch.int32), torch.ones(1, dtype=torch.int32),
            torch.zeros_like(q[None])),
        "mask_to_rows": lambda: tk.mask_to_rows(mask[None]),
        "chunk_digests": lambda: al.chunk_digests(torch.arange(512), 256),
        "cosine_topk": lambda: se.cosine_topk(torch.randn(10, 64), torch.randn(10, 64).half(), None, torch.zeros(2),
                                              torch.randn(2, 64), 2, 0.5),
    }


@pytest.mark.parametrize("name", sorted(_host_tensor_calls()))
def test_host_tensors_raise(name):
    with pytest.raises(_lib.NativeLibraryError):
        _host_tensor_calls()[name]()


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the behaviour without a CUDA device")
@pytest.mark.parametrize("name", ["chunk_alignment", "chunk_alignment_batch", "token_overlap", "estimate_reuse_ratio",
                                  "DeviceDonorMatrix", "DonorStore", "RadixDonorStore", "make_donor_store"])
def test_no_cuda_device_raises(name):
    from semblend_b200 import cagra_donor_store as cg
    from semblend_b200 import donor_store as ds
    from semblend_b200 import radix_store as rs

    toks = list(range(512))
    calls = {
        "chunk_alignment": lambda: al.chunk_alignment(toks, toks, 256),
        "chunk_alignment_batch": lambda: al.chunk_alignment_batch([toks], [toks], 256),
        "token_overlap": lambda: al.token_overlap(toks, toks),
        "estimate_reuse_ratio": lambda: al.estimate_reuse_ratio(toks, toks, 256),
        "DeviceDonorMatrix": lambda: se.DeviceDonorMatrix(10, 8),
        "DonorStore": lambda: ds.DonorStore(max_entries=10, embedding_dim=8),
        "RadixDonorStore": lambda: rs.RadixDonorStore(max_entries=10, embedding_dim=8),
        "make_donor_store": lambda: cg.make_donor_store(max_entries=10, embedding_dim=8, use_cagra=True),
    }
    with pytest.raises(_lib.NativeLibraryError):
        calls[name]()
