"""CPU oracle: partial-prefill attention and masked QKV projection — test
infrastructure only.

Restates semblend_core/triton_kernels.py (SemBlend 0.3.2): the CPU branch of
``partial_prefill_attention`` (:717-732) and of ``masked_qkv_projection``
(:512-520).  GQA (the reference has none, :669-671) is the standard mapping of
query head h to KV head h // (Hq // Hkv), applied by repeating KV heads.
"""

from __future__ import annotations

import math

import torch


def partial_prefill_attention(query, key, value, compute_mask, scale=None, compute_dtype=None):
    """Per-row causal attention at the compute-mask rows (triton_kernels.py:679-734).

    ``query``/``key``/``value`` are ``[H, S, D]``.  Rows where the mask is
    False are zero.  ``compute_dtype`` (default: the query's dtype, as in the
    reference) is the dtype the matmuls and softmax run in; the output has the
    query's dtype.
    """
    H, S, D = query.shape
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    out = torch.zeros_like(query)
    cd = compute_dtype or query.dtype
    q_all, k_all, v_all = query.to(cd), key.to(cd), value.to(cd)
    for pos in torch.where(compute_mask)[0].tolist():
        q = q_all[:, pos : pos + 1, :]
        k = k_all[:, : pos + 1, :]
        v = v_all[:, : pos + 1, :]
        scores = torch.matmul(q, k.transpose(-2, -1)) * scale
        w = torch.softmax(scores, dim=-1)
        out[:, pos : pos + 1, :] = torch.matmul(w, v).to(query.dtype)
    return out


def partial_prefill_attention_blocked(query, key, value, rows, scale=None, block=64):
    """fp32 causal attention at ``rows`` (sorted int positions) computed a block
    of rows at a time with -inf masking of keys beyond each row; equal to
    :func:`partial_prefill_attention` in fp32 up to summation order.  Returns
    ``[H, len(rows), D]`` fp32 for the given rows only."""
    H, S, D = query.shape
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    rows = torch.as_tensor(rows, dtype=torch.long)
    q32, k32, v32 = query.float(), key.float(), value.float()
    out = torch.empty(H, rows.shape[0], D, dtype=torch.float32)
    for b0 in range(0, rows.shape[0], block):
        r = rows[b0 : b0 + block]
        kmax = int(r.max()) + 1
        s = torch.matmul(q32[:, r, :], k32[:, :kmax, :].transpose(-2, -1)) * scale
        keys = torch.arange(kmax)
        s = s.masked_fill(keys[None, None, :] > r[None, :, None], float("-inf"))
        w = torch.softmax(s, dim=-1)
        out[:, b0 : b0 + r.shape[0], :] = torch.matmul(w, v32[:, :kmax, :])
    return out


def expand_kv_heads(kv: torch.Tensor, n_q_heads: int) -> torch.Tensor:
    """[Hkv, S, D] -> [Hq, S, D]: query head h reads KV head h // (Hq // Hkv)."""
    hkv = kv.shape[0]
    if n_q_heads % hkv:
        raise ValueError(f"{n_q_heads} query heads are not a multiple of {hkv} KV heads")
    return kv.repeat_interleave(n_q_heads // hkv, dim=0)


def masked_qkv_projection(hidden_states, qkv_weight, compute_mask, qkv_bias=None):
    """triton_kernels.py:512-520: fp32 linear, reuse rows zeroed, cast back."""
    projected = torch.nn.functional.linear(
        hidden_states.float(), qkv_weight.float(), qkv_bias.float() if qkv_bias is not None else None
    )
    return (projected * compute_mask.unsqueeze(1).float()).to(hidden_states.dtype)


def partial_prefill(hidden_states, donor_kv, qkv_weight, output_projection, donor_positions,
                    target_positions, compute_mask, num_heads, head_dim, qkv_bias=None,
                    output_bias=None, scale=None):
    """triton_kernels.py:769-923 on CPU: scatter, masked projection, layer-0
    merge in fp32, fp32 partial attention, fp32 output projection, reuse rows
    zeroed, new K/V written into every layer.  Returns ``(output, kv_cache)``."""
    from .rope import scatter_donor_kv

    S = hidden_states.shape[0]
    L = donor_kv.shape[0]
    if scale is None:
        scale = 1.0 / math.sqrt(head_dim)
    target = torch.zeros((L, 2, num_heads, S, head_dim), dtype=hidden_states.dtype)
    target = scatter_donor_kv(target, donor_kv.to(target.dtype), donor_positions, target_positions)
    qkv = masked_qkv_projection(hidden_states, qkv_weight, compute_mask, qkv_bias)
    qkv = qkv.float().view(S, 3, num_heads, head_dim)
    q_new, k_new, v_new = (qkv[:, i].permute(1, 0, 2) for i in range(3))
    comp = torch.where(compute_mask)[0]
    merged_k = target[0, 0].float().clone()
    merged_v = target[0, 1].float().clone()
    merged_k[:, comp] = k_new[:, comp]
    merged_v[:, comp] = v_new[:, comp]
    attn = partial_prefill_attention(q_new.contiguous(), merged_k, merged_v, compute_mask, scale)
    final = torch.nn.functional.linear(
        attn.permute(1, 0, 2).reshape(S, num_heads * head_dim), output_projection.float(),
        output_bias.float() if output_bias is not None else None,
    ).to(hidden_states.dtype)
    final[~compute_mask] = 0.0
    for layer in range(L):
        target[layer, 0][:, comp] = k_new[:, comp].to(target.dtype)
        target[layer, 1][:, comp] = v_new[:, comp].to(target.dtype)
    return final, target
