"""fp32 eager restatement of swiftLLM's prefill attention (CPU).

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Reference semantics: ``swiftLLM/swiftllm/worker/layers/transformer_layer.py:7-32``
(``flash_attn_varlen_func``, called at ``:154-164`` with the same
``cu_seqlens`` for q and k and ``causal=True``): sequence ``s`` is tokens
``cu[s] .. cu[s+1]-1``; each q head ``h`` attends with kv head ``h // gqa``
(the reference repeats K and V ``gqa`` times along the head axis), causally
within its own sequence, scores scaled by ``softmax_scale`` (default
``1/sqrt(head_dim)``, as ``scaled_dot_product_attention``).  An empty sequence
contributes no rows.
"""
from __future__ import annotations

import torch


def prefill_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cu_seqlens, softmax_scale=None):
    """q ``[T, H, D]``, k and v ``[T, Hk, D]``; returns fp32 ``[T, H, D]`` on q's device."""
    tokens, heads, dim = q.shape
    gqa = heads // k.shape[1]
    scale = softmax_scale if softmax_scale is not None else dim ** -0.5
    out = torch.zeros((tokens, heads, dim), dtype=torch.float32, device=q.device)
    cu = [int(x) for x in (cu_seqlens.tolist() if torch.is_tensor(cu_seqlens) else cu_seqlens)]
    for s, e in zip(cu[:-1], cu[1:]):
        n = e - s
        if n <= 0:
            continue
        qi = q[s:e].float().transpose(0, 1)                               # [H, n, D]
        ki = k[s:e].float().transpose(0, 1).repeat_interleave(gqa, 0)     # [H, n, D]
        vi = v[s:e].float().transpose(0, 1).repeat_interleave(gqa, 0)
        att = (qi @ ki.transpose(1, 2)) * scale
        future = torch.triu(torch.ones(n, n, dtype=torch.bool, device=q.device), 1)
        att = att.masked_fill(future, float("-inf"))
        out[s:e] = (att.softmax(-1) @ vi).transpose(0, 1)
    return out
