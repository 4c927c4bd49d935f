"""RoPE behind the reference's ``rotary_embedding_inplace`` signature.

Replaces ``swiftLLM/swiftllm/worker/kernels/rotary_emb.py:44-58``: rotate-half
on the two 64-halves of every q and k head row of token ``t`` with the fp16
``infer_state.position_cos/sin[t]``, computed with the reference's fp16
arithmetic (each multiply and add rounded to fp16, no fused multiply-add).
"""
from __future__ import annotations

import torch

from .. import _lib


def rotary_embedding_inplace(q: torch.Tensor, k: torch.Tensor, infer_state) -> None:
    num_tokens, num_q_heads, head_dim = q.shape
    num_kv_heads = k.shape[1]
    if num_tokens == 0:
        return
    cos, sin = infer_state.position_cos, infer_state.position_sin
    if not (q.is_contiguous() and k.is_contiguous() and cos.is_contiguous() and sin.is_contiguous()):
        raise ValueError("q, k and the cos/sin rows must be contiguous")
    if q.dtype != torch.float16 or k.dtype != torch.float16 or cos.dtype != torch.float16:
        raise TypeError("q, k, cos, sin must be float16")
    rc = _lib.lib.neb_rotary_inplace(q.data_ptr(), k.data_ptr(), cos.data_ptr(), sin.data_ptr(), num_tokens,
                                     num_q_heads, num_kv_heads, head_dim,
                                     torch.cuda.current_stream(q.device).cuda_stream)
    _lib.check(rc, "rotary_embedding_inplace")
