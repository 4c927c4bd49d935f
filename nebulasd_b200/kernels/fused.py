"""Fused Qwen3 QK-RMSNorm + RoPE + paged KV-store in one launch.

Replaces the sequence at ``swiftLLM/swiftllm/worker/layers/transformer_layer.py:114-143``:

    rmsnorm_inplace(q.reshape(-1, D), q_norm, eps)     # only if has_qk_norm
    rmsnorm_inplace(k.reshape(-1, D), k_norm, eps)
    rotary_embedding_inplace(q, k, infer_state)
    store_kvcache(k, v, k_cache, v_cache, block_table, ..., cur_layer)

with the same in-place results on ``q`` and ``k`` and the same cache contents
(four launches and three full passes over q/k become one pass).
"""
from __future__ import annotations

import torch

from .. import _lib
from .._workspace import error_word


def qk_norm_rope_store(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, q_norm: torch.Tensor | None,
                       k_norm: torch.Tensor | None, eps: float, k_cache: torch.Tensor | None,
                       v_cache: torch.Tensor | None, block_table: torch.Tensor | None, model_config,
                       engine_config, infer_state, cur_layer: int) -> None:
    """q ``[T, H, D]``, k/v ``[T, Hk, D]`` fp16 contiguous; norms optional, caches optional."""
    for t in (q, k, v):
        if not t.is_contiguous() or t.dtype != torch.float16:
            raise ValueError("q, k, v must be contiguous float16")
    num_tokens, num_q_heads, head_dim = q.shape
    num_kv_heads = k.shape[1]
    if num_tokens == 0:
        return
    cos, sin = infer_state.position_cos, infer_state.position_sin
    nps, npt, nd = infer_state.num_prefill_seqs, infer_state.num_prefill_tokens, infer_state.num_decoding_seqs
    store = k_cache is not None and not getattr(infer_state, "ignore_kvcache", False)
    if store:
        num_blocks, num_layers, _, block_size, _ = k_cache.shape
        mbs = engine_config.max_blocks_per_seq
    else:
        num_blocks, num_layers, block_size, mbs = 1, 1, 16, 1
    rc = _lib.lib.neb_qk_norm_rope_store(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), _lib.ptr(q_norm), _lib.ptr(k_norm), float(eps),
        _lib.ptr(cos), _lib.ptr(sin),
        k_cache.data_ptr() if store else None, v_cache.data_ptr() if store else None,
        block_table.data_ptr() if store else None, block_table.shape[0] if store else 1, mbs,
        infer_state.seq_ids.data_ptr(), _lib.ptr(infer_state.decoding_seq_lens) if nd else None, nd,
        _lib.ptr(infer_state.prefill_seq_start_locs) if nps else None,
        _lib.ptr(infer_state.prefill_seq_lens) if nps else None, nps, npt,
        num_q_heads, num_kv_heads, head_dim, block_size, num_blocks, num_layers, cur_layer if store else 0,
        error_word(q.device).data_ptr(), torch.cuda.current_stream(q.device).cuda_stream)
    _lib.check(rc, "qk_norm_rope_store")
