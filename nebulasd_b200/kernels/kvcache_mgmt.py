"""Paged KV-store behind the reference's ``store_kvcache`` signature.

Replaces ``swiftLLM/swiftllm/worker/kernels/kvcache_mgmt.py:81-122`` (prefill
kernel ``:10-48``, decode kernel ``:50-79``): K/V rows are bit-copied to
``cache[block_table[seq_id][pos // 16], cur_layer, :, pos % 16, :]`` with
``pos = seq_len - 1`` for decode rows and ``pos = i`` for prefill token ``i``.
One launch covers prefill and decode rows.  Out-of-range block ids are skipped
and recorded in a per-device error word instead of faulting.
"""
from __future__ import annotations

import torch

from .. import _lib
from .._workspace import error_word


def store_kvcache(k: torch.Tensor, v: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                  block_table: torch.Tensor, model_config, engine_config, infer_state, cur_layer: int) -> None:
    """Drop-in for the reference's ``store_kvcache`` (same signature and asserts)."""
    assert k.is_contiguous()
    assert v.is_contiguous()
    assert k_cache.is_contiguous()
    assert v_cache.is_contiguous()
    assert block_table.is_contiguous()
    assert infer_state.seq_ids.is_contiguous()
    assert infer_state.decoding_seq_lens.is_contiguous()
    if k.dtype != torch.float16 or k_cache.dtype != torch.float16:
        raise TypeError("k/v and the caches must be float16")
    nps, npt, nd = infer_state.num_prefill_seqs, infer_state.num_prefill_tokens, infer_state.num_decoding_seqs
    if nps == 0 and nd == 0:
        return
    num_blocks, num_layers, num_kv_heads, block_size, head_dim = k_cache.shape
    stream = torch.cuda.current_stream(k.device)
    starts = infer_state.prefill_seq_start_locs if nps else None
    lens = infer_state.prefill_seq_lens if nps else None
    rc = _lib.lib.neb_store_kvcache(
        k.data_ptr(), v.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), block_table.data_ptr(),
        block_table.shape[0], engine_config.max_blocks_per_seq, infer_state.seq_ids.data_ptr(),
        _lib.ptr(infer_state.decoding_seq_lens) if nd else None, nd, _lib.ptr(starts), _lib.ptr(lens), nps, npt,
        num_kv_heads, head_dim, block_size, num_blocks, num_layers, cur_layer,
        error_word(k.device).data_ptr(), stream.cuda_stream)
    _lib.check(rc, "store_kvcache")
