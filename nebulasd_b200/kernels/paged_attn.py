"""Paged decode / verify attention behind the reference's ``paged_attention`` signature.

Replaces ``swiftLLM/swiftllm/worker/kernels/paged_attn.py:152-222``.  Same
arguments, same contiguity assertions (``:163-168``), same outputs written into
``o``; one launch instead of two, no per-call ``torch.empty`` of partials.

Three CUDA kernels implement it (all correct for any row layout):
  * ``decode``: CUDA cores, for the Draft's single-token rows;
  * ``verify``: tcgen05 tensor cores, packing the GQA group and the k+1
    speculative rows of one request into the M dimension of the MMA tile;
  * ``verify_long``: tcgen05 tensor cores with 128 KV tokens on the M
    dimension, for long prefixes (the steady state dominates there).
``NEB_PAGED_ATTENTION=decode|verify|verify_long|auto`` (or ``set_kernel``)
picks one; ``auto`` uses a verify kernel when the q/kv head ratio is 4 or more
(the Qwen3-8B Target) or not one the decode kernel is built for, the long
variant when the batch's longest row has ``LONG_CONTEXT_TOKENS`` or more
tokens (``infer_state.max_decoding_len``), and ``decode`` otherwise (the
Qwen3-0.6B Draft).
"""
from __future__ import annotations

import os

import torch

from .. import _lib
from .. import _workspace as _ws
from .._workspace import attention_workspace

_MODES = {"auto": None, "decode": _lib.NEB_ATTN_DECODE, "verify": _lib.NEB_ATTN_VERIFY,
          "verify_long": _lib.NEB_ATTN_VERIFY_LONG}
_mode = os.environ.get("NEB_PAGED_ATTENTION", "auto").lower()
if _mode not in _MODES:
    raise ValueError(f"NEB_PAGED_ATTENTION must be one of {sorted(_MODES)} (got {_mode!r})")


def set_kernel(mode: str) -> None:
    """Select ``"auto"``, ``"decode"``, ``"verify"`` or ``"verify_long"`` for later calls."""
    global _mode
    if mode not in _MODES:
        raise ValueError(f"kernel must be one of {sorted(_MODES)}")
    _mode = mode


def get_kernel() -> str:
    return _mode


VERIFY_BUILT = os.environ.get("NEB_VERIFY_BUILT", "1") == "1"


DECODE_RATIOS = (1, 2, 4, 8)  # q/kv head ratios the CUDA-core kernel is built for
# Longest row (tokens) from which ``auto`` takes the long-context verify kernel:
# below it the per-launch fixed costs dominate and ``verify`` is faster.
LONG_CONTEXT_TOKENS = 8192


def choose_kernel(num_q_heads: int, num_kv_heads: int, num_rows: int = 0, max_len: int | None = None) -> int:
    """Tensor-core kernels for GQA ratios 4..16 (the rows x heads of a request
    fill its MMA tiles) and for every ratio the CUDA-core kernel is not built
    for (3, 5, 6, 7, 9..16), up to their row limit (the long-context variant
    when ``max_len``, the batch's longest row, reaches ``LONG_CONTEXT_TOKENS``);
    the CUDA-core kernel for ratios 1 and 2 and for batches beyond that limit."""
    forced = _MODES[_mode]
    if forced is not None:
        return forced
    gqa = num_q_heads // num_kv_heads
    if VERIFY_BUILT and (gqa >= 4 or gqa not in DECODE_RATIOS):
        if max_len is not None and max_len >= LONG_CONTEXT_TOKENS and 1 <= gqa <= 64 and \
                num_rows <= _lib.lib.neb_attention_max_rows(_lib.NEB_ATTN_VERIFY_LONG):
            return _lib.NEB_ATTN_VERIFY_LONG
        if gqa <= 16 and num_rows <= _lib.lib.neb_attention_max_rows(_lib.NEB_ATTN_VERIFY):
            return _lib.NEB_ATTN_VERIFY
    return _lib.NEB_ATTN_DECODE


_ENTRY = {}

# The current stream's raw handle without building a Stream object (a host
# cost of every call); torch.cuda.current_stream is the fallback.
_raw_stream_fn = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _raw_stream(index: int) -> int:
    if _raw_stream_fn is not None:
        return _raw_stream_fn(index)
    return torch.cuda.current_stream(index).cuda_stream


# The workspace of the previous call, reused while the call's kernel, device,
# stream and shape and the workspace generation stay the same (the 36 layer
# calls of a forward).  One tuple, swapped as a whole, so threads never pair
# one call's key with another's buffer.
_last = (None, None)


def _last_workspace(kernel, q, stream, stream_ptr, num_rows, num_q_heads, num_kv_heads):
    global _last
    idx = q.get_device()
    key = (kernel, idx, stream_ptr, num_rows, num_q_heads, num_kv_heads, _ws.generation)
    last_key, last_ws = _last
    if key == last_key:
        return last_ws
    s = stream if stream is not None else torch.cuda.ExternalStream(stream_ptr, device=idx)
    ws = attention_workspace(kernel, torch.device("cuda", idx), s, num_rows, num_q_heads, num_kv_heads)
    _last = (key, ws)
    return ws


def _entry(kernel: int):
    if not _ENTRY:
        _ENTRY.update({_lib.NEB_ATTN_DECODE: _lib.lib.neb_paged_attention_decode,
                       _lib.NEB_ATTN_VERIFY: _lib.lib.neb_paged_attention_verify,
                       _lib.NEB_ATTN_VERIFY_LONG: _lib.lib.neb_paged_attention_verify_long})
    return _ENTRY[kernel]


_F16, _I32 = torch.float16, torch.int32


def _check_tensors(q, k_cache, v_cache, block_table, seq_lens, seq_ids, o):
    if q.dtype != _F16 or k_cache.dtype != _F16 or v_cache.dtype != _F16 or o.dtype != _F16:
        raise TypeError("q, k_cache, v_cache and o must be float16")
    if block_table.dtype != _I32 or seq_lens.dtype != _I32 or seq_ids.dtype != _I32:
        raise TypeError("block_table, seq_lens and seq_ids must be int32")
    idx = q.get_device()  # -1 on the host
    if idx < 0 or any(t.get_device() != idx for t in (k_cache, v_cache, block_table, seq_lens, seq_ids, o)):
        raise ValueError("all tensors must be on the same CUDA device")
    if k_cache.shape != v_cache.shape or k_cache.dim() != 5:
        raise ValueError("k_cache/v_cache must be [num_blocks, num_layers, num_kv_heads, block_size, head_dim]")
    if not (seq_lens.is_contiguous() and seq_ids.is_contiguous()):
        raise ValueError("seq_lens and seq_ids must be contiguous")


def paged_attention_raw(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                        block_table: torch.Tensor, seq_lens: torch.Tensor, seq_ids: torch.Tensor,
                        cur_layer: int, softmax_scale: float, o: torch.Tensor,
                        kernel: int | None = None, workspace: torch.Tensor | None = None,
                        stream: torch.cuda.Stream | None = None, max_len: int | None = None) -> None:
    """Tensor-level entry: ``o[r] = attention(q[r], KV of seq_ids[r] up to seq_lens[r])``.

    ``max_len`` (optional, the longest of ``seq_lens``, known on the host) lets
    ``auto`` pick the long-context kernel."""
    _check_tensors(q, k_cache, v_cache, block_table, seq_lens, seq_ids, o)
    num_rows, num_q_heads, head_dim = q.shape
    num_blocks, num_layers, num_kv_heads, block_size, _ = k_cache.shape
    if o.shape != q.shape or seq_lens.shape[0] != num_rows or seq_ids.shape[0] != num_rows:
        raise ValueError("q, o, seq_lens and seq_ids disagree on the number of rows")
    if kernel is None:
        kernel = choose_kernel(num_q_heads, num_kv_heads, num_rows, max_len)
    if stream is not None:
        stream_ptr = stream.cuda_stream
    else:
        stream_ptr = _raw_stream(q.get_device())
    if workspace is None:
        workspace = _last_workspace(kernel, q, stream, stream_ptr, num_rows, num_q_heads, num_kv_heads)
    rc = _entry(kernel)(q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), block_table.data_ptr(),
            block_table.shape[0], block_table.shape[1], seq_lens.data_ptr(), seq_ids.data_ptr(),
            num_rows, num_q_heads, num_kv_heads, head_dim, block_size, num_blocks, num_layers,
            cur_layer, float(softmax_scale), o.data_ptr(), workspace.data_ptr(), workspace.numel(),
            stream_ptr)
    _lib.check(rc, "paged_attention")


def paged_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                    block_table: torch.Tensor, model_config, engine_config, infer_state,
                    cur_layer: int, o: torch.Tensor) -> None:
    """Drop-in for the reference's ``paged_attention`` (same signature and asserts)."""
    assert q.is_contiguous()
    assert k_cache.is_contiguous()
    assert v_cache.is_contiguous()
    assert block_table.is_contiguous()
    assert infer_state.seq_block_size % engine_config.block_size == 0
    assert o.is_contiguous()
    if infer_state.num_decoding_seqs == 0:
        return
    if block_table.shape[1] != engine_config.max_blocks_per_seq:
        raise ValueError("block_table.shape[1] must equal engine_config.max_blocks_per_seq")
    o3 = o.view(infer_state.num_decoding_seqs, model_config.num_q_heads, model_config.head_dim)
    q3 = q.view(infer_state.num_decoding_seqs, model_config.num_q_heads, model_config.head_dim)
    paged_attention_raw(q3, k_cache, v_cache, block_table, infer_state.decoding_seq_lens,
                        infer_state.seq_ids[infer_state.num_prefill_seqs:], cur_layer,
                        infer_state.softmax_scale, o3, max_len=getattr(infer_state, "max_decoding_len", None))
