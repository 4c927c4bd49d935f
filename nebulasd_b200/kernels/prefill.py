"""Causal prefill attention over packed variable-length sequences, without a host sync.

Replaces ``flash_attn_varlen_func`` in
``swiftLLM/swiftllm/worker/layers/transformer_layer.py:7-32``, which copies
``cu_seqlens`` to the host and runs one ``scaled_dot_product_attention`` per
sequence (repeating K and V for every q head of a kv head).  Same arguments;
``causal`` must be true and the q and k sequences the same, as in the
reference's only call (``transformer_layer.py:154-164``).

q/kv head ratios 1, 2, 4, 8 and 16 (Qwen3: 2 and 4) run the prefill kernel
(``csrc/prefill_attn.cu``: tcgen05, 128 query rows of one kv head's q heads
per tile, K and V read by TMA straight from ``k`` and ``v``; a one-CTA plan
launch orders the work from ``cu_seqlens`` on the device).  Other ratios lay
the keys and values out as a small paged cache and run the verify kernel
with one row per prompt token.  Neither reads ``cu_seqlens`` on the host.
"""
from __future__ import annotations

import threading

import torch

from .. import _lib
from .paged_attn import _raw_stream, paged_attention_raw

PREFILL_RATIOS = (1, 2, 4, 8, 16)

_lock = threading.Lock()
_buffers: dict = {}


def _workspace(device: torch.device, stream_ptr: int, need: int) -> torch.Tensor:
    key = (device.index, stream_ptr)
    with _lock:
        buf = _buffers.get(key)
        if buf is None or buf.numel() < need:
            with torch.inference_mode(False):
                buf = torch.zeros(max(need, 2 * (buf.numel() if buf is not None else 0)), dtype=torch.uint8,
                                  device=device)
            _buffers[key] = buf
        return buf


def workspace_errors(stream: torch.cuda.Stream | None = None, device: torch.device | None = None) -> int:
    """Synchronise and return (and clear) the error bits of this stream's prefill
    workspace (bit 5: a ``cu_seqlens`` that is not a split of the tokens, or a
    sequence longer than ``max_seqlen``; bit 3: a bounded wait gave up)."""
    import ctypes
    device = device or torch.device("cuda", torch.cuda.current_device())
    stream = stream or torch.cuda.current_stream(device)
    ws = _workspace(device, stream.cuda_stream, _lib.lib.neb_prefill_attention_workspace_bytes(0, 0, 1, 1))
    bits = ctypes.c_uint32(0)
    _lib.check(_lib.lib.neb_workspace_status(ws.data_ptr(), ctypes.byref(bits), stream.cuda_stream),
               "neb_workspace_status")
    return bits.value


def _check(q, k, v, cu):
    if q.dtype != torch.float16 or k.dtype != torch.float16 or v.dtype != torch.float16:
        raise TypeError("q, k and v must be float16")
    if q.dim() != 3 or k.dim() != 3 or v.shape != k.shape or q.shape[0] != k.shape[0] or q.shape[2] != k.shape[2]:
        raise ValueError("q [T, H, D] and k, v [T, Hk, D] must cover the same tokens")
    if q.shape[2] != 128:
        raise ValueError("head_dim must be 128")
    dev = q.device
    if k.device != dev or v.device != dev or cu.device != dev:
        raise ValueError("q, k, v and cu_seqlens must be on the same device")
    if cu.dtype != torch.int32 or cu.dim() != 1 or not cu.is_contiguous():
        raise ValueError("cu_seqlens must be a contiguous int32 vector")
    for name, t in (("q", q), ("k", k), ("v", v)):
        if t.stride(2) != 1 or t.stride(1) != 128:
            raise ValueError(f"{name} must have contiguous heads of 128 elements")


def flash_attn_varlen_func(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cu_seqlens_q: torch.Tensor,
                           cu_seqlens_k: torch.Tensor, max_seqlen_q: int, max_seqlen_k: int,
                           softmax_scale: float | None = None, causal: bool = True) -> torch.Tensor:
    """q ``[T, H, D]``, k and v ``[T, Hk, D]`` fp16, ``cu_seqlens`` int32 ``[S + 1]``
    on the device; returns ``[T, H, D]``: causal attention within each sequence."""
    if not causal:
        raise NotImplementedError("only causal prefill attention is supported")
    if cu_seqlens_k is not cu_seqlens_q and not torch.equal(cu_seqlens_k, cu_seqlens_q):
        raise NotImplementedError("q and k must cover the same sequences")
    _check(q, k, v, cu_seqlens_q)
    tokens, heads, dim = q.shape
    kv_heads = k.shape[1]
    out = torch.empty((tokens, heads, dim), dtype=q.dtype, device=q.device)
    nseq = cu_seqlens_q.numel() - 1
    if tokens == 0 or nseq <= 0:
        return out
    scale = softmax_scale if softmax_scale is not None else dim ** -0.5
    if heads % kv_heads == 0 and heads // kv_heads in PREFILL_RATIOS:
        stream_ptr = _raw_stream(q.get_device())
        need = _lib.lib.neb_prefill_attention_workspace_bytes(tokens, nseq, heads, kv_heads)
        ws = _workspace(q.device, stream_ptr, need)
        rc = _lib.lib.neb_prefill_attention(q.data_ptr(), q.stride(0), k.data_ptr(), k.stride(0), v.data_ptr(),
                                            v.stride(0), cu_seqlens_q.data_ptr(), nseq, tokens,
                                            int(max(max_seqlen_q, max_seqlen_k)), heads, kv_heads, dim,
                                            float(scale), out.data_ptr(), out.stride(0), ws.data_ptr(), ws.numel(),
                                            stream_ptr)
        _lib.check(rc, "flash_attn_varlen_func")
        return out
    return _via_verify(q, k, v, cu_seqlens_q, max_seqlen_k, scale, out)


def _via_verify(q, k, v, cu_seqlens, max_seqlen, scale, out):
    """Other head ratios: each sequence's keys and values in its own 16-token
    blocks of a small paged cache, then the verify kernel over one row per
    prompt token (its sequence, its position + 1 as the length)."""
    tokens, heads, dim = q.shape
    kv_heads = k.shape[1]
    dev = q.device
    nseq = cu_seqlens.numel() - 1
    cu = cu_seqlens.to(torch.int64)
    lens = cu[1:] - cu[:-1]
    t_idx = torch.arange(tokens, device=dev)
    seq = torch.searchsorted(cu[1:], t_idx, right=True)
    pos = t_idx - cu[seq]
    # Each sequence's blocks, laid end to end: at most T / 16 + S of them.
    nblk = (lens + 15) // 16
    first_blk = torch.cumsum(nblk, 0) - nblk
    max_blocks = tokens // 16 + nseq
    mbs = (int(max_seqlen) + 15) // 16
    k_cache = torch.zeros((max_blocks, 1, kv_heads, 16, dim), dtype=torch.float16, device=dev)
    v_cache = torch.zeros_like(k_cache)
    blk = first_blk[seq] + pos // 16
    slot = pos % 16
    k_cache[blk, 0, :, slot] = k
    v_cache[blk, 0, :, slot] = v
    cols = torch.arange(mbs, device=dev)
    table = torch.where(cols[None, :] < nblk[:, None], first_blk[:, None] + cols[None, :],
                        torch.full_like(first_blk[:, None], -1)).to(torch.int32).contiguous()
    seq_ids = seq.to(torch.int32)
    seq_lens = (pos + 1).to(torch.int32)
    step = _lib.lib.neb_attention_max_rows(_lib.NEB_ATTN_VERIFY)
    for r0 in range(0, tokens, step):
        r1 = min(tokens, r0 + step)
        paged_attention_raw(q[r0:r1].contiguous(), k_cache, v_cache, table, seq_lens[r0:r1].contiguous(),
                            seq_ids[r0:r1].contiguous(), 0, scale, out[r0:r1], kernel=_lib.NEB_ATTN_VERIFY)
    return out
