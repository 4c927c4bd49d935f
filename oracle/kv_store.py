"""Restatement of swiftLLM's paged KV-store placement (CPU, bit copies).

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Reference: ``swiftLLM/swiftllm/worker/kernels/kvcache_mgmt.py``
  * decode rows ``:50-79`` (+ eager spec ``:124-132``): for decode row ``r`` with
    ``pos = seq_lens[r] - 1``, ``blk = block_table[seq_ids[r], pos // 16]``,
    ``cache[blk, cur_layer, :, pos % 16, :] = k[r]`` (and the same for V);
  * prefill ``:10-48``: token ``i`` of prefill sequence ``s`` (start
    ``start_locs[s]``) goes to ``cache[block_table[seq_ids[s], i // 16], cur_layer,
    :, i % 16, :]``;
  * wrapper ``:81-122``: prefill rows first, then decode rows read
    ``k[num_prefill_tokens:]`` and ``seq_ids[num_prefill_seqs:]``.
"""
from __future__ import annotations

import torch


def store_decode(k, v, k_cache, v_cache, block_table, seq_ids, seq_lens, cur_layer: int) -> None:
    """In-place decode-row store; ``k``/``v`` are ``[R, Hk, D]`` (any dtype copy is bitwise)."""
    block_size = k_cache.shape[3]
    seq_ids = [int(x) for x in seq_ids]
    seq_lens = [int(x) for x in seq_lens]
    for r, (sid, n) in enumerate(zip(seq_ids, seq_lens)):
        pos = n - 1
        blk = int(block_table[sid, pos // block_size])
        k_cache[blk, cur_layer, :, pos % block_size, :] = k[r]
        v_cache[blk, cur_layer, :, pos % block_size, :] = v[r]


def store_prefill(k, v, k_cache, v_cache, block_table, seq_ids, start_locs, seq_lens, cur_layer: int) -> None:
    """In-place prefill store following ``kvcache_mgmt.py:10-48``."""
    block_size = k_cache.shape[3]
    for sid, start, n in zip(seq_ids, start_locs, seq_lens):
        sid, start, n = int(sid), int(start), int(n)
        for i in range(n):
            blk = int(block_table[sid, i // block_size])
            k_cache[blk, cur_layer, :, i % block_size, :] = k[start + i]
            v_cache[blk, cur_layer, :, i % block_size, :] = v[start + i]


def slot_of(block_table, seq_id: int, pos: int, block_size: int = 16) -> tuple[int, int]:
    """``(physical block, offset in block)`` of token ``pos`` of ``seq_id``."""
    return int(block_table[seq_id, pos // block_size]), pos % block_size
