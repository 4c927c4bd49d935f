"""fp32 eager restatement of swiftLLM paged decode/verify attention (CPU).

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Reference semantics:
  * ``swiftLLM/swiftllm/worker/kernels/paged_attn.py:152-222`` (wrapper) and
    ``:9-108`` (phase 1): each decode row ``r`` attends query ``q[r, h]`` to the
    first ``seq_lens[r]`` tokens of sequence ``seq_ids[r]``; token ``t`` lives in
    ``cache[block_table[seq_id, t // 16], cur_layer, h // gqa, t % 16, :]``;
    positions ``>= seq_len`` are masked (``:74-75``).
  * ``paged_attn.py:224-259``: the commented eager specification (gather blocks,
    ``repeat_interleave`` over the GQA group, mask, softmax, bmm) that this file
    follows.
  * Verify of depth k is k+1 such rows with the same ``seq_id`` and
    ``seq_lens`` L+1..L+k+1 (``nebulasd/src/nebulasd/workers/target/backend.py:102-111``,
    ``swiftLLM/swiftllm/speculative.py:75-89``); causality comes only from the
    per-row length mask.

Rows with the same ``seq_id`` that are adjacent share one gathered KV prefix here
(pure efficiency: the per-row mask keeps the semantics of the reference's
independent rows).  A row whose ``seq_len <= 0`` has every position masked; the
reference's phase 2 then divides 0 by 0 (``paged_attn.py:149``), and so does
this oracle (NaN output).
"""
from __future__ import annotations

import math

import torch


def split_heuristic(decoding_seq_lens: list[int], num_kv_heads: int) -> tuple[int, int]:
    """The reference's split-K choice, ``swiftLLM/swiftllm/worker/model.py:380-384``.

    Returns ``(seq_block_size, num_seq_blocks)``.  The CUDA kernels choose their
    own split; this is kept so the drop-in wrapper can be fed the same
    ``infer_state`` the reference builds.
    """
    seq_block_size = 2048
    total = sum(decoding_seq_lens)
    max_len = max(decoding_seq_lens) if decoding_seq_lens else 0
    while (num_kv_heads * (total / seq_block_size) < 1024 and seq_block_size // 2 >= 64
           and max_len / (seq_block_size // 2) <= 128):
        seq_block_size //= 2
    return seq_block_size, (max_len + seq_block_size - 1) // seq_block_size


def _row_groups(seq_ids: list[int]) -> list[tuple[int, int]]:
    groups, start = [], 0
    for r in range(1, len(seq_ids) + 1):
        if r == len(seq_ids) or seq_ids[r] != seq_ids[start]:
            groups.append((start, r))
            start = r
    return groups


def paged_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                    block_table: torch.Tensor, seq_lens, seq_ids, cur_layer: int,
                    softmax_scale: float) -> torch.Tensor:
    """fp32 attention output ``[R, H, D]`` for decode rows (CPU tensors).

    ``q``: ``[R, H, D]``; caches ``[NB, L, Hk, BS, D]``; ``block_table``
    ``[rows, max_blocks]`` int32; ``seq_lens``/``seq_ids``: length-R int lists or
    tensors.
    """
    seq_lens = [int(x) for x in (seq_lens.tolist() if torch.is_tensor(seq_lens) else seq_lens)]
    seq_ids = [int(x) for x in (seq_ids.tolist() if torch.is_tensor(seq_ids) else seq_ids)]
    num_rows, num_q_heads, head_dim = q.shape
    num_kv_heads, block_size = k_cache.shape[2], k_cache.shape[3]
    gqa = num_q_heads // num_kv_heads
    out = torch.empty((num_rows, num_q_heads, head_dim), dtype=torch.float32)
    for start, end in _row_groups(seq_ids):
        lens = seq_lens[start:end]
        max_len = max(lens)
        rows = end - start
        if max_len <= 0:
            out[start:end] = float("nan")
            continue
        num_blocks = (max_len + block_size - 1) // block_size
        blocks = block_table[seq_ids[start], :num_blocks].long()
        # [nb, Hk, BS, D] -> [Hk, nb*BS, D]
        keys = k_cache[blocks, cur_layer].float().permute(1, 0, 2, 3).reshape(num_kv_heads, -1, head_dim)[:, :max_len]
        vals = v_cache[blocks, cur_layer].float().permute(1, 0, 2, 3).reshape(num_kv_heads, -1, head_dim)[:, :max_len]
        qg = q[start:end].float().view(rows, num_kv_heads, gqa, head_dim)
        scores = torch.einsum("rkgd,ktd->rkgt", qg, keys) * softmax_scale
        pos = torch.arange(max_len)
        valid = pos[None, :] < torch.tensor(lens)[:, None]           # [rows, T]
        scores = scores.masked_fill(~valid[:, None, None, :], float("-inf"))
        probs = torch.softmax(scores, dim=-1)
        o = torch.einsum("rkgt,ktd->rkgd", probs, vals)
        out[start:end] = o.reshape(rows, num_q_heads, head_dim)
    return out


def paged_attention_rows(q, k_cache, v_cache, block_table, seq_lens, seq_ids, cur_layer, softmax_scale):
    """Row-by-row literal transcription of ``paged_attn.py:224-259`` (small cases).

    Used by the CPU tests to pin the grouped ``paged_attention`` above against
    the reference's own eager specification, line for line.
    """
    seq_lens = [int(x) for x in (seq_lens.tolist() if torch.is_tensor(seq_lens) else seq_lens)]
    seq_ids = [int(x) for x in (seq_ids.tolist() if torch.is_tensor(seq_ids) else seq_ids)]
    num_rows, num_q_heads, head_dim = q.shape
    num_kv_heads, block_size = k_cache.shape[2], k_cache.shape[3]
    out = torch.empty((num_rows, num_q_heads, head_dim), dtype=torch.float32)
    for r in range(num_rows):
        my_q = q[r]
        nb = (seq_lens[r] + block_size - 1) // block_size
        ks = [k_cache[int(block_table[seq_ids[r], b])][cur_layer] for b in range(nb)]
        vs = [v_cache[int(block_table[seq_ids[r], b])][cur_layer] for b in range(nb)]
        if not ks:
            out[r] = float("nan")
            continue
        my_k = torch.cat(ks, dim=1).repeat_interleave(num_q_heads // num_kv_heads, dim=0).float()
        my_v = torch.cat(vs, dim=1).repeat_interleave(num_q_heads // num_kv_heads, dim=0).float()
        s = torch.bmm(my_q.reshape(num_q_heads, 1, head_dim).float(), my_k.transpose(1, 2)).squeeze(1)
        s = s * softmax_scale
        s = torch.where(torch.arange(s.shape[1]) < seq_lens[r], s, torch.full_like(s, float("-inf")))
        p = torch.softmax(s, dim=1).unsqueeze(1)
        out[r] = torch.bmm(p, my_v).squeeze(1)
    return out


def kv_bytes(seq_lens, seq_ids, num_kv_heads: int, head_dim: int, elem_bytes: int = 2) -> int:
    """Unique K+V bytes one call must read: per adjacent same-seq group, its max length.

    This is the algorithmic-bytes figure of the roofline (``4096 B`` per token
    for Hk=8, D=128, fp16 K and V).
    """
    seq_lens = [int(x) for x in seq_lens]
    seq_ids = [int(x) for x in seq_ids]
    total = 0
    for start, end in _row_groups(seq_ids):
        total += max(0, max(seq_lens[start:end]))
    return total * num_kv_heads * head_dim * 2 * elem_bytes


DEFAULT_SCALE_128 = 1.0 / math.sqrt(128.0)
