"""Seeded synthetic paged-KV workloads with the shapes of the benchmark configs.

There is no dataset or checkpoint on this path: every config is defined by
shapes, length distributions and i.i.d. N(0,1) fp16 values, so these builders
*are* the workloads.  Host-side integers (lengths, block tables) come from a
numpy generator and are identical on every machine for a given seed; tensor
values come from a torch generator on the target device.

Layout conventions follow the reference:
  * caches ``[num_blocks, num_layers, num_kv_heads, block_size, head_dim]`` fp16
    (``swiftLLM/swiftllm/worker/model.py:152-166``);
  * a request with prefix length ``L`` verified at depth ``k`` becomes ``k+1``
    adjacent decode rows with the same ``seq_id`` and ``seq_lens`` ``L+1 .. L+k+1``
    (``nebulasd/src/nebulasd/workers/target/backend.py:102-111``); depth 0 is a
    plain decode row;
  * ``block_table[seq_id, i]`` is the physical block of logical block ``i``;
    unused entries hold ``-1`` so that any read past a sequence's end shows up.
"""
from __future__ import annotations

import dataclasses
import math

import numpy as np
import torch

BLOCK_SIZE = 16
HEAD_DIM = 128


@dataclasses.dataclass
class PagedBatch:
    q: torch.Tensor               # [R, H, D] fp16
    k_cache: torch.Tensor         # [NB, L, Hk, BS, D] fp16
    v_cache: torch.Tensor
    block_table: torch.Tensor     # [num_requests, max_blocks] int32
    seq_ids: torch.Tensor         # [R] int32
    seq_lens: torch.Tensor        # [R] int32
    seq_ids_list: list
    seq_lens_list: list
    ctx: list                     # prefix length per request
    depths: list                  # verify depth per request (rows = depth + 1)
    cur_layer: int
    num_q_heads: int
    num_kv_heads: int

    @property
    def num_rows(self) -> int:
        return len(self.seq_ids_list)

    def kv_bytes(self) -> int:
        """Unique K+V bytes of one attention call (the roofline's algorithmic bytes)."""
        per_token = self.num_kv_heads * self.k_cache.shape[-1] * 2 * self.k_cache.element_size()
        return sum(c + d + 1 for c, d in zip(self.ctx, self.depths)) * per_token


def host_layout(seed: int, *, num_requests: int, depth, ctx_lo: int, ctx_hi: int,
                pool_blocks: int, max_blocks_per_seq: int | None = None,
                block_size: int = BLOCK_SIZE, shuffle_seq_ids: bool = False):
    """Lengths, rows and a random block table (numpy, machine independent)."""
    rng = np.random.default_rng(seed)
    ctx = rng.integers(ctx_lo, ctx_hi + 1, size=num_requests).tolist()
    if isinstance(depth, int):
        depths = [depth] * num_requests
    else:
        depths = [int(d) for d in depth]
    need = [math.ceil((c + d + 1) / block_size) for c, d in zip(ctx, depths)]
    if max_blocks_per_seq is None:
        max_blocks_per_seq = max(need) if need else 1
    if sum(need) > pool_blocks:
        raise ValueError(f"pool of {pool_blocks} blocks cannot hold {sum(need)} blocks")
    perm = rng.permutation(pool_blocks)
    table = np.full((num_requests, max_blocks_per_seq), -1, dtype=np.int32)
    used = 0
    for i, n in enumerate(need):
        table[i, :n] = perm[used:used + n]
        used += n
    sid_of = rng.permutation(num_requests).tolist() if shuffle_seq_ids else list(range(num_requests))
    # Rows of request i sit in the table row sid_of[i].
    table_rows = np.full_like(table, -1)
    for i in range(num_requests):
        table_rows[sid_of[i]] = table[i]
    seq_ids, seq_lens = [], []
    for i, (c, d) in enumerate(zip(ctx, depths)):
        for j in range(d + 1):
            seq_ids.append(sid_of[i])
            seq_lens.append(c + 1 + j)
    return ctx, depths, table_rows, seq_ids, seq_lens


def make_paged_batch(seed: int, *, num_requests: int, depth, ctx_lo: int, ctx_hi: int,
                     num_q_heads: int, num_kv_heads: int, pool_blocks: int,
                     num_layers: int = 1, cur_layer: int = 0, head_dim: int = HEAD_DIM,
                     block_size: int = BLOCK_SIZE, device="cpu",
                     max_blocks_per_seq: int | None = None, shuffle_seq_ids: bool = False,
                     cache: tuple | None = None) -> PagedBatch:
    """Build a seeded verify (depth>0) or decode (depth=0) batch.

    ``cache`` may pass pre-built ``(k_cache, v_cache)`` to share one large pool
    across batches (the benchmark's 58 GB Qwen3-8B pool).
    """
    ctx, depths, table, seq_ids, seq_lens = host_layout(
        seed, num_requests=num_requests, depth=depth, ctx_lo=ctx_lo, ctx_hi=ctx_hi,
        pool_blocks=pool_blocks, max_blocks_per_seq=max_blocks_per_seq, block_size=block_size,
        shuffle_seq_ids=shuffle_seq_ids)
    device = torch.device(device)
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    if cache is None:
        shape = (pool_blocks, num_layers, num_kv_heads, block_size, head_dim)
        k_cache = torch.randn(shape, generator=gen, device=device, dtype=torch.float16)
        v_cache = torch.randn(shape, generator=gen, device=device, dtype=torch.float16)
    else:
        k_cache, v_cache = cache
    q = torch.randn((len(seq_ids), num_q_heads, head_dim), generator=gen, device=device, dtype=torch.float16)
    return PagedBatch(
        q=q, k_cache=k_cache, v_cache=v_cache,
        block_table=torch.from_numpy(table).to(device),
        seq_ids=torch.tensor(seq_ids, dtype=torch.int32, device=device),
        seq_lens=torch.tensor(seq_lens, dtype=torch.int32, device=device),
        seq_ids_list=seq_ids, seq_lens_list=seq_lens, ctx=ctx, depths=depths,
        cur_layer=cur_layer, num_q_heads=num_q_heads, num_kv_heads=num_kv_heads)


# Benchmark configurations (shapes only; see the docstring).
CONFIGS = {
    # config 1: CPU reference-path verify, Qwen3-0.6B shape
    "cpu_verify_0p6b": dict(num_requests=4, depth=4, ctx_lo=64, ctx_hi=256, num_q_heads=16,
                            num_kv_heads=8, pool_blocks=256),
    # config 2: Draft decode, Qwen3-0.6B shape (28 layers)
    "draft_decode_0p6b": dict(num_requests=64, depth=0, ctx_lo=128, ctx_hi=2048, num_q_heads=16,
                              num_kv_heads=8, pool_blocks=24576, num_layers=28),
    # config 3: Target verify, Qwen3-8B shape (36 layers) -- the headline metric
    "target_verify_8b": dict(num_requests=16, depth=4, ctx_lo=256, ctx_hi=4096, num_q_heads=32,
                             num_kv_heads=8, pool_blocks=24576, num_layers=36),
    # config 4: long-context verify stress, one-layer cache
    "long_verify_8b_k4": dict(num_requests=64, depth=4, ctx_lo=8192, ctx_hi=32768, num_q_heads=32,
                              num_kv_heads=8, pool_blocks=132 * 1024, num_layers=1),
    "long_verify_8b_k8": dict(num_requests=64, depth=8, ctx_lo=8192, ctx_hi=32768, num_q_heads=32,
                              num_kv_heads=8, pool_blocks=132 * 1024, num_layers=1),
}


def decode_infer_state(seq_lens, seq_ids, seq_lens_list, num_kv_heads: int, softmax_scale: float):
    """An ``infer_state`` with the fields the attention ops read, for decode/verify rows only.

    Mirrors what ``LlamaModel.forward`` builds (``swiftLLM/swiftllm/worker/model.py:402-430``)
    for a batch without prefill rows, including the reference's split-K choice
    (``model.py:380-384``), which the drop-in ops accept and ignore.
    """
    import types
    sbs = 2048
    total, max_len = sum(seq_lens_list), max(seq_lens_list)
    while num_kv_heads * (total / sbs) < 1024 and sbs // 2 >= 64 and max_len / (sbs // 2) <= 128:
        sbs //= 2
    return types.SimpleNamespace(
        num_decoding_seqs=len(seq_lens_list), num_prefill_seqs=0, num_prefill_tokens=0,
        decoding_seq_lens=seq_lens, seq_ids=seq_ids, softmax_scale=softmax_scale,
        seq_block_size=sbs, num_seq_blocks=(max_len + sbs - 1) // sbs, max_decoding_len=max_len,
        ignore_kvcache=False)
