"""Seeded inputs of the golden-vector cases (shared by the fixture script and the tests).

Each builder returns CPU tensors.  ``make_golden.py`` feeds them to the
reference's own kernels and stores the outputs; the tests rebuild the same
inputs, check their digest against the fixture, and compare.
"""
from __future__ import annotations

import hashlib
import math

import numpy as np
import torch

from nebulasd_b200.workloads import make_paged_batch


def digest(*tensors) -> str:
    h = hashlib.sha256()
    for t in tensors:
        if torch.is_tensor(t):
            h.update(t.detach().cpu().contiguous().view(torch.uint8).numpy().tobytes())
        else:
            h.update(np.ascontiguousarray(t).tobytes())
    return h.hexdigest()


def _batch_dict(b, scale=None):
    d = b.q.shape[-1]
    return dict(q=b.q, k_cache=b.k_cache, v_cache=b.v_cache, block_table=b.block_table,
                seq_ids=b.seq_ids, seq_lens=b.seq_lens, cur_layer=b.cur_layer,
                softmax_scale=scale if scale is not None else d ** -0.5,
                num_q_heads=b.num_q_heads, num_kv_heads=b.num_kv_heads)


def attention_cases():
    """name -> input dict for ``paged_attention`` golden cases."""
    cases = {}
    # Config 1 (Qwen3-0.6B verify shape, k=4, random-permutation table from a 256-block pool);
    # two layers so that the layer stride is exercised.
    b = make_paged_batch(101, num_requests=4, depth=4, ctx_lo=64, ctx_hi=256, num_q_heads=16,
                         num_kv_heads=8, pool_blocks=256, num_layers=2, cur_layer=1)
    cases["verify_cfg1"] = _batch_dict(b)
    # Plain decode rows with edge lengths (1 token, block edges, ragged tail), GQA 2.
    b = make_paged_batch(202, num_requests=6, depth=0, ctx_lo=0, ctx_hi=0, num_q_heads=16,
                         num_kv_heads=8, pool_blocks=96, num_layers=1, cur_layer=0,
                         max_blocks_per_seq=17)
    lens = [1, 15, 16, 17, 200, 255]
    bt = torch.full((6, 17), -1, dtype=torch.int32)
    rng = np.random.default_rng(203)
    perm = rng.permutation(96)
    used = 0
    for i, n in enumerate(lens):
        nb = math.ceil(n / 16)
        bt[i, :nb] = torch.from_numpy(perm[used:used + nb].astype(np.int32))
        used += nb
    cases["decode_edges"] = dict(_batch_dict(b), block_table=bt,
                                 seq_lens=torch.tensor(lens, dtype=torch.int32))
    # Qwen3-8B head shape (GQA 4) at depth 8, two requests.
    b = make_paged_batch(303, num_requests=2, depth=8, ctx_lo=20, ctx_hi=120, num_q_heads=32,
                         num_kv_heads=8, pool_blocks=64, num_layers=1, cur_layer=0)
    cases["verify_gqa4_k8"] = _batch_dict(b)
    # Ragged depths in one batch (0, 2, 4, 7), shuffled table rows, three layers.
    b = make_paged_batch(404, num_requests=4, depth=[0, 2, 4, 7], ctx_lo=1, ctx_hi=90,
                         num_q_heads=32, num_kv_heads=8, pool_blocks=64, num_layers=3, cur_layer=2,
                         shuffle_seq_ids=True)
    cases["verify_ragged"] = _batch_dict(b)
    return cases


def store_case():
    """Inputs for ``store_kvcache`` with 2 prefill sequences and 5 decode rows."""
    g = torch.Generator().manual_seed(505)
    nb, layers, hk, bs, d = 40, 2, 2, 16, 128
    k_cache = torch.randn((nb, layers, hk, bs, d), generator=g).half()
    v_cache = torch.randn((nb, layers, hk, bs, d), generator=g).half()
    prefill_lens = [21, 7]
    decode_lens = [1, 16, 17, 33, 40]
    seq_ids = [3, 0, 1, 4, 2, 5, 6]           # prefill seqs first, then decode rows
    table = torch.full((7, 4), -1, dtype=torch.int32)
    perm = torch.randperm(nb, generator=g).int()
    used = 0
    for sid, n in zip(seq_ids, prefill_lens + decode_lens):
        c = math.ceil(n / bs)
        table[sid, :c] = perm[used:used + c]
        used += c
    ntok = sum(prefill_lens) + len(decode_lens)
    k = torch.randn((ntok, hk, d), generator=g).half()
    v = torch.randn((ntok, hk, d), generator=g).half()
    return dict(k=k, v=v, k_cache=k_cache, v_cache=v_cache, block_table=table,
                seq_ids=torch.tensor(seq_ids, dtype=torch.int32),
                prefill_lens=prefill_lens, decode_lens=decode_lens, cur_layer=1)


def norm_rope_case():
    """Inputs for Qwen3 QK-RMSNorm + RoPE (Qwen3-8B head counts, 5 tokens)."""
    g = torch.Generator().manual_seed(606)
    t, h, hk, d = 5, 32, 8, 128
    q = (torch.randn((t, h, d), generator=g) * 3).half()
    k = (torch.randn((t, hk, d), generator=g) * 3).half()
    q_w = (1 + 0.02 * torch.randn((d,), generator=g)).half()
    k_w = (1 + 0.02 * torch.randn((d,), generator=g)).half()
    positions = torch.tensor([0, 1, 700, 4095, 30000])
    return dict(q=q, k=k, q_w=q_w, k_w=k_w, eps=1e-6, positions=positions, theta=1e6)


def prefill_case():
    """Inputs for causal prefill attention: six prompts (one empty) of 0-129
    tokens, 4 q heads over 1 kv head (ratio 4), head dim 128."""
    g = torch.Generator().manual_seed(707)
    lens = [1, 17, 40, 129, 0, 33]
    t, h, hk, d = sum(lens), 4, 1, 128
    q = torch.randn((t, h, d), generator=g).half()
    k = torch.randn((t, hk, d), generator=g).half()
    v = torch.randn((t, hk, d), generator=g).half()
    cu = torch.tensor([0] + np.cumsum(lens).tolist(), dtype=torch.int32)
    return dict(q=q, k=k, v=v, cu_seqlens=cu, max_seqlen=max(lens), softmax_scale=d ** -0.5)
