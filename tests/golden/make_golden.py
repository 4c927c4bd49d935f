"""Produce golden vectors by running the reference's own kernels on the CPU.

Usage (needs a NebulaSD checkout; nothing here runs on the GPU box):

    python tests/golden/make_golden.py --reference <NebulaSD checkout>

The reference kernels are OpenAI Triton; with ``TRITON_INTERPRET=1`` Triton
executes them in numpy on CPU tensors, so the vectors are the reference
implementation's own outputs on the seeded inputs of ``tests/golden/cases.py``.
The ``swiftllm`` package is mounted as a namespace module (its ``__init__``
imports the serving stack, which needs ``ray`` and a compiled extension that
the kernels themselves do not use).

The prefill fixture comes from the layer module's own ``flash_attn_varlen_func``
(plain PyTorch, run on the CPU); ``--only prefill`` regenerates just that one.

Outputs: ``tests/golden/<case>.npz`` holding the reference outputs, the sha256
of the inputs (so a test can prove it rebuilt identical inputs) and, for pure
byte work, only digests.
"""
from __future__ import annotations

import argparse
import os
import sys
import types
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

import numpy as np  # noqa: E402
import torch  # noqa: E402


def load_reference(root: Path):
    pkg_dir = root / "swiftLLM" / "swiftllm"
    mod = types.ModuleType("swiftllm")
    mod.__path__ = [str(pkg_dir)]
    sys.modules["swiftllm"] = mod
    from swiftllm.worker.kernels import paged_attn, kvcache_mgmt, rotary_emb, rmsnorm  # noqa: E402
    from swiftllm.worker.infer_state import LlamaInferState  # noqa: E402
    return paged_attn, kvcache_mgmt, rotary_emb, rmsnorm, LlamaInferState


def infer_state_for(LlamaInferState, *, seq_ids, decoding_seq_lens, num_prefill_seqs=0,
                    prefill_lens=(), softmax_scale, num_kv_heads, cos=None, sin=None):
    from oracle.attention import split_heuristic
    dec = [int(x) for x in decoding_seq_lens]
    sbs, nsb = split_heuristic(dec, num_kv_heads) if dec else (64, 0)
    pl = torch.tensor(list(prefill_lens), dtype=torch.int32)
    starts = torch.cumsum(pl, 0, dtype=torch.int32) - pl
    ntok = int(pl.sum()) + len(dec)
    return LlamaInferState(
        batch_size=num_prefill_seqs + len(dec), num_tokens=ntok,
        seq_ids=torch.as_tensor(seq_ids, dtype=torch.int32), softmax_scale=softmax_scale,
        num_prefill_seqs=num_prefill_seqs, num_prefill_tokens=int(pl.sum()),
        prefill_seq_start_locs=starts,
        prefill_seq_start_locs_with_end=torch.cat([starts, torch.tensor([ntok], dtype=torch.int32)]),
        prefill_seq_lens=pl, max_prefill_len=int(pl.max()) if len(pl) else 0,
        num_decoding_seqs=len(dec), decoding_seq_lens=torch.tensor(dec, dtype=torch.int32),
        max_decoding_len=max(dec) if dec else 0, seq_block_size=sbs, num_seq_blocks=nsb,
        position_cos=cos, position_sin=sin, ignore_kvcache=False)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, type=Path, help="NebulaSD project root")
    ap.add_argument("--only", choices=("all", "prefill"), default="all",
                    help="regenerate every fixture, or only prefill.npz")
    args = ap.parse_args()
    paged_attn, kvcache_mgmt, rotary_emb, rmsnorm, LlamaInferState = load_reference(args.reference)
    from tests.golden import cases as C
    from types import SimpleNamespace

    # Prefill: the layer module's own flash_attn_varlen_func (transformer_layer.py:7-32),
    # a per-prompt scaled_dot_product_attention, run here on the CPU in fp32 on the
    # fp16-valued inputs.
    from swiftllm.worker.layers import transformer_layer
    p = C.prefill_case()
    o = transformer_layer.flash_attn_varlen_func(p["q"].float(), p["k"].float(), p["v"].float(), p["cu_seqlens"],
                                                 p["cu_seqlens"], p["max_seqlen"], p["max_seqlen"],
                                                 softmax_scale=p["softmax_scale"], causal=True)
    np.savez(HERE / "prefill.npz", o=o.numpy().astype(np.float16),  # fp32 result, stored rounded to fp16
             input_sha256=C.digest(p["q"], p["k"], p["v"], p["cu_seqlens"]))
    print("prefill", tuple(o.shape))
    if args.only == "prefill":
        return

    for name, c in C.attention_cases().items():
        r, h, d = c["q"].shape
        mc = SimpleNamespace(num_q_heads=h, num_kv_heads=c["num_kv_heads"], head_dim=d,
                             num_layers=c["k_cache"].shape[1])
        ec = SimpleNamespace(block_size=16, max_blocks_per_seq=c["block_table"].shape[1])
        st = infer_state_for(LlamaInferState, seq_ids=c["seq_ids"], decoding_seq_lens=c["seq_lens"],
                             softmax_scale=c["softmax_scale"], num_kv_heads=c["num_kv_heads"])
        o = torch.empty_like(c["q"])
        paged_attn.paged_attention(c["q"], c["k_cache"], c["v_cache"], c["block_table"], mc, ec, st,
                                   c["cur_layer"], o)
        np.savez(HERE / f"{name}.npz", o=o.numpy(),
                 input_sha256=C.digest(c["q"], c["k_cache"], c["v_cache"], c["block_table"],
                                       c["seq_ids"], c["seq_lens"]),
                 seq_block_size=st.seq_block_size)
        print(name, tuple(o.shape), "seq_block_size", st.seq_block_size)

    s = C.store_case()
    in_sha = C.digest(s["k"], s["v"], s["k_cache"], s["v_cache"], s["block_table"], s["seq_ids"])
    kc, vc = s["k_cache"].clone(), s["v_cache"].clone()
    mc = SimpleNamespace(num_q_heads=2, num_kv_heads=2, head_dim=128, num_layers=kc.shape[1])
    ec = SimpleNamespace(block_size=16, max_blocks_per_seq=s["block_table"].shape[1])
    st = infer_state_for(LlamaInferState, seq_ids=s["seq_ids"], decoding_seq_lens=s["decode_lens"],
                         num_prefill_seqs=len(s["prefill_lens"]), prefill_lens=s["prefill_lens"],
                         softmax_scale=128 ** -0.5, num_kv_heads=2)
    kvcache_mgmt.store_kvcache(s["k"], s["v"], kc, vc, s["block_table"], mc, ec, st, s["cur_layer"])
    np.savez(HERE / "store_kvcache.npz", input_sha256=in_sha, k_cache_sha256=C.digest(kc),
             v_cache_sha256=C.digest(vc))
    print("store_kvcache", C.digest(kc)[:16])

    n = C.norm_rope_case()
    from oracle.qk_rope import rope_tables
    cos_t, sin_t = rope_tables(128, n["theta"], int(n["positions"].max()) + 1)
    cos, sin = cos_t[n["positions"]].contiguous(), sin_t[n["positions"]].contiguous()
    q, k = n["q"].clone(), n["k"].clone()
    rmsnorm.rmsnorm_inplace(q.view(-1, 128), n["q_w"], n["eps"])
    rmsnorm.rmsnorm_inplace(k.view(-1, 128), n["k_w"], n["eps"])
    q_norm, k_norm = q.clone(), k.clone()
    st = SimpleNamespace(position_cos=cos, position_sin=sin)
    rotary_emb.rotary_embedding_inplace(q, k, st)
    np.savez(HERE / "qk_norm_rope.npz",
             input_sha256=C.digest(n["q"], n["k"], n["q_w"], n["k_w"], cos, sin),
             q_norm=q_norm.numpy(), k_norm=k_norm.numpy(), q_rope=q.numpy(), k_rope=k.numpy(),
             cos=cos.numpy(), sin=sin.numpy())
    print("qk_norm_rope done")


if __name__ == "__main__":
    main()
