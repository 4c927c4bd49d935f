"""GPU: greedy-accept identity through the reference's own model.

A random-init Qwen3-8B-shaped Target (32 q / 8 kv heads, head dim 128, hidden
4096, QK-norm, RoPE theta 1e6, the real 151,936-token vocabulary; four
layers) is built with the reference's ``LlamaModel``
(``swiftLLM/swiftllm/worker/model.py``) and prefilled with its own kernels.
Drafts are made so that the reference's greedy verification accepts a chosen
prefix of each request's four proposals.  The same verify forward (k+1 = 5 rows
per request, ``LlamaModel.forward`` -> ``LlamaTransformerLayer.forward``,
``transformer_layer.py:83-185``, with its piggyback attention stream and
events) then runs twice from one snapshot of the KV cache: with the
reference's Triton kernels, and after ``nebulasd_b200.install()`` routed
QK-norm, RoPE, the KV store and paged attention to this package.  The argmax
tokens and the decisions of the reference's ``compute_greedy_acceptance``
(``swiftLLM/swiftllm/speculative.py:122-156``) must agree.

Two implementations that round differently can only disagree where the
reference's own top two logits are closer than the numerical noise of either
(the reference sums its dot products in fp16).  The test computes each row's
top-2 gap in fp32 from the reference's final hidden state and reports the rows
within ``NEAR_TIE`` of a tie; decisions that depend on none of them must be
identical, and every decision is reported.  The reference packages come from
``baseline/_ref``; without them the test skips.
"""
import json
import sys

import pytest
import torch

from baseline import reference as R

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not R.available(), reason="reference not installed under baseline/_ref")]

LAYERS = 4
NUM_REQ = 16
DEPTH = 4
NEAR_TIE = 0.02  # logit units; the logits of this model have unit scale
SEEDS = (1, 2, 3)

QWEN3_8B = {"model_type": "qwen3", "num_hidden_layers": LAYERS, "num_attention_heads": 32,
            "num_key_value_heads": 8, "hidden_size": 4096, "head_dim": 128, "vocab_size": 151936,
            "max_position_embeddings": 40960, "intermediate_size": 12288, "rope_theta": 1000000.0,
            "rms_norm_eps": 1e-6, "hidden_act": "silu"}

_PATCHED = ("paged_attention", "store_kvcache", "rotary_embedding_inplace", "rmsnorm_inplace")


def _init_weights(weight, gen):
    """Random init with unit-scale activations: N(0, 1/fan_in) projections, norms N(1, 0.02)."""
    def fill(t):
        if t.dim() == 1:
            t.copy_(1 + 0.02 * torch.randn(t.shape, generator=gen, device=t.device))
        else:
            t.copy_(torch.randn(t.shape, generator=gen, device=t.device) * t.shape[1] ** -0.5)
    for name in ("lm_head", "final_norm"):
        fill(getattr(weight, name))
    weight.wte.copy_(torch.randn(weight.wte.shape, generator=gen, device=weight.wte.device))
    for layer in weight.layers:
        for t in vars(layer).values():
            if torch.is_tensor(t) and t.is_floating_point():
                fill(t)


@pytest.fixture(scope="module")
def model(tmp_path_factory, cuda):
    path = tmp_path_factory.mktemp("qwen3_8b_random")
    (path / "config.json").write_text(json.dumps(QWEN3_8B))
    model_mod = R.swiftllm("worker.model")
    engine_mod = R.swiftllm("engine_config")
    mbs = 128
    ec = engine_mod.EngineConfig(model_path=str(path), use_dummy=True, block_size=16, gpu_mem_utilization=0.9,
                                 num_cpu_blocks=1, max_seqs_in_block_table=NUM_REQ, max_blocks_per_seq=mbs,
                                 max_batch_size=NUM_REQ * (DEPTH + 1), max_tokens_in_batch=NUM_REQ * 2048)
    torch.cuda.set_device(cuda)
    m = model_mod.LlamaModel(ec)
    # The reference creates its weights and caches as inference tensors.
    with torch.inference_mode():
        m.load_weights()
        gen = torch.Generator(device=cuda).manual_seed(20261202)
        _init_weights(m.weight, gen)
        m.init_kvcache_and_swap(NUM_REQ * mbs, external_layout=True)
    return m


class _Kernels:
    """Routes the layer's four ops to nebulasd_b200 (install()) and back."""

    def __init__(self):
        self.layer_mod = R.swiftllm("worker.layers.transformer_layer")
        self.kernel_mods = {n: R.swiftllm(f"worker.kernels.{m}") for n, m in
                            (("paged_attention", "paged_attn"), ("store_kvcache", "kvcache_mgmt"),
                             ("rotary_embedding_inplace", "rotary_emb"), ("rmsnorm_inplace", "rmsnorm"))}
        self.saved = {n: (getattr(self.layer_mod, n), getattr(self.kernel_mods[n], n)) for n in _PATCHED}
        self.prefill = self.layer_mod.flash_attn_varlen_func
        self.copy_mod = sys.modules.get("nebulasd.kv.cuda_transfer")
        self.copy_backend = getattr(self.copy_mod, "CudaCopyBackend", None)

    def __enter__(self):
        import nebulasd_b200
        nebulasd_b200.install()
        assert self.layer_mod.paged_attention.__module__.startswith("nebulasd_b200")
        return self

    def __exit__(self, *exc):
        for n, (layer_fn, mod_fn) in self.saved.items():
            setattr(self.layer_mod, n, layer_fn)
            setattr(self.kernel_mods[n], n, mod_fn)
        self.layer_mod.flash_attn_varlen_func = self.prefill
        if self.copy_mod is not None:
            self.copy_mod.CudaCopyBackend = self.copy_backend
        return False


def _verify(m, rows, seq_ids, lens, bt):
    out = m.forward([[t] for t in rows], seq_ids, lens, kv_block_table=bt, return_dict=True, return_hidden=True)
    torch.cuda.synchronize()
    return out.token_ids, out.hidden_states


def _top2_gap(m, hidden):
    """fp32 logits of the final hidden rows (the post layer's RMSNorm and lm_head) and their top-2 gaps."""
    h = hidden.float()
    h = h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + m.model_config.rms_norm_eps) * m.weight.final_norm.float()
    top = (h @ m.weight.lm_head.float().t()).topk(2, dim=-1).values
    return (top[:, 0] - top[:, 1]).tolist()


@pytest.mark.parametrize("seed", SEEDS)
def test_greedy_accept_identity(model, seed, cuda):
    with torch.inference_mode():
        _accept_identity(model, seed, cuda)


def _accept_identity(model, seed, cuda):
    spec = R.swiftllm("speculative")
    m = model
    g = torch.Generator().manual_seed(seed)
    vocab = QWEN3_8B["vocab_size"]
    ctx = torch.randint(256, 1025, (NUM_REQ,), generator=g).tolist()
    prompts = [torch.randint(0, vocab, (c,), generator=g).tolist() for c in ctx]
    perm = torch.randperm(m.k_cache.shape[0], generator=g)
    need = [(c + DEPTH + 1 + 15) // 16 for c in ctx]
    bt = torch.full((NUM_REQ, m.engine_config.max_blocks_per_seq), -1, dtype=torch.int32)
    used = 0
    for r, n in enumerate(need):
        bt[r, :n] = perm[used:used + n]
        used += n
    bt = bt.to(cuda)
    seq_ids = list(range(NUM_REQ))
    anchors = m.forward(prompts, seq_ids, [], kv_block_table=bt)  # prefill, the reference's kernels
    torch.cuda.synchronize()
    # Verify rows: request r contributes [anchor, d1..d4] with lengths L+1..L+5.
    row_ids = [r for r in seq_ids for _ in range(DEPTH + 1)]
    row_lens = [ctx[r] + 1 + i for r in seq_ids for i in range(DEPTH + 1)]
    target = torch.randint(0, DEPTH + 1, (NUM_REQ,), generator=g).tolist()  # drafts the reference accepts
    drafts = [torch.randint(0, vocab, (DEPTH,), generator=g).tolist() for _ in seq_ids]
    snapshot = (m.k_cache.clone(), m.v_cache.clone())

    def rows_of(drafts_):
        return [t for r in seq_ids for t in [anchors[r]] + drafts_[r]]

    def restore():
        m.k_cache.copy_(snapshot[0])
        m.v_cache.copy_(snapshot[1])

    # Position i's posterior depends on the inputs up to row i only, so the
    # drafts are fixed one position at a time from the reference's argmax.
    for i in range(DEPTH):
        restore()
        post, _ = _verify(m, rows_of(drafts), row_ids, row_lens, bt)
        for r in seq_ids:
            if target[r] > i:
                drafts[r][i] = post[r * (DEPTH + 1) + i]
    restore()
    ref_post, ref_hidden = _verify(m, rows_of(drafts), row_ids, row_lens, bt)
    gaps = _top2_gap(m, ref_hidden)
    restore()
    with _Kernels():
        ours_post, ours_hidden = _verify(m, rows_of(drafts), row_ids, row_lens, bt)
    restore()

    identical, dependent_on_tie, mismatched = 0, 0, []
    for r in seq_ids:
        lo, hi = r * (DEPTH + 1), (r + 1) * (DEPTH + 1)
        ref_acc = spec.compute_greedy_acceptance(drafts[r], ref_post[lo:hi])
        our_acc = spec.compute_greedy_acceptance(drafts[r], ours_post[lo:hi])
        # The decision reads posteriors 0..accepted (the first mismatch or the bonus).
        decided = range(lo, lo + ref_acc[1] + 1)
        tie = any(gaps[j] < NEAR_TIE for j in decided)
        if ref_acc == our_acc:
            identical += 1
        else:
            mismatched.append((r, ref_acc, our_acc, [round(gaps[j], 4) for j in decided]))
        dependent_on_tie += tie
        assert ref_acc[1] >= min(target[r], DEPTH) or tie, \
            "the drafts were built so that the reference accepts its target prefix"
    diff = (ours_hidden.float() - ref_hidden.float()).abs().max().item()
    rows_same = sum(a == b for a, b in zip(ref_post, ours_post))
    print(f"seed {seed}: accept decisions identical {identical}/{NUM_REQ}, argmax rows identical "
          f"{rows_same}/{len(ref_post)}, decisions resting on a near-tie (< {NEAR_TIE}) {dependent_on_tie}, "
          f"min top-2 gap {min(gaps):.4f}, max |hidden diff| {diff:.3e}, mismatches {mismatched}")
    for r, ref_acc, our_acc, g_ in mismatched:
        assert min(g_) < NEAR_TIE, f"request {r}: accept decision differs without a near-tie: {ref_acc} vs {our_acc}"
