"""GPU: causal prefill attention over packed variable-length sequences (the
drop-in for ``flash_attn_varlen_func``, ``transformer_layer.py:7-32``) against
the oracle's fp32 per-prompt restatement (``oracle/prefill.py``), the golden
fixture made from the reference's own function, and that function itself.
Tolerance: |ours - fp32| <= 2e-3 + 1e-2 |fp32| (fp16 P and output)."""
import pytest
import torch

from baseline import reference as R
from oracle.prefill import prefill_attention

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-3, 1e-2


def _case(lens, heads, kv_heads, seed, dev, q_pad=0):
    g = torch.Generator().manual_seed(seed)
    t = sum(lens)
    qbig = torch.randn((t, heads + q_pad, 128), generator=g).half().to(dev)
    q = qbig[:, :heads]  # token stride (heads + q_pad) * 128 when padded
    k = torch.randn((t, kv_heads, 128), generator=g).half().to(dev)
    v = torch.randn((t, kv_heads, 128), generator=g).half().to(dev)
    cu = torch.tensor([0] + torch.cumsum(torch.tensor(lens), 0).tolist(), dtype=torch.int32, device=dev)
    return q, k, v, cu


def _fp32(q, k, v, cu, scale):
    return prefill_attention(q, k, v, cu, scale)


def test_matches_the_golden_fixture(cuda):
    """The seeded inputs of the fixture made from the reference's own function."""
    import numpy as np
    from nebulasd_b200.kernels import flash_attn_varlen_func
    from tests.golden import cases as C
    p = C.prefill_case()
    g = np.load(C.__file__.rsplit("/", 1)[0] + "/prefill.npz")
    assert str(g["input_sha256"]) == C.digest(p["q"], p["k"], p["v"], p["cu_seqlens"])
    out = flash_attn_varlen_func(p["q"].to(cuda), p["k"].to(cuda), p["v"].to(cuda), p["cu_seqlens"].to(cuda),
                                 p["cu_seqlens"].to(cuda), p["max_seqlen"], p["max_seqlen"],
                                 softmax_scale=p["softmax_scale"], causal=True)
    torch.testing.assert_close(out.float().cpu(), torch.from_numpy(g["o"]).float(), atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("lens,heads,kv_heads", [
    ([1, 15, 16, 17, 100, 513], 32, 8),        # Qwen3-8B heads (ratio 4), ragged incl. block edges
    ([127, 128, 129, 255, 256, 257], 32, 8),   # key-tile edges
    ([300, 7, 1024, 64], 16, 8),               # Qwen3-0.6B heads (ratio 2)
    ([2500, 300, 0, 41], 32, 8),               # an empty sequence; more rows than one verify call takes
    ([5, 700], 8, 8),                          # ratio 1
    ([333, 64, 9], 64, 8),                     # ratio 8
    ([200, 31], 32, 2),                        # ratio 16
    ([77, 400], 24, 8),                        # ratio 3: the verify-kernel path
])
def test_matches_fp32_reference(lens, heads, kv_heads, cuda):
    from nebulasd_b200.kernels import flash_attn_varlen_func
    q, k, v, cu = _case(lens, heads, kv_heads, sum(lens) + heads, cuda)
    scale = 128 ** -0.5
    out = flash_attn_varlen_func(q, k, v, cu, cu, max(lens), max(lens), softmax_scale=scale, causal=True)
    torch.testing.assert_close(out.float(), _fp32(q, k, v, cu, scale), atol=ATOL, rtol=RTOL)


def test_many_short_prompts_and_a_strided_q(cuda):
    from nebulasd_b200.kernels import flash_attn_varlen_func
    g = torch.Generator().manual_seed(5)
    lens = torch.randint(1, 60, (300,), generator=g).tolist() + [1500]
    q, k, v, cu = _case(lens, 32, 8, 11, cuda, q_pad=8)
    assert q.stride(0) == 40 * 128
    scale = 0.1
    out = flash_attn_varlen_func(q, k, v, cu, cu, max(lens), max(lens), softmax_scale=scale, causal=True)
    torch.testing.assert_close(out.float(), _fp32(q, k, v, cu, scale), atol=ATOL, rtol=RTOL)


def test_a_thousand_tiny_prompts_with_a_loose_max_seqlen(cuda):
    """The plan orders 1,000 prompts of 1-8 tokens (many units per level) and
    takes a max_seqlen far above the real lengths (empty levels)."""
    from nebulasd_b200.kernels import flash_attn_varlen_func
    g = torch.Generator().manual_seed(9)
    lens = torch.randint(1, 9, (1000,), generator=g).tolist()
    q, k, v, cu = _case(lens, 32, 8, 21, cuda)
    out = flash_attn_varlen_func(q, k, v, cu, cu, 4096, 4096, softmax_scale=0.1, causal=True)
    torch.testing.assert_close(out.float(), _fp32(q, k, v, cu, 0.1), atol=ATOL, rtol=RTOL)


def test_long_prompt_at_the_draft_ratio(cuda):
    """Qwen3-0.6B heads (16 q / 8 kv, 64 tokens per unit), one 3,000-token prompt and a short one."""
    from nebulasd_b200.kernels import flash_attn_varlen_func
    lens = [3000, 70]
    q, k, v, cu = _case(lens, 16, 8, 33, cuda)
    out = flash_attn_varlen_func(q, k, v, cu, cu, max(lens), max(lens), softmax_scale=128 ** -0.5, causal=True)
    torch.testing.assert_close(out.float(), _fp32(q, k, v, cu, 128 ** -0.5), atol=ATOL, rtol=RTOL)


def test_large_scores_move_the_running_max(cuda):
    """Scores whose row max grows along the keys (rescaled O) and spans > 2^8 in exp2."""
    from nebulasd_b200.kernels import flash_attn_varlen_func
    lens = [1000, 600]
    q, k, v, cu = _case(lens, 32, 8, 3, cuda)
    ramp = torch.linspace(0.2, 3.0, sum(lens), device=cuda).half()[:, None, None]
    k = (k * ramp).contiguous()
    scale = 0.3
    out = flash_attn_varlen_func(q, k, v, cu, cu, max(lens), max(lens), softmax_scale=scale, causal=True)
    torch.testing.assert_close(out.float(), _fp32(q, k, v, cu, scale), atol=ATOL, rtol=RTOL)


def test_invalid_cu_seqlens_is_reported(cuda):
    from nebulasd_b200.kernels import flash_attn_varlen_func
    from nebulasd_b200.kernels.prefill import workspace_errors
    q, k, v, _ = _case([20], 32, 8, 1, cuda)
    assert workspace_errors() == 0
    # sequence 1 ends past the tokens, sequence 2 has a negative length: both left out
    bad = torch.tensor([0, 10, 30, 20], dtype=torch.int32, device=cuda)
    out = flash_attn_varlen_func(q, k, v, bad, bad, 20, 20)
    assert workspace_errors() & (1 << 5)
    # the valid sequence is still computed
    ref = _fp32(q, k, v, torch.tensor([0, 10], dtype=torch.int32, device=cuda), 128 ** -0.5)
    torch.testing.assert_close(out[:10].float(), ref[:10], atol=ATOL, rtol=RTOL)
    longer = torch.tensor([0, 20], dtype=torch.int32, device=cuda)
    flash_attn_varlen_func(q, k, v, longer, longer, 8, 8)  # max_seqlen below the real length
    assert workspace_errors() & (1 << 5)
    assert workspace_errors() == 0


@pytest.mark.skipif(not R.available(), reason="reference not installed under baseline/_ref")
def test_matches_the_reference_function(cuda):
    from nebulasd_b200.kernels import flash_attn_varlen_func
    ref_fn = R.swiftllm("worker.layers.transformer_layer").flash_attn_varlen_func
    assert ref_fn.__module__.startswith("swiftllm."), "another test left install() in place"
    lens = [129, 700, 33, 1000]
    q, k, v, cu = _case(lens, 32, 8, 7, cuda)
    scale = 128 ** -0.5
    ours = flash_attn_varlen_func(q, k, v, cu, cu, max(lens), max(lens), softmax_scale=scale, causal=True)
    theirs = ref_fn(q, k, v, cu, cu, max(lens), max(lens), softmax_scale=scale, causal=True)
    torch.testing.assert_close(ours.float(), theirs.float(), atol=4e-3, rtol=1e-2)
