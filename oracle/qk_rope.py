"""Restatement of Qwen3 QK-RMSNorm, RoPE and the RoPE tables (CPU, fp32 math).

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Reference:
  * RMSNorm ``swiftLLM/swiftllm/worker/kernels/rmsnorm.py:5-37``: per row,
    ``x32 * rsqrt(mean(x32^2) + eps) * w32`` stored as fp16.  Qwen3 applies it to
    every 128-wide head row of q and k (``worker/layers/transformer_layer.py:114-124``).
  * RoPE ``swiftLLM/swiftllm/worker/kernels/rotary_emb.py:7-58``: rotate-half on
    the two 64-halves, ``x0' = x0*cos - x1*sin``, ``x1' = x0*sin + x1*cos``, with
    per-token fp16 ``cos/sin`` rows (``infer_state.position_cos/sin``).
  * Tables ``swiftLLM/swiftllm/worker/model.py:232-252`` (scalar rope_scaling):
    ``inv_freq = 1/base^(arange(0,D,2)/D)``, ``freqs = outer(t, inv_freq)``,
    fp32 ``cos``/``sin`` cast to fp16; decode rows use position ``seq_len-1``
    (``model.py:343-354``).

The reference's RoPE multiplies and subtracts in fp16; this oracle computes it
in fp32 from the fp16 inputs and rounds once (the fp32 parity bar).  The
``rope_fp16`` variant repeats the reference's per-operation fp16 rounding for
the bit-level checks against the golden vectors.
"""
from __future__ import annotations

import torch


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """fp16 result of ``rmsnorm.py:14-24`` over the last dimension."""
    x32 = x.float()
    var = (x32 * x32).sum(-1, keepdim=True) / x.shape[-1]
    rstd = 1.0 / torch.sqrt(var + eps)
    return (x32 * rstd * w.float()).to(torch.float16)


def rope_tables(head_dim: int, base: float, max_positions: int, scaling: float = 1.0):
    """fp16 ``(cos, sin)`` tables ``[max_positions, head_dim // 2]`` (``model.py:243-252``)."""
    inv_freq = 1.0 / (base ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
    t = torch.arange(max_positions, dtype=torch.float32) / scaling
    freqs = torch.outer(t, inv_freq)
    return torch.cos(freqs).to(torch.float16), torch.sin(freqs).to(torch.float16)


def rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Rotate-half RoPE; ``x`` ``[T, heads, D]`` fp16, ``cos/sin`` ``[T, D/2]`` fp16; fp32 math."""
    half = x.shape[-1] // 2
    x0, x1 = x[..., :half].float(), x[..., half:].float()
    c, s = cos.float()[:, None, :], sin.float()[:, None, :]
    return torch.cat([x0 * c - x1 * s, x0 * s + x1 * c], dim=-1).to(torch.float16)


def rope_fp16(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """RoPE with every multiply/add rounded to fp16, as ``rotary_emb.py:36-42`` writes it."""
    half = x.shape[-1] // 2
    x0, x1 = x[..., :half].float(), x[..., half:].float()
    c, s = cos.float()[:, None, :], sin.float()[:, None, :]

    def r(t):
        return t.to(torch.float16).float()

    y0 = r(r(x0 * c) - r(x1 * s))
    y1 = r(r(x0 * s) + r(x1 * c))
    return torch.cat([y0, y1], dim=-1).to(torch.float16)


def qk_norm_rope(q, k, q_w, k_w, eps, cos, sin, fp16_rope: bool = False):
    """QK-RMSNorm then RoPE, the order of ``transformer_layer.py:114-131``."""
    qn = rmsnorm(q, q_w, eps)
    kn = rmsnorm(k, k_w, eps)
    f = rope_fp16 if fp16_rope else rope
    return f(qn, cos, sin), f(kn, cos, sin)
