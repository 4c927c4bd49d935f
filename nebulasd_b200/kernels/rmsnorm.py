"""RMSNorm behind the reference's ``rmsnorm_inplace`` signature.

Replaces ``swiftLLM/swiftllm/worker/kernels/rmsnorm.py:26-37``:
``x = fp16(x32 * (1 / sqrt(mean(x32^2) + eps)) * w32)`` per row, in place.
On the attention path it is the Qwen3 QK-norm over 128-wide head rows
(``worker/layers/transformer_layer.py:114-124``); ``qk_norm_rope_store`` fuses
it with RoPE and the KV store.
"""
from __future__ import annotations

import torch

from .. import _lib


def rmsnorm_inplace(input_and_output: torch.Tensor, weight: torch.Tensor, eps: float) -> None:
    x = input_and_output
    if x.dtype != torch.float16 or weight.dtype != torch.float16:
        raise TypeError("rmsnorm_inplace expects float16 input and weight")
    if x.dim() != 2 or x.stride(1) != 1 or x.stride(0) != x.shape[1]:
        raise ValueError("rmsnorm_inplace expects a contiguous [rows, hidden] tensor")
    rc = _lib.lib.neb_rmsnorm_inplace(x.data_ptr(), weight.data_ptr(), x.shape[0], x.shape[1], float(eps),
                                      torch.cuda.current_stream(x.device).cuda_stream)
    _lib.check(rc, "rmsnorm_inplace")
