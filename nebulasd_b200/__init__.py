"""B200-native (sm_100a) attention hot path for NebulaSD's swiftLLM backend.

Ops (``nebulasd_b200.kernels``), with the reference's names and signatures:
  * ``paged_attention``          decode (CUDA cores) and verify (tcgen05) kernels
  * ``store_kvcache``            paged KV store
  * ``rotary_embedding_inplace`` RoPE
  * ``rmsnorm_inplace``          RMSNorm (Qwen3 QK-norm)
  * ``qk_norm_rope_store``       the last three fused into one launch
  * ``flash_attn_varlen_func``   causal prefill attention (verify kernel, no host sync)
HostKV (``nebulasd_b200.hostkv``): ``NativeCopyBackend`` for restore/writeback,
``migrate_blocks`` for same-role peer migration.

``install()`` aliases the ops under the reference's module paths so that
``LlamaTransformerLayer`` and the NebulaSD workers pick them up unchanged.
"""
from __future__ import annotations

import sys

__version__ = "0.1.0"

_ALIASES = {
    "swiftllm.worker.kernels.paged_attn": ("paged_attention",),
    "swiftllm.worker.kernels.kvcache_mgmt": ("store_kvcache",),
    "swiftllm.worker.kernels.rotary_emb": ("rotary_embedding_inplace",),
    "swiftllm.worker.kernels.rmsnorm": ("rmsnorm_inplace",),
}


def install() -> None:
    """Route the reference's attention ops to this package.

    Patches the attributes of the reference modules that are already imported:
    the kernel modules' functions, ``swiftllm.worker.layers.transformer_layer``'s
    module-level names (which it binds at import) including its own
    ``flash_attn_varlen_func``, and ``nebulasd.kv.cuda_transfer.CudaCopyBackend``.
    Modules not yet imported are left alone, so call it after importing the
    reference.  Only these names change; everything else in those modules (e.g.
    ``fused_add_rmsnorm_inplace``) stays the reference's.
    """
    from . import kernels
    for mod_name, names in _ALIASES.items():
        mod = sys.modules.get(mod_name)
        if mod is None:
            continue
        for n in names:
            setattr(mod, n, getattr(kernels, n))
    layer = sys.modules.get("swiftllm.worker.layers.transformer_layer")
    if layer is not None:
        for names in _ALIASES.values():
            for n in names:
                if hasattr(layer, n):
                    setattr(layer, n, getattr(kernels, n))
        # The prefill attention the layer module defines itself
        # (transformer_layer.py:7-32): a per-sequence loop with a host sync.
        if hasattr(layer, "flash_attn_varlen_func"):
            layer.flash_attn_varlen_func = kernels.flash_attn_varlen_func
    kv = sys.modules.get("nebulasd.kv.cuda_transfer")
    if kv is not None:
        from .hostkv import NativeCopyBackend
        kv.CudaCopyBackend = NativeCopyBackend
