"""Drop-in replacements for ``swiftllm.worker.kernels`` on the attention hot path.

Module and function names, argument order and meaning follow the reference
(``swiftLLM/swiftllm/worker/kernels/{paged_attn,kvcache_mgmt,rotary_emb,rmsnorm}.py``),
so ``nebulasd_b200.install()`` can alias them under the reference's import
paths and ``LlamaTransformerLayer`` runs unchanged on top of them.
"""
from .paged_attn import paged_attention, paged_attention_raw  # noqa: F401
from .kvcache_mgmt import store_kvcache  # noqa: F401
from .rotary_emb import rotary_embedding_inplace  # noqa: F401
from .rmsnorm import rmsnorm_inplace  # noqa: F401
from .fused import qk_norm_rope_store  # noqa: F401
from .prefill import flash_attn_varlen_func  # noqa: F401
