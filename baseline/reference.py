"""Loader of the reference's own code, installed under ``baseline/_ref``.

``baseline/_ref`` holds the unmodified NebulaSD packages (``swiftllm`` and
``nebulasd``), installed from the reference checkout with

    python -m pip install --no-index --no-build-isolation --no-deps \\
        --find-links /opt/wheelhouse --target baseline/_ref <copy>/swiftLLM <copy>/nebulasd

(built from a copy under /tmp because the checkout is read-only).  The
directory is git-ignored but travels with the repository to the GPU box, where
it serves three purposes: the reference's Triton kernels JIT-compiled on the
same B200 as the bar in ``bench.py``, the reference's ``LlamaModel`` as the
accept-identity check, and the reference's HostKV arena / copy executor as
the real objects ``NativeCopyBackend`` is dropped into.  Nothing in the
product (``nebulasd_b200``) imports this module.

``swiftllm/__init__.py`` imports the serving stack (``ray`` and the compiled
``swiftllm_c`` extension), which the kernels and the model do not use, so the
package is mounted as a namespace module and ``swiftllm_c`` gets an empty
stand-in (only ``LlamaModel._swap``, CPU swapping, calls it).
"""
from __future__ import annotations

import importlib
import sys
import types
from pathlib import Path

REF = Path(__file__).resolve().parent / "_ref"


def available() -> bool:
    """True when the reference packages are installed under ``baseline/_ref``."""
    return (REF / "swiftllm" / "worker" / "kernels" / "paged_attn.py").exists() and \
        (REF / "nebulasd" / "kv" / "arena.py").exists()


def _mount() -> None:
    if not available():
        raise ImportError(f"the reference is not installed under {REF}")
    mod = sys.modules.get("swiftllm")
    if mod is None or list(getattr(mod, "__path__", [])) != [str(REF / "swiftllm")]:
        mod = types.ModuleType("swiftllm")
        mod.__path__ = [str(REF / "swiftllm")]
        sys.modules["swiftllm"] = mod
    if "swiftllm_c" not in sys.modules:
        sys.modules["swiftllm_c"] = types.ModuleType("swiftllm_c")
    if str(REF) not in sys.path:
        sys.path.append(str(REF))


def swiftllm(name: str):
    """Import ``swiftllm.<name>`` from the installed reference (e.g. ``worker.kernels.paged_attn``)."""
    _mount()
    return importlib.import_module(f"swiftllm.{name}")


def nebulasd(name: str):
    """Import ``nebulasd.<name>`` from the installed reference (e.g. ``kv.arena``)."""
    _mount()
    return importlib.import_module(f"nebulasd.{name}")


# Qwen3 shapes (random weights; the vocabulary is the real 151,936 tokens).
QWEN3_0P6B = {"model_type": "qwen3", "num_hidden_layers": 28, "num_attention_heads": 16,
              "num_key_value_heads": 8, "hidden_size": 1024, "head_dim": 128, "vocab_size": 151936,
              "max_position_embeddings": 40960, "intermediate_size": 3072, "rope_theta": 1000000.0,
              "rms_norm_eps": 1e-6, "hidden_act": "silu"}
QWEN3_8B = {"model_type": "qwen3", "num_hidden_layers": 36, "num_attention_heads": 32,
            "num_key_value_heads": 8, "hidden_size": 4096, "head_dim": 128, "vocab_size": 151936,
            "max_position_embeddings": 40960, "intermediate_size": 12288, "rope_theta": 1000000.0,
            "rms_norm_eps": 1e-6, "hidden_act": "silu"}


def random_llama(config: dict, directory, seed: int, *, max_seqs: int, max_blocks_per_seq: int,
                 num_blocks: int, max_batch: int, max_tokens: int):
    """The reference's ``LlamaModel`` (``swiftLLM/swiftllm/worker/model.py``)
    with random weights: projections N(0, 1/fan_in), norms N(1, 0.02), unit
    embeddings, so activations and logits keep unit scale; a paged KV cache of
    ``num_blocks`` blocks the caller indexes with its own block table."""
    import json

    import torch
    path = Path(directory)
    path.mkdir(parents=True, exist_ok=True)
    (path / "config.json").write_text(json.dumps(config))
    model_mod, engine_mod = swiftllm("worker.model"), swiftllm("engine_config")
    ec = engine_mod.EngineConfig(model_path=str(path), use_dummy=True, block_size=16, gpu_mem_utilization=0.9,
                                 num_cpu_blocks=1, max_seqs_in_block_table=max_seqs,
                                 max_blocks_per_seq=max_blocks_per_seq, max_batch_size=max_batch,
                                 max_tokens_in_batch=max_tokens)
    m = model_mod.LlamaModel(ec)
    with torch.inference_mode():
        m.load_weights()
        gen = torch.Generator(device="cuda").manual_seed(seed)

        def fill(t):
            if t.dim() == 1:
                t.copy_(1 + 0.02 * torch.randn(t.shape, generator=gen, device=t.device))
            else:
                t.copy_(torch.randn(t.shape, generator=gen, device=t.device) * t.shape[1] ** -0.5)
        w = m.weight
        fill(w.lm_head)
        fill(w.final_norm)
        w.wte.copy_(torch.randn(w.wte.shape, generator=gen, device=w.wte.device))
        for layer in w.layers:
            for t in vars(layer).values():
                if torch.is_tensor(t) and t.is_floating_point():
                    fill(t)
        m.init_kvcache_and_swap(num_blocks, external_layout=True)
    return m
