"""CPU: ``install()`` routes the reference's names to this package (stand-in
modules under the reference's import paths; no GPU, no reference install)."""
import sys
import types

import pytest

_PATHS = ("swiftllm.worker.kernels.paged_attn", "swiftllm.worker.kernels.kvcache_mgmt",
          "swiftllm.worker.kernels.rotary_emb", "swiftllm.worker.kernels.rmsnorm",
          "swiftllm.worker.layers.transformer_layer", "nebulasd.kv.cuda_transfer")


@pytest.fixture
def fake_reference():
    saved = {p: sys.modules.get(p) for p in _PATHS}

    def original(*a, **k):
        raise AssertionError("the reference's function ran")

    mods = {}
    for p in _PATHS:
        m = types.ModuleType(p)
        mods[p] = m
        sys.modules[p] = m
    mods["swiftllm.worker.kernels.paged_attn"].paged_attention = original
    mods["swiftllm.worker.kernels.kvcache_mgmt"].store_kvcache = original
    mods["swiftllm.worker.kernels.rotary_emb"].rotary_embedding_inplace = original
    mods["swiftllm.worker.kernels.rmsnorm"].rmsnorm_inplace = original
    mods["swiftllm.worker.kernels.rmsnorm"].fused_add_rmsnorm_inplace = original
    layer = mods["swiftllm.worker.layers.transformer_layer"]
    for n in ("paged_attention", "store_kvcache", "rotary_embedding_inplace", "rmsnorm_inplace",
              "fused_add_rmsnorm_inplace", "flash_attn_varlen_func", "linear"):
        setattr(layer, n, original)
    mods["nebulasd.kv.cuda_transfer"].CudaCopyBackend = object
    yield mods, original
    for p, m in saved.items():
        if m is None:
            sys.modules.pop(p, None)
        else:
            sys.modules[p] = m


def test_install_routes_the_hot_path_and_leaves_the_rest(fake_reference):
    mods, original = fake_reference
    import nebulasd_b200
    from nebulasd_b200 import kernels
    from nebulasd_b200.hostkv import NativeCopyBackend
    nebulasd_b200.install()
    layer = mods["swiftllm.worker.layers.transformer_layer"]
    assert layer.paged_attention is kernels.paged_attention
    assert layer.store_kvcache is kernels.store_kvcache
    assert layer.rotary_embedding_inplace is kernels.rotary_embedding_inplace
    assert layer.rmsnorm_inplace is kernels.rmsnorm_inplace
    assert layer.flash_attn_varlen_func is kernels.flash_attn_varlen_func
    assert mods["swiftllm.worker.kernels.paged_attn"].paged_attention is kernels.paged_attention
    assert mods["nebulasd.kv.cuda_transfer"].CudaCopyBackend is NativeCopyBackend
    # names outside the hot path stay the reference's
    assert layer.fused_add_rmsnorm_inplace is original and layer.linear is original
    assert mods["swiftllm.worker.kernels.rmsnorm"].fused_add_rmsnorm_inplace is original
