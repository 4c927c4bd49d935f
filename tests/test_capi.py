"""CPU: the C-ABI library loads, exports every declared symbol and validates arguments."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "nebula_b200.h"


def declared_symbols():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(neb_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_hot_path():
    names = declared_symbols()
    for must in ("neb_paged_attention_decode", "neb_paged_attention_verify", "neb_store_kvcache",
                 "neb_qk_norm_rope_store", "neb_rotary_inplace", "neb_rmsnorm_inplace", "neb_hostkv_copy",
                 "neb_greedy_accept", "neb_greedy_accept_workspace_bytes",
                 "neb_prefill_attention", "neb_prefill_attention_workspace_bytes",
                 "neb_kv_peer_copy"):
        assert must in names


def test_library_exports_every_declared_symbol():
    from nebulasd_b200 import _lib
    for name in declared_symbols():
        assert hasattr(_lib.lib, name), f"{name} declared in the header but not exported"
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_version_and_empty_error():
    from nebulasd_b200 import _lib
    assert _lib.lib.neb_version() >= 100
    assert isinstance(_lib.lib.neb_last_error(), bytes)


def _attn_args(**kw):
    a = dict(q=16, k=16, v=16, bt=16, bt_rows=4, mbs=8, lens=16, ids=16, rows=2, h=16, hk=8, d=128, bs=16,
             nb=64, layers=1, layer=0, scale=0.088, o=16, ws=256, wsb=1 << 20, stream=None)
    a.update(kw)
    return list(a.values())


@pytest.mark.parametrize("kw,msg", [
    (dict(d=64), b"head_dim must be 128"),
    (dict(bs=32), b"block_size must be 16"),
    (dict(h=12, hk=8), b"multiple of num_kv_heads"),
    (dict(layer=3, layers=2), b"cur_layer 3 outside"),
    (dict(rows=5000), b"num_rows must be in"),
    (dict(q=None), b"null tensor pointer"),
    (dict(q=8), b"16-byte aligned"),
    (dict(scale=0.0), b"softmax_scale must be positive"),
])
def test_attention_argument_validation_without_gpu(kw, msg):
    from nebulasd_b200 import _lib
    for fn in (_lib.lib.neb_paged_attention_decode, _lib.lib.neb_paged_attention_verify):
        rc = fn(*_attn_args(**kw))
        assert rc == 1 or rc == 2
        assert msg in _lib.lib.neb_last_error()


def test_zero_rows_is_a_no_op():
    from nebulasd_b200 import _lib
    assert _lib.lib.neb_paged_attention_decode(*_attn_args(rows=0)) == 0


def test_copy_validation_rejects_overlap_and_negative_ranges():
    from nebulasd_b200 import _lib
    import numpy as np
    regions = np.array([[0, 0, 4], [8, 2, 4]], dtype=np.int64)
    rc = _lib.lib.neb_hostkv_copy(1, 16, 16, 16, 16, 4096, regions.ctypes.data, 2, 0, None)
    assert rc == 1 and b"overlap" in _lib.lib.neb_last_error()
    regions = np.array([[0, -1, 4]], dtype=np.int64)
    rc = _lib.lib.neb_hostkv_copy(1, 16, 16, 16, 16, 4096, regions.ctypes.data, 1, 0, None)
    assert rc == 1 and b"negative" in _lib.lib.neb_last_error()
    rc = _lib.lib.neb_hostkv_copy(1, 16, 16, 16, 16, 4095, regions.ctypes.data, 1, 0, None)
    assert rc == 1 and b"multiple of 16" in _lib.lib.neb_last_error()


def test_store_and_rope_validation_without_gpu():
    from nebulasd_b200 import _lib
    rc = _lib.lib.neb_rotary_inplace(8, 8, 8, 8, 1, 4, 2, 64, None)
    assert rc == 2 and b"head_dim must be 128" in _lib.lib.neb_last_error()
    rc = _lib.lib.neb_rmsnorm_inplace(None, 8, 1, 128, 1e-6, None)
    assert rc == 1


def test_op_modules_import_without_gpu():
    import nebulasd_b200
    from nebulasd_b200 import kernels, hostkv  # noqa: F401
    assert callable(kernels.paged_attention) and callable(nebulasd_b200.install)


def test_copy_mode_choice_by_run_length():
    """auto mode: copy engines for long runs, the single-launch kernel for many short ones."""
    import numpy as np
    from nebulasd_b200.hostkv import ENGINE_RUN_BYTES, choose_copy_mode, host_runs, merged_runs
    block = 1_179_648  # Qwen3-8B HostKV block (36 layers x 8 kv heads x 16 x 128 x 2 B)
    long_runs = np.array([[0, 200, 253], [253, 453, 252]], dtype=np.int64)
    assert merged_runs(long_runs) == 1  # adjacent on both sides: one run per plane
    assert choose_copy_mode(long_runs, block, mapped=True) == "memcpy"
    # 64 one-block regions, none adjacent: 64 driver calls per plane for 75 MB.
    short = np.array([[2 * i, 3 * i, 1] for i in range(64)], dtype=np.int64)
    assert merged_runs(short) == 64
    assert choose_copy_mode(short, ENGINE_RUN_BYTES // 2, mapped=True) == "kernel"
    assert choose_copy_mode(short, block, mapped=True) == "memcpy"  # 1.18 MB per run is long enough
    assert choose_copy_mode(short, 4096, mapped=False) == "memcpy"  # unmapped arena: engines only
    assert choose_copy_mode(np.zeros((0, 3), dtype=np.int64), block, mapped=True) == "kernel"
    # A request's KV restored into a paged pool: one arena range, scattered GPU blocks.
    restore = np.stack([np.arange(256), np.arange(256) * 7 % 1021, np.ones(256, dtype=np.int64)], 1)
    assert host_runs(restore) == 1 and merged_runs(restore) == 256
    assert choose_copy_mode(restore, 32768, mapped=True) == "staged"
    assert choose_copy_mode(restore, 32768, mapped=False) == "staged"
    assert choose_copy_mode(restore, 32768, mapped=True, direction="D2H") == "kernel"  # writebacks: direct
    assert choose_copy_mode(restore[:16], 32768, mapped=True) == "kernel"  # 512 KB in all: too short to stage


def test_staged_pieces_cover_the_plan_within_capacity():
    import numpy as np
    from nebulasd_b200.hostkv import staged_pieces
    rng = np.random.default_rng(3)
    counts = rng.integers(1, 9, 50)
    host = np.concatenate([[0], np.cumsum(counts)[:-1]])
    gpu = rng.permutation(2000)[:50] * 10
    regions = np.stack([host, gpu, counts], 1).astype(np.int64)
    pieces = staged_pieces(regions, 16)
    moved = []
    for dma, scatter in pieces:
        assert (dma[:, 2] == scatter[:, 2]).all() and dma[:, 2].sum() <= 16
        assert (dma[:, 1] == scatter[:, 0]).all()
        for (h, sb, n), (_, g, _) in zip(dma.tolist(), scatter.tolist()):
            moved += [(h + j, g + j) for j in range(n)]
    want = [(h + j, g + j) for h, g, n in regions.tolist() for j in range(n)]
    assert moved == want


def test_greedy_accept_rejects_bad_arguments_on_the_host():
    """Argument checks run before any device work (no GPU needed)."""
    from nebulasd_b200 import _lib
    lib = _lib.lib
    assert lib.neb_greedy_accept_workspace_bytes(80) >= 256 + 80 * 8
    args = [16, 1000, 100, 4, 16, 2, 16, None, None, 0, 5, None, 16, 16, 16, 256, 4096, None]
    bad = list(args); bad[2] = 0                  # empty vocabulary
    assert lib.neb_greedy_accept(*bad) != 0
    bad = list(args); bad[1] = 10                 # row stride shorter than the vocabulary
    assert lib.neb_greedy_accept(*bad) != 0
    bad = list(args); bad[5] = 5                  # more requests than rows
    assert lib.neb_greedy_accept(*bad) != 0
    ok_empty = list(args); ok_empty[3] = 0; ok_empty[5] = 0
    assert lib.neb_greedy_accept(*ok_empty) == 0  # nothing to do
    bad = list(args); bad[16] = 8                 # workspace too small
    assert lib.neb_greedy_accept(*bad) != 0


def test_prefill_rejects_bad_arguments_on_the_host():
    """Argument checks of the prefill entry run before any device work (no GPU needed)."""
    from nebulasd_b200 import _lib
    lib = _lib.lib
    ws = lib.neb_prefill_attention_workspace_bytes(1000, 4, 32, 8)
    # units of 32 tokens x 8 kv heads: at most ceil(1000 / 32) + 4 per head, 16 bytes each
    assert ws >= 8 * (32 + 4) * 16
    assert lib.neb_prefill_attention_workspace_bytes(1000, 4, 30, 8) == 0  # heads not a multiple
    p = 1 << 20
    args = [p, 32 * 128, p, 8 * 128, p, 8 * 128, p, 4, 1000, 512, 32, 8, 128, 0.088, p, 32 * 128, p, ws, None]
    empty = list(args); empty[7] = 0
    assert lib.neb_prefill_attention(*empty) == 0               # no sequences: nothing to do
    bad = list(args); bad[10] = 24                              # q/kv head ratio 3: not this kernel's
    assert lib.neb_prefill_attention(*bad) == _lib.NEB_ERR_UNSUPPORTED
    bad = list(args); bad[12] = 64                              # head_dim 64
    assert lib.neb_prefill_attention(*bad) == _lib.NEB_ERR_UNSUPPORTED
    bad = list(args); bad[1] = 16 * 128                         # q token stride shorter than its heads
    assert lib.neb_prefill_attention(*bad) != 0
    bad = list(args); bad[2] = p + 8                            # k not 16-byte aligned
    assert lib.neb_prefill_attention(*bad) != 0
    bad = list(args); bad[17] = ws - 16                         # workspace too small
    assert lib.neb_prefill_attention(*bad) != 0
    bad = list(args); bad[9] = -1                               # negative max_seqlen
    assert lib.neb_prefill_attention(*bad) != 0


def test_accept_batch_validates_like_the_reference():
    import pytest as _pytest
    import torch
    from nebulasd_b200.accept import compute_greedy_acceptance_batch
    logits = torch.zeros((5, 10), dtype=torch.float16)
    with _pytest.raises(ValueError, match="K\\+1"):
        compute_greedy_acceptance_batch([[1, 2, 3, 4, 5]], logits)
    with _pytest.raises(ValueError, match="non-negative"):
        compute_greedy_acceptance_batch([[1, 2, 3, 4]], logits, remaining_output_len=[-1])


def test_prefill_drop_in_rejects_bad_arguments_on_the_host():
    """flash_attn_varlen_func's checks, as the reference's callers would meet them (no GPU needed)."""
    import torch
    from nebulasd_b200.kernels import flash_attn_varlen_func
    q = torch.zeros((10, 8, 128), dtype=torch.float16)
    k = torch.zeros((10, 2, 128), dtype=torch.float16)
    cu = torch.tensor([0, 4, 10], dtype=torch.int32)
    with pytest.raises(NotImplementedError):
        flash_attn_varlen_func(q, k, k, cu, cu, 6, 6, causal=False)
    with pytest.raises(NotImplementedError):
        flash_attn_varlen_func(q, k, k, cu, torch.tensor([0, 5, 10], dtype=torch.int32), 6, 6)
    with pytest.raises(TypeError):
        flash_attn_varlen_func(q.float(), k, k, cu, cu, 6, 6)
    with pytest.raises(ValueError):
        flash_attn_varlen_func(q[..., :64], k[..., :64], k[..., :64], cu, cu, 6, 6)
    with pytest.raises(ValueError):
        flash_attn_varlen_func(q, k, k, cu.long(), cu.long(), 6, 6)
