"""GPU: the allocation-free decode attention entry point.

``neb_paged_attention_decode_noalloc`` serves callers that cannot call
cudaMalloc -- for instance a worker whose device memory was all claimed by its
KV-cache pool at start-up, or a host that must not let a call synchronise the
device while other streams are busy.  It keeps its split-K scratch in a static
array inside the library instead of a caller-provided workspace.  This test
calls it through the C ABI twice in a row, on two different batches, and checks
each output against the workspace entry point (``neb_paged_attention_decode``)
within the attention tests' tolerance, and against the fp32 oracle.

The file name sorts last so that a run stopping at the first failure has
already run every other test; it also passes on its own in a fresh process.
"""
import pytest
import torch

from oracle import attention as oracle

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-2


def _batches():
    from nebulasd_b200.workloads import make_paged_batch
    yield make_paged_batch(71, num_requests=24, depth=0, ctx_lo=1, ctx_hi=1500, num_q_heads=16, num_kv_heads=8,
                           pool_blocks=3000, num_layers=2, cur_layer=1)
    yield make_paged_batch(72, num_requests=6, depth=4, ctx_lo=100, ctx_hi=2500, num_q_heads=32, num_kv_heads=8,
                           pool_blocks=1200)
    # q/kv head ratio 8 needs the most partials per worker: the call uses as many
    # workers as the static array holds partials for.
    yield make_paged_batch(73, num_requests=40, depth=0, ctx_lo=1, ctx_hi=3000, num_q_heads=32, num_kv_heads=4,
                           pool_blocks=8000)


def _noalloc_call(b, q, kc, vc, bt, lens, ids, out, stream):
    from nebulasd_b200 import _lib
    return _lib.lib.neb_paged_attention_decode_noalloc(
        q.data_ptr(), kc.data_ptr(), vc.data_ptr(), bt.data_ptr(), bt.shape[0], bt.shape[1], lens.data_ptr(),
        ids.data_ptr(), q.shape[0], q.shape[1], kc.shape[2], 128, 16, kc.shape[0], kc.shape[1], b.cur_layer,
        128 ** -0.5, out.data_ptr(), stream.cuda_stream)


def _noalloc_status(stream):
    import ctypes
    from nebulasd_b200 import _lib
    bits = ctypes.c_uint32(0xFFFF)
    _lib.check(_lib.lib.neb_paged_attention_noalloc_status(ctypes.byref(bits), stream.cuda_stream),
               "neb_paged_attention_noalloc_status")
    return bits.value


def test_noalloc_decode_matches_workspace_entry_two_calls_in_a_row(cuda):
    from nebulasd_b200 import _lib
    from nebulasd_b200.kernels import paged_attention_raw
    stream = torch.cuda.current_stream(cuda)
    for b in _batches():
        args = [t.to(cuda) for t in (b.q, b.k_cache, b.v_cache, b.block_table, b.seq_lens, b.seq_ids)]
        q, kc, vc, bt, lens, ids = args
        scale = 128 ** -0.5
        expect = torch.empty_like(q)
        paged_attention_raw(q, kc, vc, bt, lens, ids, b.cur_layer, scale, expect, kernel=_lib.NEB_ATTN_DECODE)
        got = torch.full_like(q, float("nan"))
        rc = _lib.lib.neb_paged_attention_decode_noalloc(
            q.data_ptr(), kc.data_ptr(), vc.data_ptr(), bt.data_ptr(), bt.shape[0], bt.shape[1], lens.data_ptr(),
            ids.data_ptr(), q.shape[0], q.shape[1], kc.shape[2], 128, 16, kc.shape[0], kc.shape[1], b.cur_layer,
            scale, got.data_ptr(), stream.cuda_stream)
        _lib.check(rc, "neb_paged_attention_decode_noalloc")
        torch.cuda.synchronize(cuda)
        torch.testing.assert_close(got.float(), expect.float(), atol=ATOL, rtol=RTOL)
        ref = oracle.paged_attention(b.q, b.k_cache, b.v_cache, b.block_table, b.seq_lens_list, b.seq_ids_list,
                                     b.cur_layer, scale)
        torch.testing.assert_close(got.float().cpu(), ref, atol=ATOL, rtol=RTOL)


def test_noalloc_status_reports_bad_block_index(cuda):
    """A block-table entry outside the pool is skipped by the kernel and reported by the status call."""
    from nebulasd_b200 import _lib
    from nebulasd_b200.workloads import make_paged_batch
    stream = torch.cuda.current_stream(cuda)
    b = make_paged_batch(74, num_requests=5, depth=0, ctx_lo=40, ctx_hi=400, num_q_heads=16, num_kv_heads=8,
                         pool_blocks=200)
    q, kc, vc, bt, lens, ids = [t.to(cuda) for t in (b.q, b.k_cache, b.v_cache, b.block_table, b.seq_lens,
                                                      b.seq_ids)]
    _noalloc_status(stream)  # start from a clean header
    bad = bt.clone()
    bad[2, 1] = 10 ** 6
    out = torch.empty_like(q)
    _lib.check(_noalloc_call(b, q, kc, vc, bad, lens, ids, out, stream), "neb_paged_attention_decode_noalloc")
    assert _noalloc_status(stream) & 1
    assert _noalloc_status(stream) == 0
    _lib.check(_noalloc_call(b, q, kc, vc, bt, lens, ids, out, stream), "neb_paged_attention_decode_noalloc")
    assert _noalloc_status(stream) == 0
    ref = oracle.paged_attention(b.q, b.k_cache, b.v_cache, b.block_table, b.seq_lens_list, b.seq_ids_list,
                                 b.cur_layer, 128 ** -0.5)
    torch.testing.assert_close(out.float().cpu(), ref, atol=ATOL, rtol=RTOL)
