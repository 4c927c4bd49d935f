"""GPU: paged decode/verify attention through the C ABI against the oracle and golden vectors."""
import types

import numpy as np
import pytest
import torch

from oracle import attention as oracle
from tests.golden import cases as C

pytestmark = pytest.mark.gpu

# fp16 outputs vs the fp32 oracle: |a - b| <= 2e-3 + 1e-2 * |b|.
ATOL, RTOL = 2e-3, 1e-2
# vs the reference's own fp16-summed Triton outputs (its error vs fp32 reaches 1.95e-3 itself).
GOLD_ATOL = 4e-3

from nebulasd_b200.kernels.paged_attn import VERIFY_BUILT  # noqa: E402

KERNELS = ["decode", "verify", "verify_long"] if VERIFY_BUILT else ["decode"]


def _kernel_id(name):
    from nebulasd_b200 import _lib
    return {"decode": _lib.NEB_ATTN_DECODE, "verify": _lib.NEB_ATTN_VERIFY,
            "verify_long": _lib.NEB_ATTN_VERIFY_LONG}[name]


def run_attention(c, kernel, dev, workspace=None):
    from nebulasd_b200.kernels import paged_attention_raw
    q = c["q"].to(dev)
    o = torch.full_like(q, float("nan"))
    paged_attention_raw(q, c["k_cache"].to(dev), c["v_cache"].to(dev), c["block_table"].to(dev),
                        c["seq_lens"].to(dev), c["seq_ids"].to(dev), c["cur_layer"], c["softmax_scale"], o,
                        kernel=_kernel_id(kernel), workspace=workspace)
    torch.cuda.synchronize(dev)
    return o.float().cpu()


def oracle_of(c):
    return oracle.paged_attention(c["q"], c["k_cache"], c["v_cache"], c["block_table"], c["seq_lens"],
                                  c["seq_ids"], c["cur_layer"], c["softmax_scale"])


def batch_case(seed, **kw):
    from nebulasd_b200.workloads import make_paged_batch
    b = make_paged_batch(seed, **kw)
    return dict(q=b.q, k_cache=b.k_cache, v_cache=b.v_cache, block_table=b.block_table, seq_ids=b.seq_ids,
                seq_lens=b.seq_lens, cur_layer=b.cur_layer, softmax_scale=b.q.shape[-1] ** -0.5)


@pytest.mark.parametrize("kernel", KERNELS)
@pytest.mark.parametrize("name", sorted(C.attention_cases()))
def test_golden_cases(kernel, name, cuda):
    c = C.attention_cases()[name]
    g = np.load(f"{C.__file__.rsplit('/', 1)[0]}/{name}.npz")
    out = run_attention(c, kernel, cuda)
    torch.testing.assert_close(out, oracle_of(c), atol=ATOL, rtol=RTOL)
    torch.testing.assert_close(out, torch.from_numpy(g["o"]).float(), atol=GOLD_ATOL, rtol=RTOL)


SHAPES = {
    # Draft decode (Qwen3-0.6B heads), ragged lengths incl. block edges
    "decode_gqa2": dict(num_requests=24, depth=0, ctx_lo=0, ctx_hi=700, num_q_heads=16, num_kv_heads=8,
                        pool_blocks=1400, num_layers=3, cur_layer=1),
    # Target verify (Qwen3-8B heads), k=4
    "verify_gqa4_k4": dict(num_requests=6, depth=4, ctx_lo=200, ctx_hi=1500, num_q_heads=32, num_kv_heads=8,
                           pool_blocks=800, num_layers=2, cur_layer=1),
    # k=8 and ragged depths, shuffled table rows
    "verify_gqa4_ragged": dict(num_requests=7, depth=[8, 0, 3, 8, 1, 5, 2], ctx_lo=1, ctx_hi=900,
                               num_q_heads=32, num_kv_heads=8, pool_blocks=600, shuffle_seq_ids=True),
    # group longer than one MMA tile can hold (depth 40 -> 41 rows x GQA 4 > 128)
    "verify_deep": dict(num_requests=2, depth=40, ctx_lo=50, ctx_hi=300, num_q_heads=32, num_kv_heads=8,
                        pool_blocks=64),
    # one unit cut into a piece per CTA: every piece claims at its end and one
    # merger waits for all the others' partials
    "one_unit_all_ctas": dict(num_requests=1, depth=4, ctx_lo=3000, ctx_hi=3000, num_q_heads=4, num_kv_heads=1,
                              pool_blocks=200),
    # GQA 1 and GQA 8
    "mha": dict(num_requests=5, depth=2, ctx_lo=10, ctx_hi=400, num_q_heads=4, num_kv_heads=4, pool_blocks=200),
    "gqa8": dict(num_requests=5, depth=3, ctx_lo=10, ctx_hi=400, num_q_heads=16, num_kv_heads=2,
                 pool_blocks=200),
}


@pytest.mark.parametrize("kernel", KERNELS)
@pytest.mark.parametrize("shape", sorted(SHAPES))
@pytest.mark.parametrize("seed", [1, 2])
def test_random_batches_match_oracle(kernel, shape, seed, cuda):
    c = batch_case(seed * 1000 + sorted(SHAPES).index(shape), **SHAPES[shape])
    torch.testing.assert_close(run_attention(c, kernel, cuda), oracle_of(c), atol=ATOL, rtol=RTOL)


# Every q/kv head ratio the verify kernel accepts that the decode kernel is not
# built for, or whose unit rows do not fill whole 16-lane chunks, at depths 4
# and 8: a unit's rows are cut into four chunks of gqa * ceil(rows / 4) query
# rows, which must each fit one TMEM lane quadrant.  Depth 20 at gqa 3 gives a
# request of 21 rows, one more than a unit holds.
GQA_SHAPES = {
    f"gqa{g}_k{k}": dict(num_requests=5, depth=k, ctx_lo=10, ctx_hi=700, num_q_heads=2 * g, num_kv_heads=2,
                         pool_blocks=300)
    for g in (3, 5, 6, 7, 9, 12, 16) for k in (4, 8)
}
GQA_SHAPES["gqa3_k20"] = dict(num_requests=3, depth=20, ctx_lo=30, ctx_hi=500, num_q_heads=6, num_kv_heads=2,
                              pool_blocks=120)
GQA_SHAPES["gqa5_ragged"] = dict(num_requests=6, depth=[8, 0, 3, 11, 1, 5], ctx_lo=1, ctx_hi=600,
                                 num_q_heads=10, num_kv_heads=2, pool_blocks=300, shuffle_seq_ids=True)


@pytest.mark.skipif(not VERIFY_BUILT, reason="verify kernel not built")
@pytest.mark.parametrize("kernel", ["verify", "verify_long"])
@pytest.mark.parametrize("shape", sorted(GQA_SHAPES))
def test_verify_every_gqa_ratio_matches_oracle(kernel, shape, cuda):
    c = batch_case(3000 + sorted(GQA_SHAPES).index(shape), **GQA_SHAPES[shape])
    torch.testing.assert_close(run_attention(c, kernel, cuda), oracle_of(c), atol=ATOL, rtol=RTOL)


@pytest.mark.skipif(not VERIFY_BUILT, reason="verify kernel not built")
@pytest.mark.parametrize("kernel", ["verify", "verify_long"])
def test_long_prefix_batch_matches_oracle(kernel, cuda):
    """Prefixes of 8 K - 20 K tokens (many 128-token stages per unit, units split across CTAs)."""
    c = batch_case(5150, num_requests=3, depth=[4, 8, 0], ctx_lo=8192, ctx_hi=20000, num_q_heads=32,
                   num_kv_heads=8, pool_blocks=4000)
    torch.testing.assert_close(run_attention(c, kernel, cuda), oracle_of(c), atol=ATOL, rtol=RTOL)


def test_auto_picks_long_kernel_from_max_len():
    from nebulasd_b200 import _lib
    from nebulasd_b200.kernels.paged_attn import LONG_CONTEXT_TOKENS, choose_kernel
    assert choose_kernel(32, 8, 80, 4100) == _lib.NEB_ATTN_VERIFY
    assert choose_kernel(32, 8, 80, LONG_CONTEXT_TOKENS) == _lib.NEB_ATTN_VERIFY_LONG
    assert choose_kernel(16, 8, 64, 40000) == _lib.NEB_ATTN_DECODE


def test_auto_dispatch_serves_every_ratio_up_to_16(cuda):
    """The drop-in entry picks a kernel for every integer q/kv head ratio 1..16, as the reference accepts."""
    from nebulasd_b200.kernels import paged_attention_raw
    for g in range(1, 17):
        c = batch_case(4000 + g, num_requests=3, depth=4, ctx_lo=20, ctx_hi=300, num_q_heads=g, num_kv_heads=1,
                       pool_blocks=80)
        q = c["q"].to(cuda)
        o = torch.empty_like(q)
        paged_attention_raw(q, c["k_cache"].to(cuda), c["v_cache"].to(cuda), c["block_table"].to(cuda),
                            c["seq_lens"].to(cuda), c["seq_ids"].to(cuda), c["cur_layer"], c["softmax_scale"], o)
        torch.cuda.synchronize(cuda)
        torch.testing.assert_close(o.float().cpu(), oracle_of(c), atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("kernel", KERNELS)
def test_status_after_timeout_clears_stale_counters(kernel, cuda):
    """A call that gave up on a bounded wait leaves split counters counted; the status call clears them.

    The failed call is stood in for on the host: the timeout bit and non-zero
    counters are written into the workspace, as such a call leaves them.
    """
    from nebulasd_b200._workspace import attention_workspace, workspace_errors
    stream = torch.cuda.current_stream(cuda)
    ws = attention_workspace(_kernel_id(kernel), cuda, stream, 4096, 32, 8)
    counters = ws[256:256 + 4096 * 64 * 4].view(torch.int32)
    header = ws[:4].view(torch.int32)
    header.fill_(8)                 # kErrTimeout
    counters[:4096].fill_(1)        # pieces counted in by the CTAs that did not give up
    assert workspace_errors(ws, stream) == 8
    assert int(torch.count_nonzero(counters).item()) == 0
    assert workspace_errors(ws, stream) == 0
    c = batch_case(61, **SHAPES["one_unit_all_ctas"])
    torch.testing.assert_close(run_attention(c, kernel, cuda, workspace=ws), oracle_of(c), atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("kernel", KERNELS)
def test_zero_length_rows_give_nan_and_others_unaffected(kernel, cuda):
    c = dict(C.attention_cases()["decode_edges"])
    lens = c["seq_lens"].clone()
    lens[2] = 0
    c["seq_lens"] = lens
    out = run_attention(c, kernel, cuda)
    assert torch.isnan(out[2]).all()
    ref = oracle_of(c)
    keep = [0, 1, 3, 4, 5]
    torch.testing.assert_close(out[keep], ref[keep], atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("kernel", KERNELS)
def test_bad_block_index_is_recorded_not_faulted(kernel, cuda):
    from nebulasd_b200._workspace import attention_workspace, workspace_errors
    c = dict(C.attention_cases()["verify_cfg1"])
    ref = oracle_of(c)
    bt = c["block_table"].clone()
    bt[1, 2] = 10 ** 6            # out of the 256-block pool
    c["block_table"] = bt
    stream = torch.cuda.current_stream(cuda)
    ws = attention_workspace(_kernel_id(kernel), cuda, stream, 20, 16, 8)
    workspace_errors(ws, stream)  # clear
    out = run_attention(c, kernel, cuda, workspace=ws)
    assert workspace_errors(ws, stream) & 1
    good = c["seq_ids"] != 1
    torch.testing.assert_close(out[good], ref[good], atol=ATOL, rtol=RTOL)
    assert workspace_errors(ws, stream) == 0


@pytest.mark.parametrize("kernel", KERNELS)
def test_deterministic_and_workspace_reusable(kernel, cuda):
    a = batch_case(7, **SHAPES["verify_gqa4_k4"])
    b = batch_case(8, **SHAPES["decode_gqa2"])
    o1 = run_attention(a, kernel, cuda)
    o2 = run_attention(b, kernel, cuda)
    o3 = run_attention(a, kernel, cuda)
    assert torch.equal(o1, o3)
    torch.testing.assert_close(o2, oracle_of(b), atol=ATOL, rtol=RTOL)


def test_drop_in_signature_with_infer_state(cuda):
    from nebulasd_b200.kernels import paged_attention
    c = C.attention_cases()["verify_cfg1"]
    sbs, nsb = oracle.split_heuristic(c["seq_lens"].tolist(), 8)
    r = c["q"].shape[0]
    st = types.SimpleNamespace(num_decoding_seqs=r, num_prefill_seqs=0, seq_block_size=sbs, num_seq_blocks=nsb,
                               decoding_seq_lens=c["seq_lens"].to(cuda), seq_ids=c["seq_ids"].to(cuda),
                               softmax_scale=c["softmax_scale"])
    mc = types.SimpleNamespace(num_q_heads=16, num_kv_heads=8, head_dim=128, num_layers=2)
    ec = types.SimpleNamespace(block_size=16, max_blocks_per_seq=c["block_table"].shape[1])
    o = torch.empty((r, 16 * 128), dtype=torch.float16, device=cuda)   # the layer's [tokens, width] view
    paged_attention(c["q"].to(cuda), c["k_cache"].to(cuda), c["v_cache"].to(cuda), c["block_table"].to(cuda),
                    mc, ec, st, c["cur_layer"], o)
    torch.testing.assert_close(o.view(r, 16, 128).float().cpu(), oracle_of(c), atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("kernel", KERNELS)
def test_target_verify_full_size_property(kernel, cuda):
    """Config-3 lengths and pool size (one layer): oracle on a sample of requests."""
    from nebulasd_b200.workloads import make_paged_batch
    b = make_paged_batch(2024, num_requests=16, depth=4, ctx_lo=256, ctx_hi=4096, num_q_heads=32, num_kv_heads=8,
                         pool_blocks=24576, num_layers=1, device=cuda)
    o = torch.empty_like(b.q)
    from nebulasd_b200.kernels import paged_attention_raw
    paged_attention_raw(b.q, b.k_cache, b.v_cache, b.block_table, b.seq_lens, b.seq_ids, 0, 128 ** -0.5, o,
                        kernel=_kernel_id(kernel))
    torch.cuda.synchronize()
    assert torch.isfinite(o).all()
    # Units cut across CTAs are merged by whichever piece ends last, by one of
    # two paths; both give the same bits, so a second call reproduces the first.
    o2 = torch.empty_like(o)
    paged_attention_raw(b.q, b.k_cache, b.v_cache, b.block_table, b.seq_lens, b.seq_ids, 0, 128 ** -0.5, o2,
                        kernel=_kernel_id(kernel))
    torch.cuda.synchronize()
    assert torch.equal(o, o2)
    for req in (0, 7, 15):
        rows = [i for i, s in enumerate(b.seq_ids_list) if s == req]
        nb = (max(b.seq_lens_list[i] for i in rows) + 15) // 16
        blocks = b.block_table[req, :nb].long()
        kc = b.k_cache[blocks].cpu()
        vc = b.v_cache[blocks].cpu()
        bt = torch.arange(nb, dtype=torch.int32)[None, :]
        ref = oracle.paged_attention(b.q[rows].cpu(), kc, vc, bt, [b.seq_lens_list[i] for i in rows],
                                     [0] * len(rows), 0, 128 ** -0.5)
        torch.testing.assert_close(o[rows].float().cpu(), ref, atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("kernel", KERNELS)
def test_counters_return_to_zero_across_shapes(kernel, cuda):
    """Every call leaves the workspace's arrival counters at zero, whatever the next call's shape."""
    from nebulasd_b200._workspace import attention_workspace
    stream = torch.cuda.current_stream(cuda)
    ws = attention_workspace(_kernel_id(kernel), cuda, stream, 4096, 32, 8)
    counters = ws[256:256 + 4096 * 64 * 4]
    for i, shape in enumerate(["verify_deep", "decode_gqa2", "verify_gqa4_k4", "verify_gqa4_ragged", "gqa8"]):
        c = batch_case(50 + i, **SHAPES[shape])
        out = run_attention(c, kernel, cuda, workspace=ws)
        assert int(torch.count_nonzero(counters).item()) == 0, f"stale counters after {shape}"
        torch.testing.assert_close(out, oracle_of(c), atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("kernel", ["verify"] if VERIFY_BUILT else [])
def test_plan_cache_follows_inputs(kernel, cuda):
    """The verify kernel reuses the previous call's work plan on the same
    workspace only when the rows' seq ids, lengths and the call's shape are the
    same: repeated, changed and restored batches on one workspace all match the
    oracle, as do calls after the block table's contents or width change."""
    from nebulasd_b200._workspace import attention_workspace
    stream = torch.cuda.current_stream(cuda)
    ws = attention_workspace(_kernel_id(kernel), cuda, stream, 512, 32, 8)
    a = batch_case(71, **SHAPES["verify_gqa4_k4"])
    b = batch_case(72, **SHAPES["verify_gqa4_k4"])          # same shapes, other lengths
    c = dict(a, seq_ids=a["seq_ids"].flip(0).contiguous(), seq_lens=a["seq_lens"].flip(0).contiguous(),
             q=a["q"].flip(0).contiguous())  # rows reordered
    moved = dict(a, block_table=a["block_table"].roll(1, dims=0).contiguous(),
                 seq_ids=((a["seq_ids"] + 1) % a["block_table"].shape[0]).to(torch.int32))  # same blocks, other rows
    wide = dict(a, block_table=torch.cat([a["block_table"], torch.full_like(a["block_table"], -1)], 1))
    for case in (a, a, b, a, a, c, a, moved, moved, wide, wide, a):
        torch.testing.assert_close(run_attention(case, kernel, cuda, workspace=ws), oracle_of(case),
                                   atol=ATOL, rtol=RTOL)
