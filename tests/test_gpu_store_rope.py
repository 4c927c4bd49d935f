"""GPU: KV store, RMSNorm, RoPE and the fused QK-norm+RoPE+store against golden vectors."""
import types

import numpy as np
import pytest
import torch

from oracle import kv_store, qk_rope
from tests.golden import cases as C

pytestmark = pytest.mark.gpu
GOLDEN = C.__file__.rsplit("/", 1)[0]
ATOL, RTOL = 2e-3, 1e-2
ULP = 2 ** -10  # one fp16 ulp, relative


def _store_state(s, dev):
    npf = len(s["prefill_lens"])
    pl = torch.tensor(s["prefill_lens"], dtype=torch.int32)
    starts = torch.cumsum(pl, 0, dtype=torch.int32) - pl
    return types.SimpleNamespace(
        num_prefill_seqs=npf, num_prefill_tokens=int(pl.sum()), num_decoding_seqs=len(s["decode_lens"]),
        seq_ids=s["seq_ids"].to(dev), prefill_seq_start_locs=starts.to(dev), prefill_seq_lens=pl.to(dev),
        decoding_seq_lens=torch.tensor(s["decode_lens"], dtype=torch.int32, device=dev))


def test_store_kvcache_is_bit_exact_with_reference(cuda):
    from nebulasd_b200.kernels import store_kvcache
    s = C.store_case()
    g = np.load(f"{GOLDEN}/store_kvcache.npz")
    kc, vc = s["k_cache"].to(cuda), s["v_cache"].to(cuda)
    ec = types.SimpleNamespace(block_size=16, max_blocks_per_seq=s["block_table"].shape[1])
    store_kvcache(s["k"].to(cuda), s["v"].to(cuda), kc, vc, s["block_table"].to(cuda), None, ec,
                  _store_state(s, cuda), s["cur_layer"])
    torch.cuda.synchronize()
    assert C.digest(kc.cpu()) == str(g["k_cache_sha256"])
    assert C.digest(vc.cpu()) == str(g["v_cache_sha256"])


def _norm_rope_inputs(dev):
    n = C.norm_rope_case()
    cos_t, sin_t = qk_rope.rope_tables(128, n["theta"], int(n["positions"].max()) + 1)
    cos, sin = cos_t[n["positions"]].contiguous(), sin_t[n["positions"]].contiguous()
    return n, cos.to(dev), sin.to(dev)


def test_rmsnorm_within_one_ulp_of_reference(cuda):
    from nebulasd_b200.kernels import rmsnorm_inplace
    n, _, _ = _norm_rope_inputs(cuda)
    g = np.load(f"{GOLDEN}/qk_norm_rope.npz")
    q = n["q"].to(cuda)
    rmsnorm_inplace(q.view(-1, 128), n["q_w"].to(cuda), n["eps"])
    ref = torch.from_numpy(g["q_norm"]).float()
    torch.testing.assert_close(q.float().cpu(), ref, atol=0, rtol=ULP)
    assert (q.cpu() == torch.from_numpy(g["q_norm"])).float().mean() > 0.99


def test_rotary_is_bit_exact_with_reference(cuda):
    from nebulasd_b200.kernels import rotary_embedding_inplace
    _, cos, sin = _norm_rope_inputs(cuda)
    g = np.load(f"{GOLDEN}/qk_norm_rope.npz")
    q = torch.from_numpy(g["q_norm"]).to(cuda)
    k = torch.from_numpy(g["k_norm"]).to(cuda)
    rotary_embedding_inplace(q, k, types.SimpleNamespace(position_cos=cos, position_sin=sin))
    assert np.array_equal(q.cpu().numpy(), g["q_rope"])
    assert np.array_equal(k.cpu().numpy(), g["k_rope"])


def test_fused_norm_rope_matches_reference_and_oracle(cuda):
    from nebulasd_b200.kernels import qk_norm_rope_store
    n, cos, sin = _norm_rope_inputs(cuda)
    g = np.load(f"{GOLDEN}/qk_norm_rope.npz")
    q, k = n["q"].to(cuda), n["k"].to(cuda)
    v = torch.randn_like(k)
    st = types.SimpleNamespace(position_cos=cos, position_sin=sin, num_prefill_seqs=0, num_prefill_tokens=5,
                               num_decoding_seqs=0, seq_ids=torch.zeros(1, dtype=torch.int32, device=cuda),
                               decoding_seq_lens=None, prefill_seq_start_locs=None, prefill_seq_lens=None)
    qk_norm_rope_store(q, k, v, n["q_w"].to(cuda), n["k_w"].to(cuda), n["eps"], None, None, None, None, None, st, 0)
    torch.cuda.synchronize()
    gq, gk = torch.from_numpy(g["q_rope"]), torch.from_numpy(g["k_rope"])
    torch.testing.assert_close(q.float().cpu(), gq.float(), atol=ATOL, rtol=RTOL)
    torch.testing.assert_close(k.float().cpu(), gk.float(), atol=ATOL, rtol=RTOL)
    assert (q.cpu() == gq).float().mean() > 0.99 and (k.cpu() == gk).float().mean() > 0.99
    oq, ok = qk_rope.qk_norm_rope(n["q"], n["k"], n["q_w"], n["k_w"], n["eps"], cos.cpu(), sin.cpu())
    torch.testing.assert_close(q.float().cpu(), oq.float(), atol=ATOL, rtol=RTOL)


def test_fused_store_places_rotated_k_bit_exact(cuda):
    """Prefill + decode rows through the fused kernel: cache == oracle store of the kernel's own k/v."""
    from nebulasd_b200.kernels import qk_norm_rope_store
    s = C.store_case()
    ntok = s["k"].shape[0]
    g = torch.Generator().manual_seed(9)
    q = torch.randn((ntok, 4, 128), generator=g).half()
    w = (1 + 0.02 * torch.randn((2, 128), generator=g)).half()
    cos_t, sin_t = qk_rope.rope_tables(128, 1e6, 64)
    pos = torch.randint(0, 64, (ntok,), generator=g)
    cos, sin = cos_t[pos].contiguous(), sin_t[pos].contiguous()
    st = _store_state(s, cuda)
    st.position_cos, st.position_sin = cos.to(cuda), sin.to(cuda)
    qd, kd, vd = q.to(cuda), s["k"].to(cuda), s["v"].to(cuda)
    kc, vc = s["k_cache"].to(cuda), s["v_cache"].to(cuda)
    ec = types.SimpleNamespace(block_size=16, max_blocks_per_seq=s["block_table"].shape[1])
    qk_norm_rope_store(qd, kd, vd, w[0].to(cuda), w[1].to(cuda), 1e-6, kc, vc, s["block_table"].to(cuda), None, ec,
                       st, s["cur_layer"])
    torch.cuda.synchronize()
    # placement: replay the reference's store with the kernel's own rotated k
    ekc, evc = s["k_cache"].clone(), s["v_cache"].clone()
    npf = len(s["prefill_lens"])
    starts = np.cumsum([0] + s["prefill_lens"][:-1]).tolist()
    kk = kd.cpu()
    kv_store.store_prefill(kk, s["v"], ekc, evc, s["block_table"], s["seq_ids"][:npf], starts, s["prefill_lens"],
                           s["cur_layer"])
    ntp = sum(s["prefill_lens"])
    kv_store.store_decode(kk[ntp:], s["v"][ntp:], ekc, evc, s["block_table"], s["seq_ids"][npf:], s["decode_lens"],
                          s["cur_layer"])
    assert torch.equal(kc.cpu(), ekc) and torch.equal(vc.cpu(), evc)
    # values: the oracle's norm+rope
    oq, ok = qk_rope.qk_norm_rope(q, s["k"], w[0], w[1], 1e-6, cos, sin)
    torch.testing.assert_close(qd.float().cpu(), oq.float(), atol=ATOL, rtol=RTOL)
    torch.testing.assert_close(kk.float(), ok.float(), atol=ATOL, rtol=RTOL)


def test_store_bad_block_recorded(cuda):
    from nebulasd_b200._workspace import error_word
    from nebulasd_b200.kernels import store_kvcache
    s = C.store_case()
    bt = s["block_table"].clone()
    bt[5, 2] = -7           # decode row of seq id 5 has length 33: position 32 -> block 2
    kc, vc = s["k_cache"].to(cuda), s["v_cache"].to(cuda)
    ec = types.SimpleNamespace(block_size=16, max_blocks_per_seq=bt.shape[1])
    err = error_word(cuda)
    err.zero_()
    store_kvcache(s["k"].to(cuda), s["v"].to(cuda), kc, vc, bt.to(cuda), None, ec, _store_state(s, cuda),
                  s["cur_layer"])
    torch.cuda.synchronize()
    assert int(err.item()) & 1
    err.zero_()


def test_buffers_first_made_under_inference_mode_are_normal_tensors(cuda):
    """The reference runs its forward under ``torch.inference_mode()``; the
    per-device error word and attention workspace made on a first call there
    must still accept in-place updates outside it."""
    from nebulasd_b200 import _lib, _workspace
    _workspace.release_all()
    _workspace._error_words.clear()
    stream = torch.cuda.current_stream(cuda)
    with torch.inference_mode():
        err = _workspace.error_word(cuda)
        ws = _workspace.attention_workspace(_lib.NEB_ATTN_VERIFY, cuda, stream, 8, 32, 8)
    assert not err.is_inference() and not ws.is_inference()
    err.zero_()
    ws[:1].zero_()
    torch.cuda.synchronize()
