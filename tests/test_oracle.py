"""CPU: the oracle against the reference's golden vectors and known answers."""
import math

import numpy as np
import pytest
import torch

from oracle import accept, attention, hostkv, kv_store, prefill, qk_rope
from tests.golden import cases as C

GOLDEN = C.__file__.rsplit("/", 1)[0]
# fp16 outputs: |a - b| <= 2e-3 + 1e-2 * |b|  (allclose form)
ATOL, RTOL = 2e-3, 1e-2


def _load(name):
    return np.load(f"{GOLDEN}/{name}.npz")


@pytest.mark.parametrize("name", sorted(C.attention_cases()))
def test_attention_oracle_matches_reference_golden(name):
    c = C.attention_cases()[name]
    g = _load(name)
    assert str(g["input_sha256"]) == C.digest(c["q"], c["k_cache"], c["v_cache"], c["block_table"],
                                              c["seq_ids"], c["seq_lens"])
    o = attention.paged_attention(c["q"], c["k_cache"], c["v_cache"], c["block_table"], c["seq_lens"],
                                  c["seq_ids"], c["cur_layer"], c["softmax_scale"])
    ref = torch.from_numpy(g["o"]).float()
    torch.testing.assert_close(o, ref, atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("name", sorted(C.attention_cases()))
def test_grouped_oracle_equals_row_by_row_spec(name):
    c = C.attention_cases()[name]
    a = attention.paged_attention(c["q"], c["k_cache"], c["v_cache"], c["block_table"], c["seq_lens"],
                                  c["seq_ids"], c["cur_layer"], c["softmax_scale"])
    b = attention.paged_attention_rows(c["q"], c["k_cache"], c["v_cache"], c["block_table"], c["seq_lens"],
                                       c["seq_ids"], c["cur_layer"], c["softmax_scale"])
    torch.testing.assert_close(a, b, atol=1e-5, rtol=1e-5)


def test_zero_length_row_is_nan_like_reference():
    c = C.attention_cases()["decode_edges"]
    lens = c["seq_lens"].clone()
    lens[0] = 0
    o = attention.paged_attention(c["q"], c["k_cache"], c["v_cache"], c["block_table"], lens, c["seq_ids"],
                                  0, c["softmax_scale"])
    assert torch.isnan(o[0]).all() and not torch.isnan(o[1:]).any()


def test_store_oracle_matches_reference_golden_bit_exact():
    s = C.store_case()
    g = _load("store_kvcache")
    assert str(g["input_sha256"]) == C.digest(s["k"], s["v"], s["k_cache"], s["v_cache"], s["block_table"],
                                              s["seq_ids"])
    kc, vc = s["k_cache"].clone(), s["v_cache"].clone()
    npf = len(s["prefill_lens"])
    starts = np.cumsum([0] + s["prefill_lens"][:-1]).tolist()
    kv_store.store_prefill(s["k"], s["v"], kc, vc, s["block_table"], s["seq_ids"][:npf], starts,
                           s["prefill_lens"], s["cur_layer"])
    ntp = sum(s["prefill_lens"])
    kv_store.store_decode(s["k"][ntp:], s["v"][ntp:], kc, vc, s["block_table"], s["seq_ids"][npf:],
                          s["decode_lens"], s["cur_layer"])
    assert C.digest(kc) == str(g["k_cache_sha256"])
    assert C.digest(vc) == str(g["v_cache_sha256"])


def test_qk_norm_rope_oracle_matches_reference_golden():
    n = C.norm_rope_case()
    g = _load("qk_norm_rope")
    cos_t, sin_t = qk_rope.rope_tables(128, n["theta"], int(n["positions"].max()) + 1)
    cos, sin = cos_t[n["positions"]].contiguous(), sin_t[n["positions"]].contiguous()
    assert str(g["input_sha256"]) == C.digest(n["q"], n["k"], n["q_w"], n["k_w"], cos, sin)
    assert np.array_equal(cos.numpy(), g["cos"]) and np.array_equal(sin.numpy(), g["sin"])
    qn = qk_rope.rmsnorm(n["q"], n["q_w"], n["eps"])
    kn = qk_rope.rmsnorm(n["k"], n["k_w"], n["eps"])
    # fp32 RMSNorm rounded once to fp16: within one fp16 ulp of the reference.
    torch.testing.assert_close(qn.float(), torch.from_numpy(g["q_norm"]).float(), atol=0, rtol=2 ** -10)
    torch.testing.assert_close(kn.float(), torch.from_numpy(g["k_norm"]).float(), atol=0, rtol=2 ** -10)
    # The reference's fp16-rounded RoPE applied to the reference's normalised values is bit-exact.
    q16 = qk_rope.rope_fp16(torch.from_numpy(g["q_norm"]), cos, sin)
    k16 = qk_rope.rope_fp16(torch.from_numpy(g["k_norm"]), cos, sin)
    assert np.array_equal(q16.numpy(), g["q_rope"]) and np.array_equal(k16.numpy(), g["k_rope"])
    # The fp32 restatement is within the fp16 tolerance.
    q32 = qk_rope.rope(torch.from_numpy(g["q_norm"]), cos, sin)
    torch.testing.assert_close(q32.float(), torch.from_numpy(g["q_rope"]).float(), atol=ATOL, rtol=RTOL)


def test_prefill_oracle_matches_reference_golden():
    """Against the layer module's own flash_attn_varlen_func (transformer_layer.py:7-32),
    run in fp32 on the same inputs; the fixture stores it rounded to fp16."""
    p = C.prefill_case()
    g = _load("prefill")
    assert str(g["input_sha256"]) == C.digest(p["q"], p["k"], p["v"], p["cu_seqlens"])
    o = prefill.prefill_attention(p["q"], p["k"], p["v"], p["cu_seqlens"], p["softmax_scale"])
    torch.testing.assert_close(o, torch.from_numpy(g["o"]).float(), atol=1e-3, rtol=2 ** -10)


# Known answers of swiftLLM/tests/test_speculative_planning.py:25-178.
def test_linear_rows_known_answer():
    tokens, lens = accept.linear_rows(100, [10, 11, 12], [21, 22, 23])
    assert tokens == [12, 21, 22, 23] and lens == [103, 104, 105, 106]


@pytest.mark.parametrize("draft,post,remaining,stops,expected,count", [
    ([21, 22, 23], [21, 99, 0, 0], None, (), [21, 99], 1),
    ([21, 22, 23], [21, 22, 23, 99], 1, (), [21], 1),
    ([21, 22, 23], [21, 99, 0, 0], 1, (), [21], 1),
    ([21, 22, 23], [99, 0, 0, 0], 1, (), [99], 0),
    ([21, 22, 23], [21, 22, 23, 99], 0, (), [], 0),
    ([21, 22, 23], [21, 22, 23, 99], None, (22,), [21, 22], 2),
    ([21, 22], [21, 22, 99], 1, (), [21], 1),
    ([21, 22, 23], [99, 0, 0, 0], None, (), [99], 0),
    ([21, 22, 23], [21, 22, 23, 99], None, (), [21, 22, 23, 99], 3),
])
def test_greedy_acceptance_known_answers(draft, post, remaining, stops, expected, count):
    assert accept.greedy_accept(draft, post, remaining, stops) == (expected, count)


def test_greedy_acceptance_rejects_negative_budget():
    with pytest.raises(ValueError, match="remaining_output_len must be non-negative"):
        accept.greedy_accept([21, 22, 23], [21, 22, 23, 99], -1)


def test_split_heuristic_matches_reference_rule():
    # model.py:380-384 halves from 2048 while Hk*sum/sbs < 1024, sbs/2 >= 64, max/(sbs/2) <= 128
    assert attention.split_heuristic([100] * 4, 8) == (64, 2)
    assert attention.split_heuristic([32768] * 64, 8) == (2048, 16)


def test_hostkv_region_semantics_and_guards():
    bb = 64
    host = (np.zeros(20 * bb, np.uint8), np.zeros(20 * bb, np.uint8))
    gpu = (np.arange(12 * bb, dtype=np.uint8), (np.arange(12 * bb) * 3).astype(np.uint8))
    hostkv.apply_regions("D2H", [(2, 5, 3), (10, 0, 1)], host, gpu, bb)
    assert np.array_equal(host[0][2 * bb:5 * bb], gpu[0][5 * bb:8 * bb])
    assert np.array_equal(host[1][10 * bb:11 * bb], gpu[1][0:bb])
    assert not host[0][:2 * bb].any() and not host[0][5 * bb:10 * bb].any()
    gpu2 = (np.zeros_like(gpu[0]), np.zeros_like(gpu[1]))
    hostkv.apply_regions("H2D", [(2, 5, 3), (10, 0, 1)], host, gpu2, bb)
    assert np.array_equal(gpu2[0][5 * bb:8 * bb], gpu[0][5 * bb:8 * bb])
    assert hostkv.guard_pattern(1, 2, 3) == 1 + (79 + 14 + 3) % 180


def test_block_table_fill_matches_bank_layout():
    bt = np.full((4, 6), -1, np.int32)
    hostkv.fill_table(bt, rows=[0, 2], begins=[100, 7], counts=[3, 6])
    assert bt[0, :3].tolist() == [100, 101, 102] and bt[0, 3] == -1
    assert bt[2].tolist() == list(range(7, 13))


def test_kv_bytes_counts_each_group_once():
    # two requests verified at depth 4 (lens L+1..L+5) and one decode row
    ids = [0] * 5 + [1] * 5 + [2]
    lens = [11, 12, 13, 14, 15] + [101, 102, 103, 104, 105] + [7]
    assert attention.kv_bytes(lens, ids, 8, 128) == (15 + 105 + 7) * 8 * 128 * 2 * 2
    assert math.isclose(attention.DEFAULT_SCALE_128, 128 ** -0.5)
