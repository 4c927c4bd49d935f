"""GPU: device-side greedy acceptance against torch.argmax and the oracle's
restatement of compute_greedy_acceptance (swiftLLM/swiftllm/speculative.py:122-156)."""
import pytest
import torch

from oracle import accept as oracle

pytestmark = pytest.mark.gpu

VOCAB = 151936  # Qwen3


def _batch(seed, depths, dev, vocab=VOCAB, accept_upto=None):
    """Logits of sum(k+1) rows and drafts whose first accept_upto[r] tokens
    equal the rows' arg-maxes (so every acceptance length occurs)."""
    g = torch.Generator().manual_seed(seed)
    rows = sum(k + 1 for k in depths)
    logits = (torch.randn((rows, vocab), generator=g) * 4).half()
    am = logits.float().argmax(1).tolist()
    drafts, r0 = [], 0
    for i, k in enumerate(depths):
        n = accept_upto[i] if accept_upto else int(torch.randint(0, k + 1, (1,), generator=g))
        d = []
        for j in range(k):
            d.append(am[r0 + j] if j < n else (am[r0 + j] + 1 + j) % vocab)
        drafts.append(d)
        r0 += k + 1
    return logits.to(dev), drafts


def _oracle(logits, drafts, remaining=None, stops=()):
    post = logits.float().argmax(1).tolist()
    out, r0 = [], 0
    for i, d in enumerate(drafts):
        out.append(oracle.greedy_accept(d, post[r0:r0 + len(d) + 1], None if remaining is None else remaining[i],
                                        stops))
        r0 += len(d) + 1
    return out


@pytest.mark.parametrize("depths", [[4] * 16, [8, 0, 3, 8, 1, 5, 2], [0] * 64])
def test_matches_oracle_and_torch_argmax(depths, cuda):
    from nebulasd_b200.accept import compute_greedy_acceptance_batch, greedy_accept
    logits, drafts = _batch(len(depths), depths, cuda)
    assert compute_greedy_acceptance_batch(drafts, logits) == _oracle(logits, drafts)
    starts = torch.tensor([0] + list(torch.cumsum(torch.tensor([k + 1 for k in depths]), 0)), dtype=torch.int32)
    flat = torch.tensor([t for d in drafts for t in d] or [0], dtype=torch.int32)[:sum(depths)]
    _, _, _, am = greedy_accept(logits, starts.to(cuda), flat.contiguous().to(cuda))
    assert torch.equal(am.long().cpu(), logits.argmax(1).cpu())


def test_ties_nan_and_signed_zero_follow_torch(cuda):
    from nebulasd_b200.accept import greedy_accept
    logits = torch.full((6, VOCAB), -1.0, dtype=torch.float16)
    logits[0, [7, 70000, 150000]] = 3.0                    # tie: lowest index
    logits[1, 123] = float("nan"); logits[1, 5] = 60000.0   # NaN counts as the largest
    logits[2] = -0.0; logits[2, 9] = 0.0                    # all zeros of either sign: index 0
    logits[3] = float("-inf"); logits[3, VOCAB - 1] = -65504.0
    logits[4, VOCAB - 1] = 1.0; logits[4, VOCAB - 2] = 1.0
    logits[5] = -2.0
    logits = logits.to(cuda)
    starts = torch.arange(7, dtype=torch.int32, device=cuda)
    _, _, _, am = greedy_accept(logits, starts, torch.zeros(0, dtype=torch.int32, device=cuda))
    assert am.long().cpu().tolist() == logits.argmax(1).cpu().tolist()


def test_budget_and_stop_tokens(cuda):
    from nebulasd_b200.accept import compute_greedy_acceptance_batch
    logits, drafts = _batch(11, [4] * 8, cuda, accept_upto=[4, 3, 2, 1, 0, 4, 4, 2])
    post = logits.float().argmax(1).tolist()
    remaining = [None, 0, 1, 2, 5, 3, None, 4]
    stops = [drafts[0][1], post[5 * 5 + 4]]
    assert compute_greedy_acceptance_batch(drafts, logits, remaining, stops) == \
        _oracle(logits, drafts, remaining, stops)


def test_workspace_reused_across_sizes(cuda):
    from nebulasd_b200.accept import compute_greedy_acceptance_batch
    for seed, depths, vocab in ((1, [4] * 16, VOCAB), (2, [2] * 3, 1000), (3, [8] * 40, 32000), (4, [4] * 16, VOCAB)):
        logits, drafts = _batch(seed, depths, cuda, vocab=vocab)
        assert compute_greedy_acceptance_batch(drafts, logits) == _oracle(logits, drafts)


def test_odd_vocab_and_strided_rows(cuda):
    from nebulasd_b200.accept import greedy_accept
    g = torch.Generator().manual_seed(5)
    wide = (torch.randn((10, 50021), generator=g)).half().to(cuda)
    logits = wide[:, 3:50000]  # rows start off 16-byte alignment
    starts = torch.arange(11, dtype=torch.int32, device=cuda)
    _, _, _, am = greedy_accept(logits, starts, torch.zeros(0, dtype=torch.int32, device=cuda))
    assert torch.equal(am.long().cpu(), logits.argmax(1).cpu())


def test_invalid_rows_are_reported(cuda):
    from nebulasd_b200.accept import greedy_accept, workspace_errors
    logits = torch.randn((4, 100), device=cuda).half()
    assert workspace_errors() == 0
    bad_starts = torch.tensor([0, 3, 2], dtype=torch.int32, device=cuda)  # a request with -1 rows
    tokens, count, _, _ = greedy_accept(logits, bad_starts, torch.zeros(2, dtype=torch.int32, device=cuda))
    assert workspace_errors() & 16
    assert int(count[1]) == 0 and workspace_errors() == 0


def test_batches_beyond_the_staged_rows(cuda):
    """More rows than phase 2 stages in shared memory (2048): the global path."""
    from nebulasd_b200.accept import compute_greedy_acceptance_batch
    logits, drafts = _batch(21, [4] * 450, cuda, vocab=2048)
    assert compute_greedy_acceptance_batch(drafts, logits) == _oracle(logits, drafts)
