"""Restatement of linear verification rows and greedy acceptance (host integers).

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Reference: ``swiftLLM/swiftllm/speculative.py``
  * ``build_linear_verification_plan`` ``:75-89``: tokens ``[anchor, *draft]``,
    ``seq_lens`` ``base+0 .. base+k`` with ``base = prompt_len + len(outputs)``;
  * ``compute_greedy_acceptance`` ``:122-156``: longest prefix with
    ``posterior[i] == draft[i]`` plus the posterior token at the first mismatch,
    truncated by the output budget and at the first stop token.
Known answers: ``swiftLLM/tests/test_speculative_planning.py:25-178``.
"""
from __future__ import annotations


def linear_rows(prompt_len: int, output_token_ids: list[int], draft: list[int]):
    if not output_token_ids:
        raise ValueError("linear speculative verification requires an unstored anchor token")
    tokens = [output_token_ids[-1]] + list(draft)
    base = prompt_len + len(output_token_ids)
    return tokens, [base + i for i in range(len(tokens))]


def greedy_accept(draft: list[int], posterior: list[int], remaining: int | None = None,
                  stops=()) -> tuple[list[int], int]:
    if remaining is not None and remaining < 0:
        raise ValueError("remaining_output_len must be non-negative")
    if len(posterior) < len(draft) + 1:
        raise ValueError("posterior_token_ids must contain K+1 tokens for K draft tokens")
    n = 0
    while n < len(draft) and posterior[n] == draft[n]:
        n += 1
    out = list(draft[:n]) + [posterior[n]]
    if remaining is not None:
        out = out[:remaining]
    stop_set = frozenset(int(t) for t in stops)
    if any(t < 0 for t in stop_set):
        raise ValueError("stop_token_ids must be non-negative")
    for i, t in enumerate(out):
        if t in stop_set:
            out = out[:i + 1]
            break
    return out, min(n, len(out))
