"""Greedy speculative acceptance on the GPU: the verify forward's tail without a host sync.

Replaces ``torch.argmax(logits, dim=1)``
(``swiftLLM/swiftllm/worker/layers/post_layer.py:72``), the ``.tolist()`` of
the posterior tokens (``swiftLLM/swiftllm/worker/model.py:465``) and the host
loop of ``compute_greedy_acceptance``
(``swiftLLM/swiftllm/speculative.py:122-156``).  ``greedy_accept`` leaves the
tokens to append, their count and the number of accepted drafts per request in
device memory; ``compute_greedy_acceptance_batch`` returns the reference's
``(tokens_to_append, num_accepted)`` tuples for a batch after one copy to the
host.
"""
from __future__ import annotations

import threading

import torch

from . import _lib

_lock = threading.Lock()
_buffers: dict[tuple[int, int], torch.Tensor] = {}
_stops: dict[tuple, torch.Tensor] = {}


def _stop_tensor(device: torch.device, stops: tuple) -> torch.Tensor:
    key = (device.index, stops)
    with _lock:
        t = _stops.get(key)
        if t is None:
            with torch.inference_mode(False):
                t = torch.tensor(list(stops) or [0], dtype=torch.int32, device=device)
            _stops[key] = t
        return t


def _workspace(device: torch.device, stream: torch.cuda.Stream, num_rows: int) -> torch.Tensor:
    need = _lib.lib.neb_greedy_accept_workspace_bytes(num_rows)
    key = (device.index, stream.cuda_stream)
    with _lock:
        buf = _buffers.get(key)
        if buf is None or buf.numel() < need:
            with torch.cuda.stream(stream), torch.inference_mode(False):
                buf = torch.zeros(max(need, 2 * (buf.numel() if buf is not None else 0), 4096), dtype=torch.uint8,
                                  device=device)
            _buffers[key] = buf
        return buf


def greedy_accept(logits: torch.Tensor, row_start: torch.Tensor, draft_tokens: torch.Tensor,
                  remaining: torch.Tensor | None = None, stop_token_ids=(), max_out: int | None = None,
                  stream: torch.cuda.Stream | None = None, out=None):
    """Per request r (rows ``row_start[r] .. row_start[r+1]-1``, its k drafts at
    ``draft_tokens[row_start[r] - r:]``): the arg-max of each row's logits, the
    longest prefix of drafts equal to them plus the next arg-max, cut at
    ``remaining[r]`` (-1: no budget) and after the first stop token.

    Returns device tensors ``(tokens [R, max_out] (-1 padded), count [R],
    num_accepted [R], argmax [num_rows])``; ``out`` may pass those four
    tensors (int32, contiguous) to be filled instead."""
    if logits.dtype != torch.float16 or logits.dim() != 2 or logits.stride(1) != 1:
        raise ValueError("logits must be a float16 [rows, vocab] tensor with contiguous rows")
    dev = logits.device
    for name, t in (("row_start", row_start), ("draft_tokens", draft_tokens)):
        if t.dtype != torch.int32 or t.device != dev or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous int32 tensor on {dev}")
    num_rows, vocab = logits.shape
    num_requests = row_start.numel() - 1
    if num_requests < 0 or draft_tokens.numel() != num_rows - num_requests:
        raise ValueError("draft_tokens must hold num_rows - num_requests tokens")
    if remaining is not None and (remaining.dtype != torch.int32 or remaining.numel() != num_requests
                                  or remaining.device != dev):
        raise ValueError("remaining must be an int32 tensor with one budget per request")
    stops = tuple(int(t) for t in stop_token_ids)
    if any(t < 0 for t in stops):
        raise ValueError("stop_token_ids must be non-negative")
    stream = stream or torch.cuda.current_stream(dev)
    stop_t = _stop_tensor(dev, stops)
    if out is not None:
        tokens, count, accepted, argmax = out
        max_out = tokens.shape[1]
        if (tokens.dtype != torch.int32 or not tokens.is_contiguous() or tokens.shape[0] < num_requests
                or count.numel() < num_requests or accepted.numel() < num_requests or argmax.numel() < num_rows):
            raise ValueError("out tensors are too small or not contiguous int32")
    else:
        if max_out is None:
            max_out = num_rows - num_requests + 1 if num_requests else 1
        tokens = torch.empty((max(num_requests, 1), max_out), dtype=torch.int32, device=dev)
        count = torch.empty(max(num_requests, 1), dtype=torch.int32, device=dev)
        accepted = torch.empty_like(count)
        argmax = torch.empty(max(num_rows, 1), dtype=torch.int32, device=dev)
    ws = _workspace(dev, stream, num_rows)
    rc = _lib.lib.neb_greedy_accept(
        logits.data_ptr(), logits.stride(0), vocab, num_rows, row_start.data_ptr(), num_requests,
        draft_tokens.data_ptr(), remaining.data_ptr() if remaining is not None else None, stop_t.data_ptr(),
        len(stops), max_out, argmax.data_ptr(), tokens.data_ptr(), count.data_ptr(), accepted.data_ptr(),
        ws.data_ptr(), ws.numel(), stream.cuda_stream)
    _lib.check(rc, "neb_greedy_accept")
    return tokens[:num_requests], count[:num_requests], accepted[:num_requests], argmax[:num_rows]


def workspace_errors(stream: torch.cuda.Stream | None = None, device: torch.device | None = None) -> int:
    """Synchronise and return (and clear) the error bits of this stream's accept workspace."""
    import ctypes
    device = device or torch.device("cuda", torch.cuda.current_device())
    stream = stream or torch.cuda.current_stream(device)
    ws = _workspace(device, stream, 1)
    bits = ctypes.c_uint32(0)
    _lib.check(_lib.lib.neb_workspace_status(ws.data_ptr(), ctypes.byref(bits), stream.cuda_stream),
               "neb_workspace_status")
    return bits.value


def compute_greedy_acceptance_batch(drafts: list[list[int]], logits: torch.Tensor,
                                    remaining_output_len: list[int | None] | None = None,
                                    stop_token_ids=()) -> list[tuple[list[int], int]]:
    """``compute_greedy_acceptance`` for every request of a verify batch, from the
    logits of its rows (request r's k + 1 rows follow request r - 1's)."""
    dev = logits.device
    rows = [len(d) + 1 for d in drafts]
    starts = [0]
    for n in rows:
        starts.append(starts[-1] + n)
    if starts[-1] != logits.shape[0]:
        raise ValueError("posterior_token_ids must contain K+1 tokens for K draft tokens")
    budgets = None
    if remaining_output_len is not None:
        if any(b is not None and b < 0 for b in remaining_output_len):
            raise ValueError("remaining_output_len must be non-negative")
        budgets = torch.tensor([-1 if b is None else b for b in remaining_output_len], dtype=torch.int32).to(dev)
    # Row starts and drafts go up in one copy; the results come back in one.
    nreq, ndraft, max_out = len(drafts), starts[-1] - len(drafts), max(rows)
    host = torch.tensor(starts + [t for d in drafts for t in d], dtype=torch.int32).pin_memory()
    inputs = host.to(dev, non_blocking=True)
    result = torch.empty(nreq * max_out + 2 * nreq + logits.shape[0], dtype=torch.int32, device=dev)
    o_tok = result[:nreq * max_out].view(nreq, max_out)
    o_cnt = result[nreq * max_out:nreq * max_out + nreq]
    o_acc = result[nreq * max_out + nreq:nreq * max_out + 2 * nreq]
    o_am = result[nreq * max_out + 2 * nreq:]
    greedy_accept(logits, inputs[:nreq + 1], inputs[nreq + 1:nreq + 1 + ndraft], budgets, stop_token_ids,
                  out=(o_tok, o_cnt, o_acc, o_am))
    res = result.cpu().tolist()
    t = [res[r * max_out:(r + 1) * max_out] for r in range(nreq)]
    c, a = res[nreq * max_out:nreq * max_out + nreq], res[nreq * max_out + nreq:nreq * max_out + 2 * nreq]
    return [(t[r][:c[r]], a[r]) for r in range(nreq)]
