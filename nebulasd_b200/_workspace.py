"""Device scratch for the attention kernels, one buffer per (device, stream).

The split-K kernels keep per-unit arrival counters and per-slot fp32 partials
in this buffer, and the verify kernel the work plan of its previous call (its
plan cache: calls on one buffer must be ordered on one stream) (the reference allocates its fp32 ``mid_o`` partials with
``torch.empty`` on every call, ``swiftLLM/swiftllm/worker/kernels/paged_attn.py:170-180``).
The counters must be zero when a call starts, and every call leaves them at
zero, so a buffer is zero-filled once when it is created and then reused by
the calls queued on its stream; calls on different streams (the compute
stream and the decoding piggyback stream of ``transformer_layer.py:169-185``,
or the two bank streams) get separate buffers, so they never race.
"""
from __future__ import annotations

import threading

import torch

from . import _lib

_lock = threading.Lock()
_buffers: dict[tuple[int, int], torch.Tensor] = {}


def attention_workspace(kernel: int, device: torch.device, stream: torch.cuda.Stream, num_rows: int,
                        num_q_heads: int, num_kv_heads: int) -> torch.Tensor:
    index = device.index if device.index is not None else torch.cuda.current_device()
    need = _lib.lib.neb_attention_workspace_bytes(kernel, index, max(num_rows, 1), num_q_heads, num_kv_heads)
    if need == 0:
        raise _lib.NebError(f"attention kernel {kernel} does not support {num_q_heads} q heads over "
                            f"{num_kv_heads} kv heads on device {index}")
    key = (index, stream.cuda_stream)
    with _lock:
        buf = _buffers.get(key)
        if buf is None or buf.numel() < need:
            # Round up so that slowly growing batches do not reallocate every call.
            size = max(need, 2 * buf.numel() if buf is not None else 0, 1 << 20)
            # Long-lived buffers are never inference tensors, even when the first
            # call comes from inside ``torch.inference_mode()`` (the reference's
            # model forward): callers may update them in place outside it.
            with torch.cuda.stream(stream), torch.inference_mode(False):
                buf = torch.zeros(size, dtype=torch.uint8, device=torch.device("cuda", index))
            _buffers[key] = buf
        return buf


def workspace_errors(buf: torch.Tensor, stream: torch.cuda.Stream) -> int:
    """Synchronise ``stream`` and return (and clear) the kernels' recorded error bits."""
    import ctypes
    bits = ctypes.c_uint32(0)
    _lib.check(_lib.lib.neb_workspace_status(buf.data_ptr(), ctypes.byref(bits), stream.cuda_stream),
               "neb_workspace_status")
    return bits.value


# Bumped whenever buffers are dropped, so that callers keeping a reference to
# the last buffer they used look it up again.
generation = 0


def release_all() -> None:
    global generation
    with _lock:
        _buffers.clear()
        generation += 1


_error_words: dict[int, torch.Tensor] = {}


def error_word(device: torch.device) -> torch.Tensor:
    """Per-device int32 where the store/RoPE kernels record out-of-range block ids (never a trap)."""
    index = device.index if device.index is not None else torch.cuda.current_device()
    with _lock:
        t = _error_words.get(index)
        if t is None:
            with torch.inference_mode(False):  # see attention_workspace
                t = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", index))
            _error_words[index] = t
        return t
