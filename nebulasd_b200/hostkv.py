"""HostKV restore/writeback and same-role KV migration on the native copy path.

``NativeCopyBackend`` is a drop-in for ``nebulasd.kv.cuda_transfer.CudaCopyBackend``
(``nebulasd/src/nebulasd/kv/cuda_transfer.py:30-133``): same constructor
arguments, ``fork``/``initialize``/``launch``/``close``, and tickets with
``query``/``synchronize``/``duration_ms``, so ``CopyExecutor``, the per-bank DMA
process and the copy benchmark use it unchanged.  ``launch`` moves every region
of a ``CopyPlan`` (both planes) in ONE kernel launch that reads the pinned,
device-mapped host arena directly (``mode="kernel"``), or with one
``cudaMemcpyAsync`` per merged run of adjacent regions and plane
(``mode="memcpy"``, the reference's transfer engine); ``mode="auto"`` decides
per plan (``choose_copy_mode``): the copy engines for plans of long runs, where
they reach the PCIe roofline (55.6 GB/s on B200, against 51 GB/s for the
kernel), the single-launch kernel for plans of many short runs, where one
driver call per run and plane would dominate; the kernel needs the arena
mapped into the device address space.  A restore whose arena ranges are long
but whose GPU blocks are scattered (a request's KV into a paged pool) goes
``mode="staged"``: the copy engines move the ranges into a device staging
buffer and a device-to-device kernel scatters the blocks, so the restore holds
no SM while it waits on the host link and the attention of the other bank
keeps its speed.

``migrate_blocks`` is same-role migration as a direct peer copy over NVLink: the
destination GPU's kernel reads the source GPU's cache through its unified
address, leaving the destination bytes exactly as the reference's
writeback-then-restore through HostKV (``nebulasd/docs/current/KV.md:3-22``).
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _lib

MODES = {"memcpy": 0, "kernel": 1}


class NativeCopyTicket:
    def __init__(self, start: torch.cuda.Event, done: torch.cuda.Event) -> None:
        self.start, self.done = start, done

    def query(self) -> bool:
        return bool(self.done.query())

    def synchronize(self) -> None:
        self.done.synchronize()

    def duration_ms(self) -> float:
        return float(self.start.elapsed_time(self.done))


class _OwnRegistration:
    """cudaHostRegister(PORTABLE | MAPPED) when the caller supplies no registration pool.

    Counted per arena address, so that a backend and its forks (which share
    the registration, as the reference's ``fork`` does) register the arena
    once and unregister it when the last of them closes."""

    _lock = __import__("threading").Lock()
    _count: dict[int, int] = {}

    def acquire(self, arena):
        address = arena.address()
        with self._lock:
            if self._count.get(address, 0) == 0:
                cudart = torch.cuda.cudart()
                status = cudart.cudaHostRegister(address, arena.descriptor.total_bytes, 3)
                code = int(status[0] if isinstance(status, tuple) else status)
                if code != 0:
                    raise RuntimeError(f"cudaHostRegister failed with CUDA status {code}")
            self._count[address] = self._count.get(address, 0) + 1
        return address

    def release(self, record) -> None:
        with self._lock:
            left = self._count.get(record, 0) - 1
            if left > 0:
                self._count[record] = left
                return
            self._count.pop(record, None)
            cudart = torch.cuda.cudart()
            status = cudart.cudaHostUnregister(record)
            code = int(status[0] if isinstance(status, tuple) else status)
            if code != 0:
                raise RuntimeError(f"cudaHostUnregister failed with CUDA status {code}")


def plan_regions(plan, arena, gpu_blocks: int) -> np.ndarray:
    """``[n, 3]`` int64 ``(host_block, gpu_block, count)`` of a ``CopyPlan``.

    Applies the reference's per-launch checks (``cuda_transfer.py:320-323``):
    the extent must belong to the arena and the GPU range must fit the cache.
    ``host_block`` is ``extent.offset_blocks + host_begin_block`` (``:337``).
    """
    rows = []
    for region in plan.regions:
        arena._validate_extent(region.extent)
        if region.gpu_begin_block + region.block_count > gpu_blocks:
            raise ValueError("copy exceeds GPU KV cache")
        rows.append((region.extent.offset_blocks + region.host_begin_block, region.gpu_begin_block,
                     region.block_count))
    return np.asarray(rows, dtype=np.int64).reshape(-1, 3)


# Mean bytes per merged run and plane from which the copy engines are used.
ENGINE_RUN_BYTES = 1 << 20


def merged_runs(regions: np.ndarray) -> int:
    """Runs of regions adjacent on both sides (each run is one copy per plane)."""
    if len(regions) == 0:
        return 0
    host, gpu, count = regions[:, 0], regions[:, 1], regions[:, 2]
    cont = (host[1:] == host[:-1] + count[:-1]) & (gpu[1:] == gpu[:-1] + count[:-1])
    return int(len(regions) - np.count_nonzero(cont))


def host_runs(regions: np.ndarray) -> int:
    """Runs of regions adjacent in the arena (whatever their GPU blocks)."""
    if len(regions) == 0:
        return 0
    host, count = regions[:, 0], regions[:, 2]
    return int(len(regions) - np.count_nonzero(host[1:] == host[:-1] + count[:-1]))


# Device staging buffer of the staged restore, per plane and buffer (two buffers).
STAGING_BYTES = 64 << 20


def choose_copy_mode(regions: np.ndarray, block_bytes: int, mapped: bool, direction: str = "H2D") -> str:
    """Per plan: ``memcpy`` when its runs (adjacent on both sides) average
    ``ENGINE_RUN_BYTES`` or more per plane; for a restore whose arena ranges
    are that long but whose GPU blocks are scattered (a request's KV into a
    paged pool), ``staged``: the copy engines move the arena ranges into a
    device staging buffer and a device-to-device kernel scatters the blocks,
    so the restore holds no SM while it waits on the host link; else
    ``kernel`` (the arena must be mapped) or ``memcpy``."""
    runs = merged_runs(regions)
    if runs == 0:
        return "kernel" if mapped else "memcpy"
    total = int(regions[:, 2].sum()) * block_bytes
    if total >= ENGINE_RUN_BYTES * runs:
        return "memcpy"
    if direction == "H2D" and total >= ENGINE_RUN_BYTES * host_runs(regions):
        return "staged"
    return "kernel" if mapped else "memcpy"


def staged_pieces(regions: np.ndarray, capacity: int):
    """Cut a restore plan into pieces of at most ``capacity`` blocks: per piece
    the arena-to-staging regions and the staging-to-cache regions, both as
    ``(src_block, dst_block, count)`` rows in plan order."""
    if len(regions) == 0:
        return []
    host, gpu, count = regions[:, 0], regions[:, 1], regions[:, 2]
    end = np.cumsum(count)
    begin = end - count
    # A region crossing a piece boundary is cut there: one row per (region, piece).
    first, last = begin // capacity, (end - 1) // capacity
    reps = last - first + 1
    idx = np.repeat(np.arange(len(regions)), reps)
    piece = np.repeat(first, reps) + (np.arange(reps.sum()) - np.repeat(np.cumsum(reps) - reps, reps))
    lo = np.maximum(begin[idx], piece * capacity)
    hi = np.minimum(end[idx], (piece + 1) * capacity)
    src = host[idx] + (lo - begin[idx])
    dst = gpu[idx] + (lo - begin[idx])
    n = hi - lo
    slot = lo - piece * capacity
    bounds = np.flatnonzero(np.diff(piece)) + 1
    out = []
    for sel in np.split(np.arange(len(piece)), bounds):
        out.append((np.stack([src[sel], slot[sel], n[sel]], 1).astype(np.int64),
                    np.stack([slot[sel], dst[sel], n[sel]], 1).astype(np.int64)))
    return out


def host_device_pointer(host_address: int) -> int | None:
    """Device address of pinned host memory, or None if it is not mapped."""
    out = ctypes.c_void_p()
    rc = _lib.lib.neb_host_device_pointer(host_address, ctypes.byref(out))
    return out.value if rc == 0 else None


class NativeCopyBackend:
    def __init__(self, *, arena, k_cache, v_cache, registration=None, registration_pool=None,
                 mode: str = "auto") -> None:
        if (not k_cache.is_cuda or not v_cache.is_cuda
                or k_cache.device != v_cache.device or k_cache.dtype != v_cache.dtype
                or k_cache.shape != v_cache.shape
                or not k_cache.is_contiguous() or not v_cache.is_contiguous()):
            raise ValueError("copy backend requires matching contiguous CUDA KV caches")
        block_bytes = k_cache[0].numel() * k_cache.element_size()
        if arena.descriptor.block_bytes != block_bytes:
            raise ValueError("HostKV block byte size does not match GPU layout")
        if (arena.descriptor.dtype != str(k_cache.dtype)
                or tuple(arena.descriptor.kv_block_shape) != tuple(k_cache.shape[1:])):
            raise ValueError("HostKV dtype/block shape does not match GPU layout")
        if mode not in ("auto", "kernel", "memcpy", "staged"):
            raise ValueError("mode must be auto, kernel, memcpy or staged")
        self.arena = arena
        self.k_cache, self.v_cache = k_cache, v_cache
        self._device = k_cache.device
        self._mode_request = mode
        self._registration = registration_pool
        self._own_registration = registration_pool is None and registration is None
        if registration is not None and registration_pool is None:
            self._registration = _PoolAdapter(registration)
        self._record = None
        self._stream = None
        self._scatter_stream = None
        self._staging = None
        self.last_mode = None  # the mode the last launch used
        self._host_base = None  # address the copy uses for the arena (device-mapped or host)
        self._mapped = None     # device address of the arena, when it is mapped
        self.mode = None
        self._closed = False
        self._close_error = None

    def fork(self):
        """Own another stream/events, sharing only cache storage and registration."""
        other = type(self)(arena=self.arena, k_cache=self.k_cache, v_cache=self.v_cache,
                           registration_pool=self._registration, mode=self._mode_request)
        return other

    def initialize(self) -> None:
        if self._closed:
            raise RuntimeError("native copy backend is closed")
        torch.cuda.set_device(self._device)
        if self._stream is not None:
            return
        if self._registration is None:
            self._registration = _OwnRegistration()
        self._stream = torch.cuda.Stream(device=self._device)
        self._scatter_stream = torch.cuda.Stream(device=self._device)
        self._record = self._registration.acquire(self.arena)
        mapped = host_device_pointer(self.arena.address())
        if self._mode_request == "kernel" and mapped is None:
            raise RuntimeError("kernel copies need the HostKV arena mapped into the device address space")
        self._mapped = mapped
        if self._mode_request in ("memcpy", "staged") or mapped is None:
            self.mode, self._host_base = self._mode_request if self._mode_request != "auto" else "memcpy", \
                self.arena.address()
        else:
            self.mode, self._host_base = "kernel", mapped

    def launch(self, plan) -> NativeCopyTicket:
        self.initialize()
        if plan.direction not in ("D2H", "H2D"):
            raise ValueError("copy plan requires a direction")
        regions = plan_regions(plan, self.arena, self.k_cache.shape[0])
        d = self.arena.descriptor
        mode, host_base = self.mode, self._host_base
        if self._mode_request == "auto":
            mode = choose_copy_mode(regions, d.block_bytes, self._mapped is not None, plan.direction)
        if mode == "staged" and plan.direction != "H2D":  # writebacks: the direct path
            mode = "kernel" if self._mapped is not None else "memcpy"
        self.last_mode = mode
        host_base = self._mapped if mode == "kernel" else self.arena.address()
        with torch.cuda.stream(self._stream):
            for dependency in plan.dependencies:
                if hasattr(dependency, "query") and hasattr(dependency, "record"):
                    self._stream.wait_event(dependency)
            start = torch.cuda.Event(enable_timing=True)
            done = torch.cuda.Event(enable_timing=True, blocking=True)
            start.record(self._stream)
            if len(regions) and mode == "staged":
                self._staged_restore(regions, host_base)
            elif len(regions):
                rc = _lib.lib.neb_hostkv_copy(
                    1 if plan.direction == "H2D" else 0, host_base + d.k_plane_offset,
                    host_base + d.v_plane_offset, self.k_cache.data_ptr(), self.v_cache.data_ptr(),
                    d.block_bytes, regions.ctypes.data, len(regions), MODES[mode],
                    self._stream.cuda_stream)
                _lib.check(rc, "neb_hostkv_copy")
            done.record(self._stream)
        return NativeCopyTicket(start, done)

    def _staged_restore(self, regions: np.ndarray, host_base: int) -> None:
        """Arena ranges -> staging buffer (copy engines, backend stream) ->
        cache blocks (copy kernel, scatter stream), two buffers in flight; the
        backend stream waits for the last scatter."""
        d = self.arena.descriptor
        bb = d.block_bytes
        cap = max(1, STAGING_BYTES // bb)
        if self._staging is None:
            with torch.inference_mode(False):
                self._staging = torch.empty((2, 2, cap * bb), dtype=torch.uint8, device=self._device)
        scattered = []
        for i, (dma, scatter) in enumerate(staged_pieces(regions, cap)):
            buf = self._staging[i % 2]
            if i >= 2:
                self._stream.wait_event(scattered[i - 2])
            rc = _lib.lib.neb_hostkv_copy(1, host_base + d.k_plane_offset, host_base + d.v_plane_offset,
                                          buf[0].data_ptr(), buf[1].data_ptr(), bb, dma.ctypes.data, len(dma),
                                          MODES["memcpy"], self._stream.cuda_stream)
            _lib.check(rc, "neb_hostkv_copy")
            landed = torch.cuda.Event()
            landed.record(self._stream)
            self._scatter_stream.wait_event(landed)
            rc = _lib.lib.neb_kv_peer_copy(buf[0].data_ptr(), buf[1].data_ptr(), self.k_cache.data_ptr(),
                                           self.v_cache.data_ptr(), bb, scatter.ctypes.data, len(scatter),
                                           MODES["kernel"], self._scatter_stream.cuda_stream)
            _lib.check(rc, "neb_kv_peer_copy")
            ev = torch.cuda.Event()
            ev.record(self._scatter_stream)
            scattered.append(ev)
        self._stream.wait_event(scattered[-1])

    def close(self) -> None:
        if self._close_error is not None:
            raise self._close_error
        if self._closed:
            return
        self._closed = True
        try:
            if self._stream is not None:
                self._stream.synchronize()
                self._scatter_stream.synchronize()
            if self._record is not None:
                self._registration.release(self._record)
                self._record = None
        except BaseException as error:  # keep the reference's close-error contract
            self._close_error = error
            raise
        self._stream = self._scatter_stream = self._staging = None
        self.k_cache = self.v_cache = None


class _PoolAdapter:
    """Wraps a single registration adapter (reference ``CudaHostRegistrationAdapter``) as a pool."""

    def __init__(self, adapter) -> None:
        self.adapter = adapter

    def acquire(self, arena):
        return self.adapter.register(arena, executor_id=f"native-copy:{arena.address()}", process_generation=1)

    def release(self, record) -> None:
        self.adapter.unregister(record)


def migrate_blocks(src_k: torch.Tensor, src_v: torch.Tensor, dst_k: torch.Tensor, dst_v: torch.Tensor,
                   regions, *, mode: str = "kernel", stream: torch.cuda.Stream | None = None,
                   src_stream: torch.cuda.Stream | None = None) -> None:
    """Copy ``(src_block, dst_block, count)`` block ranges from one GPU's caches to another's.

    Runs on ``dst``'s device, on ``stream`` (default: its current stream).
    ``mode="kernel"`` reads the source cache over NVLink from a copy kernel
    (peer access is enabled on first use); ``mode="memcpy"`` issues peer
    ``cudaMemcpyAsync`` per merged run.  The copy is ordered after the work
    queued so far on ``src_stream`` (default: the source device's current
    stream), where the caller wrote the source KV, through an event the copy's
    stream waits on; the caller keeps the source blocks unchanged until the
    copy is done (``stream`` synchronised or waited on).
    """
    if src_k.shape[1:] != dst_k.shape[1:] or src_k.dtype != dst_k.dtype:
        raise ValueError("source and destination caches must share the block layout")
    arr = np.asarray(regions, dtype=np.int64).reshape(-1, 3)
    if len(arr) and ((arr[:, 0] + arr[:, 2]).max() > src_k.shape[0] or (arr[:, 1] + arr[:, 2]).max() > dst_k.shape[0]):
        raise ValueError("migration range exceeds a KV cache")
    block_bytes = src_k[0].numel() * src_k.element_size()
    src_s = src_stream or torch.cuda.current_stream(src_k.device)
    ready = torch.cuda.Event()
    ready.record(src_s)
    with torch.cuda.device(dst_k.device):
        if src_k.device != dst_k.device:
            _lib.check(_lib.lib.neb_enable_peer_access(src_k.device.index), "neb_enable_peer_access")
        s = stream or torch.cuda.current_stream(dst_k.device)
        s.wait_event(ready)
        rc = _lib.lib.neb_kv_peer_copy(src_k.data_ptr(), src_v.data_ptr(), dst_k.data_ptr(), dst_v.data_ptr(),
                                       block_bytes, arr.ctypes.data, len(arr), MODES[mode], s.cuda_stream)
        _lib.check(rc, "neb_kv_peer_copy")
