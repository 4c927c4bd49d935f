"""GPU: NativeCopyBackend dropped under the reference's own HostKV objects.

The reference's ``SharedHostKVArena`` (``nebulasd/src/nebulasd/kv/arena.py``),
its ``HostRegistrationPool`` with the portable-only registration it makes
(``cudaHostRegister`` flag 1, ``kv/host_registration.py:83``) and its
``CopyExecutor`` (``kv/transfer.py:96-172``) with H2D chunking and grouping
drive ``NativeCopyBackend`` exactly as the DMA process drives
``CudaCopyBackend``.  Payload and guard blocks are checked byte for byte, as
in the reference's copy fixture (``nebulasd/tests/support/copy_benchmark.py:67-103``).
The reference packages come from ``baseline/_ref`` (an offline install of the
reference); without them the tests skip.
"""
import ctypes

import numpy as np
import pytest
import torch

from baseline import reference as R
from oracle import hostkv as oracle

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not R.available(), reason="reference not installed under baseline/_ref")]

SHAPE = (2, 2, 16, 128)  # [layers, kv_heads, block, head_dim] -> 16 KiB blocks


def _host_bytes(arena):
    total = arena.descriptor.total_bytes
    return np.ctypeslib.as_array((ctypes.c_uint8 * total).from_address(arena.address()))


def _setup(batch, blocks, dev):
    arena_mod = R.nebulasd("kv.arena")
    cap = blocks + 2
    k = torch.empty((batch * cap, *SHAPE), dtype=torch.float16, device=dev)
    v = torch.empty_like(k)
    bb = k[0].numel() * 2
    arena = arena_mod.SharedHostKVArena.create(total_blocks=batch * cap, block_bytes=bb, dtype=str(k.dtype),
                                               kv_block_shape=SHAPE)
    extents = [arena.make_extent(request_slot=i, request_epoch=1, host_slot=i, host_slot_generation=1,
                                 writer_lease_generation=1, offset_blocks=i * cap, capacity_blocks=cap)
               for i in range(batch)]
    return k, v, arena, extents, cap, bb


def _fill(host, plane_bytes, k, v, cap, blocks, batch, bb, direction, it):
    for slot in range(batch):
        for plane, cache in enumerate((k, v)):
            base = slot * cap
            h = host[plane * plane_bytes:(plane + 1) * plane_bytes]
            cache[base:base + cap].view(torch.uint8).fill_(204)
            h[base * bb:(base + cap) * bb] = 221
            val = oracle.guard_pattern(plane, slot, it)
            if direction == "D2H":
                cache[base + 1:base + 1 + blocks].view(torch.uint8).fill_(val)
            else:
                h[(base + 1) * bb:(base + 1 + blocks) * bb] = val


def _check(host, plane_bytes, k, v, cap, blocks, batch, bb, it):
    for slot in range(batch):
        for plane, cache in enumerate((k, v)):
            base = slot * cap
            gpu = cache[base:base + cap].view(torch.uint8).cpu().numpy().reshape(-1)
            h = host[plane * plane_bytes:(plane + 1) * plane_bytes][base * bb:(base + cap) * bb]
            val = oracle.guard_pattern(plane, slot, it)
            assert (gpu[bb:-bb] == val).all() and (h[bb:-bb] == val).all(), "copy payload mismatch"
            assert (h[:bb] == 221).all() and (h[-bb:] == 221).all(), "HostKV guard overwritten"
            assert (gpu[:bb] == 204).all() and (gpu[-bb:] == 204).all(), "GPU guard overwritten"


@pytest.mark.parametrize("mode", ["auto", "memcpy"])
def test_reference_arena_executor_and_registration(mode, cuda):
    """Restore/writeback round trips through the reference's executor, chunked and grouped H2D."""
    from nebulasd_b200.hostkv import NativeCopyBackend
    tr = R.nebulasd("kv.transfer")
    pool = R.nebulasd("kv.registration_pool").HostRegistrationPool()
    batch, blocks = 5, 3
    k, v, arena, extents, cap, bb = _setup(batch, blocks, cuda)
    host = _host_bytes(arena)
    plane_bytes = arena.descriptor.plane_bytes
    backend = NativeCopyBackend(arena=arena, k_cache=k, v_cache=v, registration_pool=pool, mode=mode)
    # Two blocks per H2D chunk, two chunks per group: the executor splits each
    # restore plan into several backend launches, as the DMA process does.
    executor = tr.CopyExecutor(backend, h2d_chunk_bytes=2 * bb, h2d_group_size=2, h2d_wait_mode="event")
    try:
        for it, direction in enumerate(("D2H", "H2D", "D2H", "H2D")):
            plan = tr.CopyPlan(direction, tuple(tr.CopyRegion(e, i * cap + 1, 1, blocks)
                                                for i, e in enumerate(extents)))
            _fill(host, plane_bytes, k, v, cap, blocks, batch, bb, direction, it)
            torch.cuda.synchronize()
            receipt = executor.submit(plan).result(timeout=60)
            assert receipt.duration_ms >= 0
            torch.cuda.synchronize()
            _check(host, plane_bytes, k, v, cap, blocks, batch, bb, it)
        # Under the portable-only registration the arena may or may not be
        # device-mapped; auto takes the kernel only when it is.
        assert backend.mode in (("kernel", "memcpy") if mode == "auto" else ("memcpy",))
    finally:
        executor.close()
        del host
        arena.close()
        arena.unlink()


def test_reference_backend_and_native_backend_agree(cuda):
    """The reference's own CudaCopyBackend and NativeCopyBackend leave identical bytes."""
    from nebulasd_b200.hostkv import NativeCopyBackend
    tr = R.nebulasd("kv.transfer")
    ct = R.nebulasd("kv.cuda_transfer")
    batch, blocks = 4, 5
    k, v, arena, extents, cap, bb = _setup(batch, blocks, cuda)
    host = _host_bytes(arena)
    rng = np.random.default_rng(5)
    host[:] = rng.integers(0, 256, host.shape[0], dtype=np.uint8)
    pool = R.nebulasd("kv.registration_pool").HostRegistrationPool()
    ours = NativeCopyBackend(arena=arena, k_cache=k, v_cache=v, registration_pool=pool)
    k2, v2 = torch.zeros_like(k), torch.zeros_like(v)
    ref = ct.CudaCopyBackend(arena=arena, k_cache=k2, v_cache=v2, registration_pool=pool)
    try:
        k.zero_()
        v.zero_()
        plan = tr.CopyPlan("H2D", tuple(tr.CopyRegion(e, i * cap + 1, 1, blocks) for i, e in enumerate(extents)))
        ours.launch(plan).synchronize()
        t = ref.launch(plan)
        while not t.query():
            pass
        torch.cuda.synchronize()
        assert torch.equal(k.view(torch.uint8), k2.view(torch.uint8))
        assert torch.equal(v.view(torch.uint8), v2.view(torch.uint8))
        assert int(k.view(torch.uint8).count_nonzero()) > 0
    finally:
        ours.close()
        ref.close()
        del host
        arena.close()
        arena.unlink()


@pytest.mark.parametrize("mode", ["auto", "staged", "kernel"])
def test_reference_dma_windows(mode, cuda):
    """Restore plans cut by the reference DMA process's window policy
    (``bounded_regions``, ``nebulasd/src/nebulasd/workers/dma_process.py:21-37``,
    here a two-block window) run through NativeCopyBackend under the
    reference's CopyExecutor leave the arena's bytes in the GPU blocks."""
    from nebulasd_b200.hostkv import NativeCopyBackend
    tr = R.nebulasd("kv.transfer")
    dma = R.nebulasd("workers.dma_process")
    batch, blocks = 4, 7
    k, v, arena, extents, cap, bb = _setup(batch, blocks, cuda)
    host = _host_bytes(arena)
    plane_bytes = arena.descriptor.plane_bytes
    backend = NativeCopyBackend(arena=arena, k_cache=k, v_cache=v, mode=mode)
    executor = tr.CopyExecutor(backend, h2d_wait_mode="event")
    try:
        plan = tr.CopyPlan("H2D", tuple(tr.CopyRegion(e, i * cap + 1, 1, blocks) for i, e in enumerate(extents)))
        windowed = dma.bounded_regions(plan, bb, 2 * 2 * bb)
        assert len(windowed.regions) == batch * ((blocks + 1) // 2)
        _fill(host, plane_bytes, k, v, cap, blocks, batch, bb, "H2D", 3)
        torch.cuda.synchronize()
        executor.submit(windowed).result(timeout=60)
        torch.cuda.synchronize()
        _check(host, plane_bytes, k, v, cap, blocks, batch, bb, 3)
    finally:
        executor.close()
        del host
        arena.close()
        arena.unlink()
