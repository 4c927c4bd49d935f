"""GPU: HostKV restore/writeback and peer migration, bit-exact with guard blocks.

Follows the reference's copy fixture (``nebulasd/tests/support/copy_benchmark.py:11-103``):
every request extent and GPU range has a guard block on each side, payload
blocks get a per-(plane, slot, iteration) byte pattern, guards must survive.
"""
import numpy as np
import pytest
import torch

from oracle import hostkv as oracle
from tests.hostkv_support import Arena, CopyPlan, CopyRegion

pytestmark = pytest.mark.gpu

SHAPE = (2, 2, 16, 128)  # [layers, kv_heads, block, head_dim] -> 16 KiB blocks


def _setup(batch, blocks, dev):
    cap = blocks + 2
    k = torch.empty((batch * cap, *SHAPE), dtype=torch.float16, device=dev)
    v = torch.empty_like(k)
    bb = k[0].numel() * 2
    arena = Arena(batch * cap, bb, dtype=str(k.dtype), kv_block_shape=SHAPE)
    extents = [arena.make_extent(i * cap, cap) for i in range(batch)]
    return k, v, arena, extents, cap, bb


def _fill(arena, extents, k, v, cap, blocks, direction, it):
    hk, hv = arena.planes()
    bb = arena.descriptor.block_bytes
    for slot, ext in enumerate(extents):
        for plane, (cache, host) in enumerate(((k, hk), (v, hv))):
            base = slot * cap
            cache[base:base + cap].view(torch.uint8).fill_(204)
            host[base * bb:(base + cap) * bb] = 221
            val = oracle.guard_pattern(plane, slot, it)
            if direction == "D2H":
                cache[base + 1:base + 1 + blocks].view(torch.uint8).fill_(val)
            else:
                host[(base + 1) * bb:(base + 1 + blocks) * bb] = val


def _check(arena, extents, k, v, cap, blocks, it):
    hk, hv = arena.planes()
    bb = arena.descriptor.block_bytes
    for slot, ext in enumerate(extents):
        for plane, (cache, host) in enumerate(((k, hk), (v, hv))):
            base = slot * cap
            gpu = cache[base:base + cap].view(torch.uint8).cpu().numpy().reshape(-1)
            h = host[base * bb:(base + cap) * bb]
            val = oracle.guard_pattern(plane, slot, it)
            assert (gpu[bb:-bb] == val).all() and (h[bb:-bb] == val).all(), "copy payload mismatch"
            assert (h[:bb] == 221).all() and (h[-bb:] == 221).all(), "HostKV guard overwritten"
            assert (gpu[:bb] == 204).all() and (gpu[-bb:] == 204).all(), "GPU guard overwritten"


@pytest.mark.parametrize("mode", ["kernel", "memcpy", "staged"])
def test_copy_backend_guard_blocks(mode, cuda):
    from nebulasd_b200.hostkv import NativeCopyBackend
    batch, blocks = 5, 3
    k, v, arena, extents, cap, bb = _setup(batch, blocks, cuda)
    backend = NativeCopyBackend(arena=arena, k_cache=k, v_cache=v, mode=mode)
    try:
        for it, direction in enumerate(("D2H", "H2D", "D2H", "H2D")):
            plan = CopyPlan(direction, tuple(CopyRegion(e, i * cap + 1, 1, blocks) for i, e in enumerate(extents)))
            _fill(arena, extents, k, v, cap, blocks, direction, it)
            torch.cuda.synchronize()
            ticket = backend.launch(plan)
            ticket.synchronize()
            assert ticket.query() and ticket.duration_ms() >= 0
            _check(arena, extents, k, v, cap, blocks, it)
        assert backend.mode == mode
    finally:
        backend.close()


@pytest.mark.parametrize("mode", ["kernel", "memcpy", "staged"])
def test_random_regions_match_oracle(mode, cuda):
    from nebulasd_b200.hostkv import NativeCopyBackend
    rng = np.random.default_rng(5)
    nb = 64
    k = torch.randint(-1000, 1000, (nb, *SHAPE), device=cuda).half()
    v = torch.randint(-1000, 1000, (nb, *SHAPE), device=cuda).half()
    bb = k[0].numel() * 2
    arena = Arena(96, bb, dtype=str(k.dtype), kv_block_shape=SHAPE)
    hk, hv = arena.planes()
    hk[:] = rng.integers(0, 256, hk.shape, dtype=np.uint8)
    hv[:] = rng.integers(0, 256, hv.shape, dtype=np.uint8)
    ext = arena.make_extent(8, 80)
    backend = NativeCopyBackend(arena=arena, k_cache=k, v_cache=v, mode=mode)
    try:
        for direction in ("D2H", "H2D"):
            # disjoint destinations: consecutive, non-overlapping host and GPU ranges in shuffled order
            cuts = np.sort(rng.choice(np.arange(1, 60), 6, replace=False))
            spans = list(zip(np.r_[0, cuts], np.r_[cuts, 60]))
            order = rng.permutation(len(spans))
            regions = tuple(CopyRegion(ext, int(a + 2), int(a + 10), int(b - a)) for a, b in (spans[i] for i in order))
            host_before = (hk.copy(), hv.copy())
            gpu_before = (k.view(torch.uint8).cpu().numpy().reshape(-1).copy(),
                          v.view(torch.uint8).cpu().numpy().reshape(-1).copy())
            backend.launch(CopyPlan(direction, regions)).synchronize()
            triples = [(ext.offset_blocks + r.host_begin_block, r.gpu_begin_block, r.block_count) for r in regions]
            oracle.apply_regions(direction, triples, host_before, gpu_before, bb)
            assert np.array_equal(hk, host_before[0]) and np.array_equal(hv, host_before[1])
            assert np.array_equal(k.view(torch.uint8).cpu().numpy().reshape(-1), gpu_before[0])
            assert np.array_equal(v.view(torch.uint8).cpu().numpy().reshape(-1), gpu_before[1])
    finally:
        backend.close()


def test_copy_backend_rejects_out_of_range(cuda):
    from nebulasd_b200.hostkv import NativeCopyBackend
    k, v, arena, extents, cap, bb = _setup(2, 2, cuda)
    backend = NativeCopyBackend(arena=arena, k_cache=k, v_cache=v)
    try:
        with pytest.raises(ValueError, match="copy exceeds GPU KV cache"):
            backend.launch(CopyPlan("H2D", (CopyRegion(extents[0], k.shape[0] - 1, 0, 2),)))
    finally:
        backend.close()


@pytest.mark.parametrize("mode", ["kernel", "memcpy"])
def test_migration_matches_writeback_then_restore(mode, cuda):
    from nebulasd_b200.hostkv import migrate_blocks
    ndev = torch.cuda.device_count()
    src_dev = cuda
    dst_dev = torch.device("cuda", 1) if ndev > 1 else cuda
    g = torch.Generator(device=src_dev).manual_seed(3)
    sk = torch.randn((40, *SHAPE), generator=g, device=src_dev).half()
    sv = torch.randn((40, *SHAPE), generator=g, device=src_dev).half()
    dk = torch.zeros((50, *SHAPE), dtype=torch.float16, device=dst_dev)
    dv = torch.zeros_like(dk)
    regions = [(0, 10, 7), (20, 30, 12), (35, 0, 5)]
    migrate_blocks(sk, sv, dk, dv, regions, mode=mode)
    torch.cuda.synchronize(dst_dev)
    bb = sk[0].numel() * 2
    src = (sk.view(torch.uint8).cpu().numpy().reshape(-1), sv.view(torch.uint8).cpu().numpy().reshape(-1))
    exp = (np.zeros(50 * bb, np.uint8), np.zeros(50 * bb, np.uint8))
    oracle.migrate(src, exp, regions, bb)
    assert np.array_equal(dk.view(torch.uint8).cpu().numpy().reshape(-1), exp[0])
    assert np.array_equal(dv.view(torch.uint8).cpu().numpy().reshape(-1), exp[1])


def test_fork_shares_its_own_registration(cuda):
    """A backend that registered the arena itself and its fork (the second
    bank's stream) share that registration: both copy, the arena is
    registered once and unregistered when the last of them closes."""
    from nebulasd_b200.hostkv import NativeCopyBackend, host_device_pointer
    batch, blocks = 3, 2
    k, v, arena, extents, cap, bb = _setup(batch, blocks, cuda)
    be = NativeCopyBackend(arena=arena, k_cache=k, v_cache=v, mode="kernel")
    be.initialize()
    other = be.fork()
    other.initialize()
    for it, (backend, direction) in enumerate(((be, "H2D"), (other, "D2H"), (other, "H2D"), (be, "D2H"))):
        plan = CopyPlan(direction, tuple(CopyRegion(e, i * cap + 1, 1, blocks) for i, e in enumerate(extents)))
        _fill(arena, extents, k, v, cap, blocks, direction, it)
        torch.cuda.synchronize()
        backend.launch(plan).synchronize()
        _check(arena, extents, k, v, cap, blocks, it)
    be.close()
    assert host_device_pointer(arena.address()) is not None  # the fork still holds it
    other.close()
    assert host_device_pointer(arena.address()) is None


def test_staged_restore_in_small_pieces(cuda, monkeypatch):
    """The staged restore cut into many 3-block pieces (both staging buffers
    reused over and over) leaves the same bytes as the oracle."""
    from nebulasd_b200 import hostkv
    rng = np.random.default_rng(9)
    nb = 64
    k = torch.zeros((nb, *SHAPE), dtype=torch.float16, device=cuda)
    v = torch.zeros_like(k)
    bb = k[0].numel() * 2
    monkeypatch.setattr(hostkv, "STAGING_BYTES", 3 * bb)
    arena = Arena(96, bb, dtype=str(k.dtype), kv_block_shape=SHAPE)
    hk, hv = arena.planes()
    hk[:] = rng.integers(0, 256, hk.shape, dtype=np.uint8)
    hv[:] = rng.integers(0, 256, hv.shape, dtype=np.uint8)
    ext = arena.make_extent(4, 60)
    dst = rng.permutation(nb)[:40]  # 40 one-block regions of one arena range, scattered GPU blocks
    regions = tuple(CopyRegion(ext, int(g), j, 1) for j, g in enumerate(dst))
    backend = hostkv.NativeCopyBackend(arena=arena, k_cache=k, v_cache=v, mode="staged")
    try:
        gpu_before = (k.view(torch.uint8).cpu().numpy().reshape(-1).copy(),
                      v.view(torch.uint8).cpu().numpy().reshape(-1).copy())
        host_before = (hk.copy(), hv.copy())
        backend.launch(CopyPlan("H2D", regions)).synchronize()
        assert backend.last_mode == "staged"
        triples = [(ext.offset_blocks + r.host_begin_block, r.gpu_begin_block, r.block_count) for r in regions]
        oracle.apply_regions("H2D", triples, host_before, gpu_before, bb)
        assert np.array_equal(k.view(torch.uint8).cpu().numpy().reshape(-1), gpu_before[0])
        assert np.array_equal(v.view(torch.uint8).cpu().numpy().reshape(-1), gpu_before[1])
    finally:
        backend.close()
