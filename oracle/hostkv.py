"""Byte-level restatement of HostKV restore/writeback and same-role migration.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Reference: ``nebulasd/src/nebulasd/kv/cuda_transfer.py:95-106``.  For every
region and for each plane (K at ``k_plane_offset``, V at ``v_plane_offset``):

    host = arena + plane + (extent.offset_blocks + host_begin_block) * block_bytes
    gpu  = cache + gpu_begin_block * block_bytes
    copy block_count * block_bytes bytes (D2H: gpu -> host, H2D: host -> gpu)

Regions are applied in order (a later region overwrites an earlier one where
they overlap, the order in which the reference's single stream executes its
``cudaMemcpyAsync`` calls).  Migration (``nebulasd/docs/current/KV.md:3-22``)
is a writeback on the source worker followed by a restore on the destination;
a direct peer copy must leave the destination bytes exactly as that two-step
path would.
"""
from __future__ import annotations

import numpy as np


def apply_regions(direction: str, regions, host_planes: tuple[np.ndarray, np.ndarray],
                  gpu_planes: tuple[np.ndarray, np.ndarray], block_bytes: int) -> None:
    """Apply ``(host_block, gpu_block, count)`` regions to uint8 buffers in place.

    ``host_block`` is already ``extent.offset_blocks + host_begin_block``.
    """
    if direction not in ("D2H", "H2D"):
        raise ValueError("direction must be D2H or H2D")
    for host_block, gpu_block, count in regions:
        n = count * block_bytes
        h0, g0 = host_block * block_bytes, gpu_block * block_bytes
        for host, gpu in zip(host_planes, gpu_planes):
            if direction == "D2H":
                host[h0:h0 + n] = gpu[g0:g0 + n]
            else:
                gpu[g0:g0 + n] = host[h0:h0 + n]


def migrate(src_planes, dst_planes, regions, block_bytes: int) -> None:
    """Peer migration ``(src_block, dst_block, count)``: bytes move unchanged, in order."""
    for src_block, dst_block, count in regions:
        n = count * block_bytes
        for src, dst in zip(src_planes, dst_planes):
            dst[dst_block * block_bytes:dst_block * block_bytes + n] = src[src_block * block_bytes:src_block * block_bytes + n]


def guard_pattern(plane: int, slot: int, iteration: int) -> int:
    """Fill byte of ``nebulasd/tests/support/copy_benchmark.py:67-68``."""
    return 1 + (plane * 79 + slot * 7 + iteration) % 180


def fill_table(block_table: np.ndarray, rows, begins, counts) -> None:
    """``block_table[row, :count] = arange(begin, begin + count)``.

    Restates ``nebulasd/src/nebulasd/workers/target/backend.py:71-84`` and
    ``workers/dma_process.py:95-125`` (the bank layout of ``workers/banks.py:43-60``).
    """
    for row, begin, count in zip(rows, begins, counts):
        block_table[row, :count] = np.arange(begin, begin + count, dtype=block_table.dtype)
