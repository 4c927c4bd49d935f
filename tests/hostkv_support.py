"""A small in-process HostKV arena and copy-plan types for the tests.

They carry exactly the surface ``NativeCopyBackend`` uses of the reference's
``SharedHostKVArena`` / ``HostKVExtent`` / ``CopyRegion`` / ``CopyPlan``
(``nebulasd/src/nebulasd/kv/arena.py``, ``kv/transfer.py:15-46``): K plane at
offset 0, V plane right after it, extents addressed in blocks, the same
validation errors.  Host memory is a page-aligned numpy buffer.
"""
from __future__ import annotations

import dataclasses

import numpy as np


@dataclasses.dataclass(frozen=True)
class ArenaHandle:
    offset_blocks: int
    block_count: int
    generation: int

    def within_blocks(self, total: int) -> bool:
        return 0 <= self.offset_blocks and self.offset_blocks + self.block_count <= total


@dataclasses.dataclass(frozen=True)
class Extent:
    arena: ArenaHandle
    capacity_blocks: int

    @property
    def offset_blocks(self) -> int:
        return self.arena.offset_blocks


@dataclasses.dataclass(frozen=True)
class Descriptor:
    block_bytes: int
    total_blocks: int
    k_plane_offset: int
    v_plane_offset: int
    plane_bytes: int
    total_bytes: int
    dtype: str
    kv_block_shape: tuple
    descriptor_generation: int = 1


class Arena:
    def __init__(self, total_blocks: int, block_bytes: int, dtype: str = "torch.float16", kv_block_shape=()):
        plane = total_blocks * block_bytes
        self._raw = np.zeros(2 * plane + 8192, dtype=np.uint8)
        off = (-self._raw.ctypes.data) % 4096
        self.buf = self._raw[off:off + 2 * plane]
        self.descriptor = Descriptor(block_bytes, total_blocks, 0, plane, plane, 2 * plane, dtype,
                                     tuple(kv_block_shape))

    def address(self) -> int:
        return self.buf.ctypes.data

    def planes(self):
        p = self.descriptor.plane_bytes
        return self.buf[:p], self.buf[p:]

    def make_extent(self, offset_blocks: int, capacity_blocks: int, generation: int = 1) -> Extent:
        return Extent(ArenaHandle(offset_blocks, capacity_blocks, generation), capacity_blocks)

    def _validate_extent(self, extent: Extent) -> None:
        if extent.arena.generation != self.descriptor.descriptor_generation:
            raise ValueError("HostKV extent generation does not match arena descriptor")
        if extent.arena.block_count != extent.capacity_blocks:
            raise ValueError("HostKV handle block count must match extent capacity")
        if not extent.arena.within_blocks(self.descriptor.total_blocks):
            raise ValueError("HostKV extent exceeds arena capacity")


@dataclasses.dataclass(frozen=True)
class CopyRegion:
    extent: Extent
    gpu_begin_block: int
    host_begin_block: int
    block_count: int

    def __post_init__(self):
        if min(self.gpu_begin_block, self.host_begin_block, self.block_count) < 0:
            raise ValueError("negative copy range")
        if self.host_begin_block + self.block_count > self.extent.capacity_blocks:
            raise ValueError("copy exceeds HostKV extent")


@dataclasses.dataclass(frozen=True)
class CopyPlan:
    direction: str
    regions: tuple
    dependencies: tuple = ()
