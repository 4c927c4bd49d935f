"""Host-side mirror of the attention kernels' work plan (``csrc/plan.cuh``).

The kernels build this plan on the device; this mirror exists so that the
partition arithmetic (groups, balanced tile ranges, piece slots, arrival
counts) can be checked exhaustively on the CPU, and so that tools can predict
how a batch is split.
"""
from __future__ import annotations

import dataclasses


def groups(seq_ids: list[int], seq_lens: list[int], max_group_rows: int):
    """``[(first_row, nrows, tiles)]``: adjacent same-seq rows, cut every ``max_group_rows``."""
    out = []
    run_start = 0
    for r in range(len(seq_ids)):
        seq_start = r == 0 or seq_ids[r] != seq_ids[r - 1]
        if seq_start:
            run_start = r
        if seq_start or (r - run_start) % max_group_rows == 0:
            out.append([r, 0, 0])
        out[-1][1] += 1
    res = []
    for first, n, _ in out:
        mx = max(seq_lens[first:first + n])
        res.append((first, n, (max(mx, 0) + 15) // 16))
    return res


def range_begin(w: int, total: int, workers: int) -> int:
    return (w * total) // workers


def worker_of(t: int, total: int, workers: int) -> int:
    return ((t + 1) * workers - 1) // total


class CostSplit:
    """Cost-weighted split of ``csrc/plan.cuh`` (``CostSplit``).

    Each unit (group, kv head) counts ``piece_cost`` virtual tiles ahead of
    its own tiles; workers split the virtual range ``[0, V)`` evenly and own
    the tiles whose virtual positions fall in their share.  ``piece_cost = 0``
    is the plain tile split (``range_begin`` / ``worker_of``).
    """

    def __init__(self, prefix: list[int], hk: int, piece_cost: int, workers: int):
        self.prefix, self.hk, self.pc = prefix, hk, piece_cost
        self.ng = len(prefix) - 1
        self.total = hk * prefix[-1]
        self.vtotal = self.total + piece_cost * hk * self.ng
        self.workers = min(workers, self.vtotal)

    def _find_group(self, t: int) -> int:   # largest g < ng with hk*prefix[g] <= t
        lo, hi = 0, self.ng
        while hi - lo > 1:
            mid = (lo + hi) // 2
            if self.hk * self.prefix[mid] <= t:
                lo = mid
            else:
                hi = mid
        return lo

    def _vbase(self, g: int) -> int:
        return self.hk * (self.prefix[g] + self.pc * g)

    def vpos(self, t: int) -> int:
        g = self._find_group(t)
        nb = self.prefix[g + 1] - self.prefix[g]
        h = (t - self.hk * self.prefix[g]) // nb
        return t + self.pc * (g * self.hk + h + 1)

    def tile_at(self, v: int) -> int:
        if v >= self.vtotal:
            return self.total
        lo, hi = 0, self.ng
        while hi - lo > 1:
            mid = (lo + hi) // 2
            if self._vbase(mid) <= v:
                lo = mid
            else:
                hi = mid
        nb = self.prefix[lo + 1] - self.prefix[lo]
        off = v - self._vbase(lo)
        h = off // (nb + self.pc)
        in_unit = off - h * (nb + self.pc)
        return self.hk * self.prefix[lo] + h * nb + max(0, in_unit - self.pc)

    def begin(self, w: int) -> int:
        return self.tile_at(w * self.vtotal // self.workers)

    def worker_of_tile(self, t: int) -> int:
        return ((self.vpos(t) + 1) * self.workers - 1) // self.vtotal


def piece_slot(w: int, w0: int) -> int:
    return 2 * w + 1 if w == w0 else 2 * w


@dataclasses.dataclass
class Piece:
    worker: int
    group: int
    kv_head: int
    tile_lo: int
    tile_hi: int
    whole: bool
    slot: int | None
    w0: int
    w1: int


def pieces(seq_ids, seq_lens, num_kv_heads: int, workers: int, max_group_rows: int,
           piece_cost: int = 0) -> list[Piece]:
    """Every piece every worker processes, in worker order (``piece_cost``: see CostSplit;
    the verify kernel uses 8, the decode kernel 0)."""
    gs = groups(seq_ids, seq_lens, max_group_rows)
    prefix = [0]
    for _, _, nb in gs:
        prefix.append(prefix[-1] + nb)
    total = num_kv_heads * prefix[-1]
    out = []
    if total == 0:
        return out
    # Only min(workers, V) workers take part.  Every worker strictly between a
    # split unit's first and last owns some of its tiles, so w0..w1 all report.
    split = CostSplit(prefix, num_kv_heads, piece_cost, workers)
    workers = split.workers
    for w in range(workers):
        t, t_end = split.begin(w), split.begin(w + 1)
        g = 0
        while t < t_end:
            while num_kv_heads * prefix[g + 1] <= t:
                g += 1
            nb = prefix[g + 1] - prefix[g]
            gbase = num_kv_heads * prefix[g]
            h = (t - gbase) // nb
            off = t - gbase - h * nb
            cnt = min(nb - off, t_end - t)
            ustart = gbase + h * nb
            whole = off == 0 and cnt == nb
            w0, w1 = split.worker_of_tile(ustart), split.worker_of_tile(ustart + nb - 1)
            out.append(Piece(w, g, h, off, off + cnt, whole, None if whole else piece_slot(w, w0), w0, w1))
            t += cnt
    return out
