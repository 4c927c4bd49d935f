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


def pieces(seq_ids, seq_lens, num_kv_heads: int, workers: int, max_group_rows: int) -> list[Piece]:
    """Every piece every worker processes, in worker order."""
    gs = groups(seq_ids, seq_lens, max_group_rows)
    prefix = [0]
    for _, _, nb in gs:
        prefix.append(prefix[-1] + nb)
    total = num_kv_heads * prefix[-1]
    out = []
    if total == 0:
        return out
    # Only min(workers, total) workers take part, so that every one of them
    # owns at least one tile and a split unit's workers w0..w1 all report.
    workers = min(workers, total)
    for w in range(workers):
        t, t_end = range_begin(w, total, workers), range_begin(w + 1, total, workers)
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
            w0, w1 = worker_of(ustart, total, workers), worker_of(ustart + nb - 1, total, workers)
            out.append(Piece(w, g, h, off, off + cnt, whole, None if whole else piece_slot(w, w0), w0, w1))
            t += cnt
    return out
