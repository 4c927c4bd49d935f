"""CPU: the attention kernels' work-partition arithmetic (mirror of csrc/plan.cuh)."""
import itertools
import random

import pytest

from nebulasd_b200 import schedule as S


def test_worker_of_inverts_range_begin():
    for total in range(1, 60):
        for workers in range(1, 40):
            for t in range(total):
                w = S.worker_of(t, total, workers)
                assert S.range_begin(w, total, workers) <= t < S.range_begin(w + 1, total, workers)


def test_groups_follow_seq_runs_and_cap():
    ids = [3, 3, 3, 3, 3, 7, 7, 3, 3]
    lens = [10, 11, 12, 13, 14, 1, 2, 40, 41]
    assert S.groups(ids, lens, 2) == [(0, 2, 1), (2, 2, 1), (4, 1, 1), (5, 2, 1), (7, 2, 3)]
    assert S.groups(ids, lens, 16) == [(0, 5, 1), (5, 2, 1), (7, 2, 3)]
    assert S.groups([1, 1], [0, 0], 4) == [(0, 2, 0)]


def _check_partition(ids, lens, hk, workers, mg, pc=0):
    ps = S.pieces(ids, lens, hk, workers, mg, pc)
    gs = S.groups(ids, lens, mg)
    covered = {}
    slots = set()
    per_unit = {}
    for p in ps:
        for t in range(p.tile_lo, p.tile_hi):
            key = (p.group, p.kv_head, t)
            assert key not in covered
            covered[key] = p.worker
        if not p.whole:
            assert p.slot not in slots
            assert 0 <= p.slot < 2 * workers
            slots.add(p.slot)
            per_unit.setdefault((p.group, p.kv_head), []).append(p)
    expect = {(g, h, t) for g, (_, _, nb) in enumerate(gs) for h in range(hk) for t in range(nb)}
    assert set(covered) == expect
    for unit, pieces in per_unit.items():
        w0, w1 = pieces[0].w0, pieces[0].w1
        assert [p.worker for p in pieces] == list(range(w0, w1 + 1))
        assert sorted(p.slot for p in pieces) == sorted(S.piece_slot(w, w0) for w in range(w0, w1 + 1))
    load = {}
    starts = {}
    for p in ps:
        load[p.worker] = load.get(p.worker, 0) + p.tile_hi - p.tile_lo
        starts[p.worker] = starts.get(p.worker, 0) + (p.tile_lo == 0)
    total = sum(load.values())
    if pc == 0:
        # balance: every worker gets floor or ceil of T/W tiles
        workers = min(workers, total) if total else workers
        for w in range(workers):
            assert load.get(w, 0) in (total // workers, -(-total // workers))
    elif all(nb > 0 for _, _, nb in gs):
        # balance of tiles + pc per unit started, within one piece's cost
        # (an empty unit carries cost but no piece, so batches with one are skipped)
        vtotal = total + pc * hk * len(gs)
        workers = min(workers, vtotal)
        for w in range(workers):
            cost = load.get(w, 0) + pc * starts.get(w, 0)
            assert abs(cost - vtotal / workers) <= pc + 1


@pytest.mark.parametrize("seed", range(40))
def test_partition_covers_every_tile_once_with_unique_slots(seed):
    rng = random.Random(seed)
    nreq = rng.randint(1, 12)
    ids, lens = [], []
    for r in range(nreq):
        depth = rng.randint(0, 9)
        base = rng.choice([0, 1, 15, 16, 17, rng.randint(1, 700)])
        sid = rng.randint(0, 5) if rng.random() < 0.3 else r
        for j in range(depth + 1):
            ids.append(sid)
            lens.append(base + j)
    hk = rng.choice([1, 2, 8])
    workers = rng.choice([1, 2, 3, 7, 148, 600])
    mg = rng.choice([1, 4, 16])
    _check_partition(ids, lens, hk, workers, mg)


def test_partition_exhaustive_small():
    for lens in itertools.product([0, 1, 16, 17, 40], repeat=3):
        for workers in (1, 2, 5, 9):
            _check_partition([0, 1, 2], list(lens), 2, workers, 1)
            _check_partition([0, 0, 0], list(lens), 2, workers, 2)


@pytest.mark.parametrize("seed", range(40))
@pytest.mark.parametrize("pc", [1, 5, 12])
def test_cost_split_partition(seed, pc):
    rng = random.Random(1000 + seed)
    nreq = rng.randint(1, 12)
    ids, lens = [], []
    for r in range(nreq):
        depth = rng.randint(0, 9)
        base = rng.choice([0, 1, 15, 16, 17, rng.randint(1, 700)])
        sid = rng.randint(0, 5) if rng.random() < 0.3 else r
        for j in range(depth + 1):
            ids.append(sid)
            lens.append(base + j)
    _check_partition(ids, lens, rng.choice([1, 2, 8]), rng.choice([1, 2, 3, 7, 148, 600]), rng.choice([1, 4, 16]), pc)


def test_cost_split_inverse_and_zero_cost_identity():
    prefix = [0, 3, 3, 10, 11]   # one empty group
    for hk in (1, 2, 8):
        for pc in (0, 1, 7):
            for workers in (1, 3, 10, 50):
                sp = S.CostSplit(prefix, hk, pc, workers)
                bounds = [sp.begin(w) for w in range(sp.workers + 1)]
                assert bounds[0] == 0 and bounds[-1] == sp.total and bounds == sorted(bounds)
                for t in range(sp.total):
                    w = sp.worker_of_tile(t)
                    assert bounds[w] <= t < bounds[w + 1]
                if pc == 0:
                    assert bounds == [S.range_begin(w, sp.total, sp.workers) for w in range(sp.workers + 1)]
