"""The fused reduce-scatter's cross-rank protocol, modelled on the CPU with one
thread per rank (the device code is csrc/gemm_i8.cu: the scatter epilogue,
publish_counts and reduce_phase; the host side is peer_reduce._PeerBuffers).

Per call a rank uses buffer set ``calls & 1`` and bumps that set's use count;
it stores its partial rows for owner j into owner j's slot (set, source =
this rank), then adds the element count to owner j's counter (set, source);
the counters only grow.  The owner then waits, bounded, until every source's
counter of the set reaches ``uses x rows_per_owner x N`` and sums its slots in
rank order.  A rank runs its calls in order (one launch after the other on its
stream), so a rank can be at most one call ahead of any other: the model
checks that two sets are enough for no slot to be overwritten before its
owner has read it, under random delays, and that a source that never reports
makes the owner's wait run out (rows poisoned, status set) instead of hang.
"""
from __future__ import annotations

import random
import threading
import time

import numpy as np


class _Rank:
    def __init__(self, rank: int, world: int, rows: int, cols: int):
        self.rank, self.world = rank, world
        # [set][source] slots of this rank's rows, and [set][source] counters
        self.slots = np.zeros((2, world, rows, cols), dtype=np.float64)
        self.counters = np.zeros((2, world), dtype=np.int64)
        self.lock = threading.Lock()
        self.calls = 0
        self.uses = [0, 0]
        self.status = 0


def _partial(call: int, src: int, owner: int, rows: int, cols: int) -> np.ndarray:
    return np.full((rows, cols), 1000.0 * call + 10.0 * src + owner)


def _run(world: int, calls: int, rows: int, cols: int, seed: int, silent: int | None = None,
         wait_limit_s: float = 2.0):
    ranks = [_Rank(r, world, rows, cols) for r in range(world)]
    results: dict[tuple[int, int], np.ndarray] = {}
    errors: list[str] = []

    def worker(me: _Rank):
        rng = random.Random(seed * 97 + me.rank)
        for _ in range(calls):
            me.calls += 1
            h = me.calls & 1
            me.uses[h] += 1
            call = me.calls
            if me.rank != silent:
                # scatter epilogue: the partial rows of every owner go to its slot
                for d in range(world):
                    j = (me.rank + 1 + d) % world
                    owner = ranks[j]
                    time.sleep(rng.random() * 2e-4)
                    data = _partial(call, me.rank, j, rows, cols)
                    owner.slots[h, me.rank] = data            # plain stores
                    with owner.lock:                          # fence + red.release.sys
                        owner.counters[h, me.rank] += rows * cols
            # owner side: bounded wait for every source, then the rank-order sum
            target = me.uses[h] * rows * cols
            t0 = time.monotonic()
            while True:
                with me.lock:
                    ready = bool((me.counters[h] >= target).all())
                if ready or time.monotonic() - t0 > wait_limit_s:
                    break
                time.sleep(1e-5)
            if not ready:
                me.status = 1
                results[(me.rank, call)] = np.full((rows, cols), np.nan)
                continue
            time.sleep(rng.random() * 2e-4)
            acc = np.zeros((rows, cols))
            for src in range(world):
                acc += me.slots[h, src]
            results[(me.rank, call)] = acc

    threads = [threading.Thread(target=worker, args=(r,)) for r in ranks]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=60)
        if t.is_alive():
            errors.append("a rank did not finish")
    return ranks, results, errors


def test_two_buffer_sets_never_expose_a_later_calls_partial():
    world, calls, rows, cols = 4, 8, 3, 2
    for seed in range(6):
        ranks, results, errors = _run(world, calls, rows, cols, seed)
        assert not errors
        for r in range(world):
            assert ranks[r].status == 0
            for call in range(1, calls + 1):
                want = sum(_partial(call, src, r, rows, cols) for src in range(world))
                np.testing.assert_array_equal(results[(r, call)], want)


def test_a_source_that_never_reports_makes_the_wait_run_out():
    world, rows, cols = 3, 2, 2
    ranks, results, errors = _run(world, 1, rows, cols, seed=1, silent=2, wait_limit_s=0.2)
    assert not errors
    for r in range(world):
        assert ranks[r].status == 1
        assert np.isnan(results[(r, 1)]).all()


def test_all_reduce_output_stays_valid_until_the_second_call_after():
    """The all-reduce adds a gather: each owner stores its reduced rows into
    every rank's output of the call's set and bumps that rank's gather counter
    (set, owner); a rank returns once every owner's rows are there.  The
    output of call c must stay intact until this rank makes call c + 2 (the
    host API's contract): another rank can only write this set again for call
    c + 2, which needs this rank's own partials of call c + 2."""
    world, calls, rows, cols = 4, 8, 2, 2
    for seed in range(6):
        outs = [np.zeros((2, world * rows, cols)) for _ in range(world)]
        gather = [np.zeros((2, world), dtype=np.int64) for _ in range(world)]
        slots = [np.zeros((2, world, rows, cols)) for _ in range(world)]
        counts = [np.zeros((2, world), dtype=np.int64) for _ in range(world)]
        locks = [threading.Lock() for _ in range(world)]
        bad: list[str] = []

        def wait(lock, arr, h, target):
            t0 = time.monotonic()
            while time.monotonic() - t0 < 5.0:
                with lock:
                    if bool((arr[h] >= target).all()):
                        return True
                time.sleep(1e-5)
            return False

        def worker(me: int):
            rng = random.Random(seed * 31 + me)
            uses = [0, 0]
            kept: dict[int, np.ndarray] = {}
            for call in range(1, calls + 1):
                h = call & 1
                if call - 2 in kept and not np.array_equal(outs[me][h], kept[call - 2]):
                    bad.append(f"rank {me}: output of call {call - 2} changed before call {call}")
                uses[h] += 1
                for d in range(world):
                    j = (me + 1 + d) % world
                    time.sleep(rng.random() * 2e-4)
                    slots[j][h, me] = _partial(call, me, j, rows, cols)
                    with locks[j]:
                        counts[j][h, me] += rows * cols
                if not wait(locks[me], counts[me], h, uses[h] * rows * cols):
                    bad.append(f"rank {me}: partial wait ran out")
                    return
                reduced = slots[me][h].sum(axis=0)
                for d in range(world):
                    j = (me + 1 + d) % world
                    time.sleep(rng.random() * 2e-4)
                    outs[j][h, me * rows:(me + 1) * rows] = reduced
                    with locks[j]:
                        gather[j][h, me] += rows * cols
                if not wait(locks[me], gather[me], h, uses[h] * rows * cols):
                    bad.append(f"rank {me}: gather wait ran out")
                    return
                want = np.concatenate([sum(_partial(call, s, o, rows, cols) for s in range(world))
                                       for o in range(world)])
                if not np.array_equal(outs[me][h], want):
                    bad.append(f"rank {me}: call {call} output wrong")
                kept[call] = outs[me][h].copy()
                time.sleep(rng.random() * 4e-4)  # the caller still reads the output

        threads = [threading.Thread(target=worker, args=(r,)) for r in range(world)]
        for t in threads:
            t.start()
        for t in threads:
            t.join(timeout=60)
        assert not any(t.is_alive() for t in threads)
        assert not bad, bad
