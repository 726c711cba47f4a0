"""CPU: the fused all-reduce's flag protocol, driven by host threads.

ocl_q_linear_allreduce (ocelotl_b200/csrc/gemv.cu, tp_epilogue) runs this state
machine per row group g on every rank r, launch after launch:
  1. push the group's partial rows into slot [epoch parity][r] of every rank;
  2. store flag[r][g] = epoch + 1 on every rank;
  3. wait (bounded) until every rank's flag[p][g] here has *reached* epoch + 1;
  4. sum the slots of this parity in rank order; epoch += 1.
Each rank's flag slot is single-buffered, so a peer that is a launch ahead can
overwrite tag e + 1 with e + 2 before a slow rank polls it.  The simulation
makes one rank fast and the others slow and checks that the "reached" test
(tp_flag_reached in ocelotl_b200/csrc/internal.cuh) finishes every launch with
the exact sums, while an equality test -- the protocol as first written --
times out.  The predicate is restated here with the same 32-bit wrap.
"""
import threading
import time

import numpy as np
import pytest


def flag_reached(v: int, tag: int) -> bool:
    """(int32)(v - tag) >= 0 on u32 values."""
    return ((v - tag) & 0xFFFFFFFF) < 0x80000000


def flag_equal(v: int, tag: int) -> bool:
    return v == tag


def _simulate(world, launches, groups, reached, slow_ranks, limit_s=1.0, first_epoch=0):
    data = np.zeros((world, 2, world, groups), dtype=np.int64)  # [owner][parity][src rank][group]
    flags = np.zeros((world, world, groups), dtype=np.uint64)   # [owner][src rank][group]
    flags[:] = first_epoch
    results = np.zeros((world, launches, groups), dtype=np.int64)
    timeouts = [0] * world
    lock = threading.Lock()

    def rank(r):
        rng = np.random.default_rng(r)
        for i in range(launches):
            ep = (first_epoch + i) & 0xFFFFFFFF
            tag, par = (ep + 1) & 0xFFFFFFFF, ep & 1
            for g in range(groups):
                v = (r + 1) * 1000 * (i + 1) + g
                with lock:
                    for p in range(world):
                        data[p, par, r, g] = v
                    for p in range(world):  # release after the data (the lock orders them)
                        flags[p, r, g] = tag
            for g in range(groups):
                if r in slow_ranks:
                    time.sleep(float(rng.uniform(0.0, 0.002)))
                t0 = time.monotonic()
                ok = True
                while True:
                    with lock:
                        if all(reached(int(flags[r, p, g]), tag) for p in range(world)):
                            results[r, i, g] = int(data[r, par, :, g].sum())
                            break
                    if time.monotonic() - t0 > limit_s:
                        ok = False
                        break
                    time.sleep(0)
                if not ok:
                    timeouts[r] += 1
    ts = [threading.Thread(target=rank, args=(r,)) for r in range(world)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    expect = np.array([[sum((p + 1) * 1000 * (i + 1) + g for p in range(world)) for g in range(groups)]
                       for i in range(launches)])
    return results, expect, timeouts


@pytest.mark.parametrize("world", [2, 4])
def test_reached_wait_survives_a_rank_running_ahead(world):
    res, expect, timeouts = _simulate(world, launches=40, groups=4, reached=flag_reached,
                                      slow_ranks=set(range(1, world)))
    assert timeouts == [0] * world
    for r in range(world):
        assert np.array_equal(res[r], expect)


def test_equality_wait_loses_flags_to_a_rank_running_ahead():
    # the single-buffered flag gets overwritten with the next launch's tag
    res, expect, timeouts = _simulate(2, launches=12, groups=4, reached=flag_equal, slow_ranks={1},
                                      limit_s=0.2)
    assert sum(timeouts) > 0


def test_reached_wait_across_tag_wrap():
    res, expect, timeouts = _simulate(2, launches=8, groups=2, reached=flag_reached, slow_ranks={1},
                                      first_epoch=0xFFFFFFFC)
    assert timeouts == [0, 0]
    assert np.array_equal(res[0], expect) and np.array_equal(res[1], expect)


def test_reached_predicate_edges():
    assert flag_reached(5, 5) and flag_reached(6, 5) and not flag_reached(4, 5)
    assert flag_reached(0, 0xFFFFFFFF)          # tag wrapped past the peer's value
    assert not flag_reached(0xFFFFFFFF, 0)      # one launch behind across the wrap
    assert not flag_reached(0, 1)               # never-signalled slot
