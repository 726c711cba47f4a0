"""CPU: the fused all-reduce's packet protocol, driven by host threads.

ocl_q_linear_allreduce (ocelotl_b200/csrc/gemv.cu, tp_epilogue) runs this per
output element on every rank r, launch after launch (epoch e, tag e + 1,
parity e % 2):
  1. store packet (value, tag) into slot [parity][r][elem] of every rank;
  2. poll this rank's own slots [parity][*][elem] until every tag has *reached*
     tag (tp_flag_reached in ocelotl_b200/csrc/internal.cuh, restated here with
     the same 32-bit wrap), then sum the values in rank order; epoch += 1.
A value and its tag are one 8-byte store, so they are observed together (the
lock below stands in for that atomicity).  The simulation makes one rank fast
and the others slow, so the fast rank keeps storing the next launch's packets
into the other parity while the slow ones still read: every launch must finish
with the exact sums, with no timeout, also across the tag wrap.  A variant that
drops the parity double buffer shows why it is needed: the fast rank then
overwrites packets a slow rank has not read yet.
"""
import threading
import time

import numpy as np
import pytest


def flag_reached(v: int, tag: int) -> bool:
    """(int32)(v - tag) >= 0 on u32 values."""
    return ((v - tag) & 0xFFFFFFFF) < 0x80000000


def _simulate(world, launches, n_elem, slow_ranks, parities=2, limit_s=1.0, first_epoch=0):
    val = np.zeros((world, parities, world, n_elem), dtype=np.int64)   # [owner][parity][src][elem]
    tags = np.full((world, parities, world, n_elem), first_epoch, dtype=np.uint64)
    results = np.zeros((world, launches, n_elem), dtype=np.int64)
    bad = [0] * world
    lock = threading.Lock()

    def rank(r):
        rng = np.random.default_rng(r)
        for i in range(launches):
            ep = (first_epoch + i) & 0xFFFFFFFF
            tag, par = (ep + 1) & 0xFFFFFFFF, ep % parities
            for e in range(n_elem):
                v = (r + 1) * 1000 * (i + 1) + e
                for p in range(world):
                    with lock:  # one 8-byte store: value and tag together
                        val[p, par, r, e] = v
                        tags[p, par, r, e] = tag
            if r in slow_ranks:
                time.sleep(float(rng.uniform(0.0, 0.003)))
            t0 = time.monotonic()
            for e in range(n_elem):
                acc = 0
                for s in range(world):
                    while True:
                        with lock:
                            if flag_reached(int(tags[r, par, s, e]), tag):
                                acc += int(val[r, par, s, e])
                                break
                        if time.monotonic() - t0 > limit_s:
                            bad[r] += 1
                            break
                        time.sleep(0)
                results[r, i, e] = acc
    ts = [threading.Thread(target=rank, args=(r,)) for r in range(world)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    expect = np.array([[sum((p + 1) * 1000 * (i + 1) + e for p in range(world)) for e in range(n_elem)]
                       for i in range(launches)])
    return results, expect, bad


@pytest.mark.parametrize("world", [2, 4])
def test_packets_survive_a_rank_running_ahead(world):
    res, expect, bad = _simulate(world, launches=40, n_elem=6, slow_ranks=set(range(1, world)))
    assert bad == [0] * world
    for r in range(world):
        assert np.array_equal(res[r], expect)


def test_packets_across_tag_wrap():
    res, expect, bad = _simulate(2, launches=8, n_elem=4, slow_ranks={1}, first_epoch=0xFFFFFFFC)
    assert bad == [0, 0]
    assert np.array_equal(res[0], expect) and np.array_equal(res[1], expect)


def test_single_buffer_lets_a_fast_rank_overwrite_unread_packets():
    # without the parity double buffer a reader can see the NEXT launch's value
    # (its tag has "reached" too), so the sums go wrong
    res, expect, bad = _simulate(2, launches=40, n_elem=6, slow_ranks={1}, parities=1)
    assert not all(np.array_equal(res[r], expect) for r in range(2))


def test_reached_predicate_edges():
    assert flag_reached(5, 5) and flag_reached(6, 5) and not flag_reached(4, 5)
    assert flag_reached(0, 0xFFFFFFFF)          # tag wrapped past the peer's value
    assert not flag_reached(0xFFFFFFFF, 0)      # one launch behind across the wrap
    assert not flag_reached(0, 1)               # a slot never written
