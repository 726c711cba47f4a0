"""CPU: tensor-parallel sharding logic with world_size 2 over gloo.

Each rank shards the GGUF blocks with ocelotl_b200.tp, computes its partial
result with the CPU oracle (standing in for the GPU kernel), and the row-split
partials are summed with a gloo all-reduce; the result must match the
unsharded oracle (to f32 reordering: the all-reduce changes the summation
order, so no bit equality is asserted).
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tests.tolerance import GEMV_RTOL, rel_err


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, t, n, k, rows, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import oracle
    from ocelotl_b200 import synth, tp
    blocks = synth.quant_blocks(t, n, k, 5, "tpw").numpy()
    x = synth.activations(rows, k, 5, "tpx").numpy()
    # column split
    bo, r0, r1 = tp.shard_out(blocks, t, n, k, rank, world)
    y_col = oracle.q_linear(t, bo, x, rows, k, r1 - r0)
    parts = [torch.zeros(rows, n * (i + 1) // world - n * i // world) for i in range(world)]
    dist.all_gather(parts, torch.from_numpy(y_col))
    y_col_full = torch.cat(parts, dim=1).numpy()
    # row split
    bi, k0, k1 = tp.shard_in(blocks, t, n, k, rank, world)
    y_row = torch.from_numpy(oracle.q_linear(t, bi, np.ascontiguousarray(x[:, k0:k1]), rows, k1 - k0, n))
    dist.all_reduce(y_row)
    if rank == 0:
        ref = oracle.q_linear(t, blocks, x, rows, k, n)
        q.put((rel_err(y_col_full, ref), rel_err(y_row.numpy(), ref), np.array_equal(y_col_full, ref)))
    dist.destroy_process_group()


@pytest.mark.parametrize("t,n,k", [(12, 96, 1024), (14, 64, 2048), (8, 80, 512)])
def test_tp2_column_and_row_split_match_unsharded(oracle, t, n, k):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, t, n, k, 3, q))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    col_err, row_err, col_exact = q.get(timeout=10)
    assert col_exact  # column split keeps every output's accumulation order
    assert row_err <= GEMV_RTOL and col_err == 0.0


def test_row_split_rejects_ragged_blocks():
    from ocelotl_b200 import UnsupportedError, tp
    with pytest.raises(UnsupportedError):
        tp.shard_in(np.zeros(2 * 3 * 144, np.uint8), 12, 2, 768, 0, 2)


def _head_worker(rank, world, port, logits, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import oracle
    from ocelotl_b200.tp import _range, merge_argmax
    rows, vocab = logits.shape
    v0, v1 = _range(vocab, rank, world)
    shard = logits[:, v0:v1].copy()
    if v0 > 0:  # as TPHead: a NaN at a later shard's first element must not hide its maximum
        shard[:, 0] = np.where(np.isnan(shard[:, 0]), -np.inf, shard[:, 0])
    # each rank's local greedy answer on its shard (the oracle stands in for the device argmax)
    local = np.array([oracle.greedy_sample(shard[r]) for r in range(rows)])
    vals = torch.from_numpy(logits[np.arange(rows), v0 + local].astype(np.float32))
    vals = torch.where(torch.isnan(vals) & torch.tensor(v0 > 0), torch.tensor(float("-inf")), vals)
    gids = torch.from_numpy(local + v0)
    gv = [torch.empty_like(vals) for _ in range(world)]
    gi = [torch.empty_like(gids) for _ in range(world)]
    dist.all_gather(gv, vals)
    dist.all_gather(gi, gids)
    got = merge_argmax(torch.stack(gv), torch.stack(gi)).numpy()
    if rank == 0:
        q.put(got.tolist())
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_vocab_split_greedy_matches_full_scan(world):
    """Head split by vocab over ranks: the merged pick equals greedy_sample over all logits
    (ties across shards, -0.0 / +0.0, NaN at index 0, NaN elsewhere and at a shard's
    first element next to the maximum, all -inf)."""
    import oracle
    rng = np.random.default_rng(3)
    vocab = 1000
    rows = [rng.standard_normal(vocab).astype(np.float32) for _ in range(6)]
    tie = np.full(vocab, -1.0, np.float32)
    tie[[130, 700, 999]] = 5.0           # equal maxima in different shards -> lowest id
    rows.append(tie)
    z = np.full(vocab, -1.0, np.float32)
    z[600], z[10] = 0.0, -0.0            # -0.0 at a lower id ties with +0.0
    rows.append(z)
    n0 = rng.standard_normal(vocab).astype(np.float32)
    n0[0] = np.nan                        # NaN at index 0: the scan stays at 0
    rows.append(n0)
    nm = rng.standard_normal(vocab).astype(np.float32)
    nm[[5, 250, 501, 502, 998]] = np.nan  # NaNs elsewhere never win
    rows.append(nm)
    for start in (250, 500):             # a later shard starts with NaN and holds the maximum next to it
        sh = rng.standard_normal(vocab).astype(np.float32)
        sh[start], sh[start + 1] = np.nan, 50.0
        rows.append(sh)
    rows.append(np.full(vocab, -np.inf, np.float32))
    logits = np.stack(rows)
    expect = [oracle.greedy_sample(r) for r in logits]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_head_worker, args=(r, world, port, logits, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    assert q.get(timeout=10) == expect
