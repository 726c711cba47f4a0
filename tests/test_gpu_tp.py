"""GPU: the GEMV with the tensor-parallel all-reduce fused in (peer memory).

Protocol (ocelotl_b200/csrc/gemv.cu, tp_epilogue): launch e sends every output
value to every rank as one 8-byte packet (value, tag e + 1) and waits until
every rank's packet for its outputs has reached tag e + 1.

* loopback (1 GPU): a communicator whose second rank is mapped back onto the
  first.  With rank 1's packets never sent, the bounded wait must run out,
  report a timeout (counter and OCL_ERR_TIMEOUT), write nothing and leave the
  context usable.  With rank 1's slots already holding tags past the next
  launches' (a peer running ahead), no launch may time out, and y must equal the
  plain GEMV's result bit for bit (rank 1's slot holds zeros).
* 2 and 4 GPUs (each skipped below its GPU count): row-split shards on one
  process per GPU; 120 back-to-back launches alternating the o and down shapes
  of the 8B layer with no host synchronisation in between; every launch's
  output must be identical on all ranks and equal to the first launch of its
  kind, the final outputs must match the unsharded oracle, and no wait may
  time out; the vocab-split Q6_K head (TPHead) must pick greedy_sample's id
  over the gathered logits, which must match the oracle.
"""
import ctypes as C
import hashlib
import os
import socket

import numpy as np
import pytest
import torch

from tests.tolerance import GEMV_RTOL, record_err, rel_err

pytestmark = pytest.mark.gpu


def _loopback(backend, n):
    from ocelotl_b200 import tp
    c = tp.TPComm.__new__(tp.TPComm)
    h = C.c_void_p()
    own = (C.c_char * 64)()
    backend._check(backend._lib.ocl_tp_comm_create(backend._ctx, 0, 2, 16 * n, 4096, C.byref(h), own))
    buf = (C.c_char * 128).from_buffer_copy(bytes(own) * 2)
    backend._check(backend._lib.ocl_tp_comm_open(backend._ctx, h, buf))
    c.backend, c.handle, c.rank, c.world = backend, h, 0, 2
    return c


def test_fused_allreduce_bounded_wait_times_out(backend, oracle):
    from ocelotl_b200 import synth
    from ocelotl_b200 import _lib
    n, k = 256, 1024
    blocks = synth.quant_blocks(12, n, k, 4, "lb")
    w = backend.upload_quant(12, blocks, n, k)
    c = _loopback(backend, n)  # rank 1 never signals
    x = synth.activations(1, k, 4, "lbx", device="cuda")
    y = torch.full((1, n), float("nan"), device="cuda")
    backend.take_device_errors()
    backend.linear_allreduce(c, w, x, 1, y)
    torch.cuda.synchronize()
    bad, timeouts = backend.take_device_errors()
    assert timeouts > 0 and bad == 0
    assert torch.isnan(y).all()  # nothing written on timeout
    # the status-only check reports it too
    backend.linear_allreduce(c, w, x, 1, y)
    torch.cuda.synchronize()
    rc = backend._lib.ocl_take_device_errors(backend._ctx, None, None)
    assert rc == _lib.OCL_ERR_TIMEOUT
    assert "gave up" in backend._lib.ocl_last_error(backend._ctx).decode()
    c.close()
    # the context still works
    out = backend.alloc(n)
    backend.linear_d(backend.upload(x.cpu().numpy()), 1, k, w, n, None, out)
    ref = oracle.q_linear(12, blocks.numpy(), x.cpu().numpy(), 1, k, n)
    assert rel_err(out.to_host_owned().reshape(1, n), ref) <= GEMV_RTOL


def test_fused_allreduce_peer_already_ahead(backend):
    """Rank 1's packets already carry tag 6: launches with tags 1..6 must pass."""
    from ocelotl_b200 import synth
    for t, n, k in ((12, 4096, 4096), (14, 4096, 14336)):
        w = backend.upload_quant(t, synth.quant_blocks(t, n, k, 5, f"ahead{t}", device="cuda"), n, k)
        c = _loopback(backend, n)
        # rank 1's slots of both parities already hold (0.0, tag 6): the peer is up
        # to five launches ahead of launch 1
        torch.cuda.synchronize()
        cudart = C.CDLL("libcudart.so.12")  # already loaded by the library
        cudart.cudaMemcpy.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_int]
        pk = backend._lib.ocl_tp_comm_packets(c.handle)
        assert pk
        max_elems = 16 * n
        pkt = torch.full((max_elems,), 6 << 32, dtype=torch.int64, device="cuda")
        for par in (0, 1):
            dst = pk + ((par * 2 + 1) * max_elems) * 8
            assert cudart.cudaMemcpy(dst, pkt.data_ptr(), max_elems * 8, 3) == 0  # D2D
        x = synth.activations(1, k, 5, "aheadx", device="cuda")
        ref = torch.empty(1, n, device="cuda")
        backend.linear_dev(w, x, 1, ref)
        backend.take_device_errors()
        for _ in range(6):
            y = torch.full((1, n), float("nan"), device="cuda")
            backend.linear_allreduce(c, w, x, 1, y)
            torch.cuda.synchronize()
            assert backend.take_device_errors() == (0, 0)
            assert torch.equal(y, ref)  # own slot + rank 1's zero slot, same bits as the plain GEMV
        c.close()


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.cuda.set_device(rank)
    import oracle
    from ocelotl_b200 import synth, tp
    from ocelotl_b200.backend import CudaKernelBackend
    be = CudaKernelBackend(rank)
    comm = tp.TPComm(be, rank, world, max_elems=16 * 4096)
    results = {}
    # 1) alternating o / down shapes of the 8B layer, 120 launches, no host sync
    shapes = {"o": (12, 4096, 4096), "down": (14, 4096, 14336)}
    lins, xs, full = {}, {}, {}
    for nm, (t, n, k) in shapes.items():
        blocks = synth.quant_blocks(t, n, k, 9, f"tp.{nm}").numpy()
        x = synth.activations(1, k, 9, f"tpx.{nm}").numpy()
        shard, k0, k1 = tp.shard_in(blocks, t, n, k, rank, world)
        lins[nm] = tp.TPLinear(be, t, shard, n, k1 - k0, "in", comm=comm)
        xs[nm] = torch.from_numpy(np.ascontiguousarray(x[:, k0:k1])).cuda()
        full[nm] = (blocks, x)
    n_launch = 120
    outs = [torch.full((1, 4096), float("nan"), device="cuda") for _ in range(n_launch)]
    for i in range(n_launch):
        nm = "o" if i % 2 == 0 else "down"
        be.linear_allreduce(comm, lins[nm].weight, xs[nm], 1, outs[i])
    torch.cuda.synchronize()
    host = [o.cpu().numpy() for o in outs]
    errs = be.take_device_errors()
    first = {"o": host[0], "down": host[1]}
    stable = all(np.array_equal(host[i], first["o" if i % 2 == 0 else "down"]) for i in range(n_launch))
    digest = hashlib.sha256(b"".join(h.tobytes() for h in host)).hexdigest()
    gathered = [None] * world
    dist.all_gather_object(gathered, digest)
    results["alternating"] = {"same": all(g == gathered[0] for g in gathered), "stable": stable, "errs": errs}
    if rank == 0:
        for nm, (t, n, k) in shapes.items():
            blocks, x = full[nm]
            ref = oracle.q_linear(t, blocks, x, 1, k, n, threads=8)
            results[f"err_{nm}"] = rel_err(first[nm], ref)
    dist.barrier()
    # 2) several rows (rows > 1 layouts) and repeated calls
    t, n, k, rows = 12, 512, 2048, 5
    blocks = synth.quant_blocks(t, n, k, 9, "tp5").numpy()
    x = synth.activations(rows, k, 9, "tpx5").numpy()
    shard, k0, k1 = tp.shard_in(blocks, t, n, k, rank, world)
    lin = tp.TPLinear(be, t, shard, n, k1 - k0, "in", comm=comm)
    xd = torch.from_numpy(np.ascontiguousarray(x[:, k0:k1])).cuda()
    y = torch.empty(rows, n, device="cuda")
    for _ in range(3):
        lin.forward(xd, rows, y)
    torch.cuda.synchronize()
    yh = y.cpu().numpy()
    gathered = [None] * world
    dist.all_gather_object(gathered, yh.tobytes())
    results["rows5"] = {"same": all(g == gathered[0] for g in gathered), "errs": be.take_device_errors()}
    if rank == 0:
        results["err_rows5"] = rel_err(yh, oracle.q_linear(t, blocks, x, rows, k, n, threads=8))
    # 3) vocab-split head with the cross-rank greedy pick (TPHead): the merged ids
    # must be greedy_sample over the gathered logits, which must match the oracle
    vocab, hk, hrows = 5000, 512, 3
    hblocks = synth.quant_blocks(14, vocab, hk, 9, "tphead").numpy()
    h = synth.activations(hrows, hk, 9, "tpheadx").numpy()
    v0, v1 = tp._range(vocab, rank, world)
    row_bytes = (hk // 256) * 210
    head = tp.TPHead(be, 14, np.ascontiguousarray(hblocks.reshape(vocab, row_bytes)[v0:v1]).reshape(-1), v0, v1, hk,
                     rank, world, group=dist.new_group(backend="nccl"))
    logits = torch.empty(hrows, v1 - v0, device="cuda")
    ids = torch.empty(hrows, dtype=torch.int64, device="cuda")
    head.forward(torch.from_numpy(h).cuda(), hrows, logits, ids)
    torch.cuda.synchronize()
    shards = [None] * world
    dist.all_gather_object(shards, logits.cpu().numpy())
    if rank == 0:
        full = np.concatenate(shards, axis=1)
        results["err_head"] = rel_err(full, oracle.q_linear(14, hblocks, h, hrows, hk, vocab, threads=8))
        results["head_ids_ok"] = ids.cpu().tolist() == [oracle.greedy_sample(r) for r in full]
        q.put(results)
    comm.close()
    dist.barrier()
    dist.destroy_process_group()


def _run_world(world):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(600)
        assert p.exitcode == 0
    res = q.get(timeout=10)
    alt = res["alternating"]
    assert alt["errs"] == (0, 0) and alt["same"] and alt["stable"]
    assert res["rows5"]["same"] and res["rows5"]["errs"] == (0, 0)
    assert res["head_ids_ok"]
    for key in ("err_o", "err_down", "err_rows5", "err_head"):
        record_err(f"tp{world}.{key}", res[key])
        assert res[key] <= GEMV_RTOL, (key, res[key])


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_fused_allreduce_two_gpus():
    _run_world(2)


@pytest.mark.skipif(torch.cuda.device_count() < 4, reason="needs four GPUs")
def test_fused_allreduce_four_gpus():
    _run_world(4)
