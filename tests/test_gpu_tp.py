"""GPU: the GEMV with the tensor-parallel all-reduce fused in (peer memory).

* loopback (1 GPU): a communicator whose second rank is mapped back onto the
  first never receives that rank's flags, so the bounded wait must run out,
  report a timeout through ocl_take_device_errors, and leave the context usable;
* two GPUs (skipped with fewer): row-split shards on two processes must give
  the unsharded oracle's result, with identical bits on both ranks.
"""
import os
import socket

import numpy as np
import pytest
import torch

from tests.tolerance import GEMV_RTOL, rel_err

pytestmark = pytest.mark.gpu


def test_fused_allreduce_bounded_wait_times_out(backend, oracle):
    from ocelotl_b200 import synth, tp
    n, k = 256, 1024
    blocks = synth.quant_blocks(12, n, k, 4, "lb")
    w = backend.upload_quant(12, blocks, n, k)
    # loopback: rank 1's slot is this process's own buffer, so rank 1 never signals
    c = tp.TPComm.__new__(tp.TPComm)
    import ctypes as C
    h = C.c_void_p()
    own = (C.c_char * 64)()
    backend._check(backend._lib.ocl_tp_comm_create(backend._ctx, 0, 2, 16 * n, 4096, C.byref(h), own))
    buf = (C.c_char * 128).from_buffer_copy(bytes(own) * 2)
    backend._check(backend._lib.ocl_tp_comm_open(backend._ctx, h, buf))
    c.backend, c.handle, c.rank, c.world = backend, h, 0, 2
    x = synth.activations(1, k, 4, "lbx", device="cuda")
    y = torch.full((1, n), float("nan"), device="cuda")
    backend.take_device_errors()
    backend.linear_allreduce(c, w, x, 1, y)
    torch.cuda.synchronize()
    bad, timeouts = backend.take_device_errors()
    assert timeouts > 0 and bad == 0
    assert torch.isnan(y).all()  # nothing written on timeout
    c.close()
    # the context still works
    out = backend.alloc(n)
    backend.linear_d(backend.upload(x.cpu().numpy()), 1, k, w, n, None, out)
    ref = oracle.q_linear(12, blocks.numpy(), x.cpu().numpy(), 1, k, n)
    assert rel_err(out.to_host_owned().reshape(1, n), ref) <= GEMV_RTOL


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
    results = []
    for t, n, k, rows in ((12, 4096, 4096, 1), (14, 4096, 14336, 1), (12, 512, 2048, 5)):
        blocks = synth.quant_blocks(t, n, k, 9, f"tp{t}").numpy()
        x = synth.activations(rows, k, 9, "tpx").numpy()
        comm = tp.TPComm(be, rank, world, max_elems=16 * n)
        shard, k0, k1 = tp.shard_in(blocks, t, n, k, rank, world)
        lin = tp.TPLinear(be, t, shard, n, k1 - k0, "in", comm=comm)
        xd = torch.from_numpy(np.ascontiguousarray(x[:, k0:k1])).cuda()
        y = torch.empty(rows, n, device="cuda")
        for _ in range(3):  # repeated calls exercise the epoch / parity handling
            lin.forward(xd, rows, y)
        torch.cuda.synchronize()
        yh = y.cpu().numpy()
        errs = be.take_device_errors()
        gathered = [None] * world
        dist.all_gather_object(gathered, yh.tobytes())
        same = all(g == gathered[0] for g in gathered)
        ref = oracle.q_linear(t, blocks, x, rows, k, n, threads=4) if rank == 0 else None
        results.append((rel_err(yh, ref) if rank == 0 else 0.0, same, errs))
        comm.close()
        dist.barrier()
    if rank == 0:
        q.put(results)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_fused_allreduce_two_gpus(oracle):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
        assert p.exitcode == 0
    for err, same, errs in q.get(timeout=10):
        assert same and errs == (0, 0)
        assert err <= GEMV_RTOL
