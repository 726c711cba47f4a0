"""Tensor parallelism for the quantized linear path (one process per GPU).

Only the naturally sharded case is supported, as in Megatron-style decoders:
  * column split ("out"): each rank holds a contiguous range of output rows
    (q/k/v, gate, up); no communication, each rank produces its slice of y;
  * row split ("in"): each rank holds a contiguous range of K for every row
    (o, down); each rank produces a partial y over its K range and the partials
    are summed with an all-reduce (NCCL over NVLink on the GPU path).
GGUF blocks never straddle a shard: K splits are whole blocks.

The reference has no multi-device code (its `Device::Gpu{ordinal}`,
crates/core/src/lib.rs:437-441, names one device); this module is new.
"""
from __future__ import annotations

import numpy as np

from .errors import UnsupportedError
from .ggml import geometry


def _range(n: int, rank: int, world: int) -> tuple[int, int]:
    return n * rank // world, n * (rank + 1) // world


def shard_out(blocks, ggml_type: int, n_rows: int, k: int, rank: int, world: int):
    """Rows [r0, r1) of an [n_rows, k] GGUF weight -> (blocks, r0, r1)."""
    g = geometry(ggml_type)
    row_bytes = (k // g.elems) * g.nbytes
    b = np.asarray(blocks, dtype=np.uint8).reshape(n_rows, row_bytes)
    r0, r1 = _range(n_rows, rank, world)
    return np.ascontiguousarray(b[r0:r1]).reshape(-1), r0, r1


def shard_in(blocks, ggml_type: int, n_rows: int, k: int, rank: int, world: int):
    """K columns [k0, k1) of every row (whole blocks) -> (blocks, k0, k1)."""
    g = geometry(ggml_type)
    nkb = k // g.elems
    if nkb % world:
        raise UnsupportedError("row-split in_features", f"{k} over {world} ranks",
                               [f"multiples of {g.elems * world}"])
    b = np.asarray(blocks, dtype=np.uint8).reshape(n_rows, nkb, g.nbytes)
    kb0, kb1 = _range(nkb, rank, world)
    return np.ascontiguousarray(b[:, kb0:kb1]).reshape(-1), kb0 * g.elems, kb1 * g.elems


class TPComm:
    """This rank's peer-memory buffers for the fused all-reduce (one per process and GPU).

    Creates the receive buffer, exchanges CUDA IPC handles over `group` (any
    torch.distributed backend; handles travel as bytes) and maps the peers'
    buffers.  `handles` may be given instead of a group (all ranks' 64-byte
    handles in rank order), e.g. for a loopback test.
    """

    def __init__(self, backend, rank: int, world: int, max_elems: int, max_groups: int = 4096,
                 group=None, handles: list[bytes] | None = None):
        import ctypes as C
        self.backend = backend
        self.rank, self.world = rank, world
        h = C.c_void_p()
        own = (C.c_char * 64)()
        backend._check(backend._lib.ocl_tp_comm_create(backend._ctx, rank, world, max_elems, max_groups,
                                                       C.byref(h), own))
        self.handle = h
        self.own_handle = bytes(own)
        if handles is None:
            import torch.distributed as dist
            gathered = [None] * world
            dist.all_gather_object(gathered, self.own_handle, group=group)
            handles = gathered
        buf = (C.c_char * (64 * world)).from_buffer_copy(b"".join(handles))
        backend._check(backend._lib.ocl_tp_comm_open(backend._ctx, h, buf))

    def close(self):
        if self.handle:
            self.backend._lib.ocl_tp_comm_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class TPLinear:
    """One rank's shard of a quantized linear layer on its own GPU.

    mode "out": y_local [rows, n_local] = x . W_shard^T (no communication).
    mode "in":  y [rows, n] = all_reduce_sum(x[:, k0:k1] . W_shard^T).
    """

    def __init__(self, backend, ggml_type: int, shard_blocks, n_local: int, k_local: int, mode: str,
                 group=None, comm: TPComm | None = None):
        if mode not in ("out", "in"):
            raise ValueError(mode)
        self.backend = backend
        self.mode = mode
        self.group = group
        self.comm = comm  # mode "in": fused peer-memory all-reduce instead of torch.distributed
        self.fused: dict[int, bool] = {}  # rows -> whether the fused path applies
        self.n, self.k = n_local, k_local
        self.weight = backend.upload_quant(ggml_type, shard_blocks, n_local, k_local)

    def forward(self, x_local, rows: int, out) -> None:
        """x_local: this rank's input ([rows, k] for "out", [rows, k_local] for "in"), out [rows, n]."""
        if self.mode == "in" and self.comm is not None and self.fused.get(rows, True):
            try:
                self.backend.linear_allreduce(self.comm, self.weight, x_local, rows, out)
                self.fused[rows] = True
                return
            except UnsupportedError:
                # shapes whose activation planes do not fit one CTA (e.g. K >= 4096
                # at 16 rows): local GEMV + torch.distributed all-reduce instead
                self.fused[rows] = False
        self.backend.linear_dev(self.weight, x_local, rows, out)
        if self.mode == "in":
            import torch.distributed as dist
            if dist.is_initialized() and dist.get_world_size(self.group) > 1:
                dist.all_reduce(out, group=self.group)


def merge_argmax(vals, ids):
    """greedy_sample over a vocab split in rank order, from each shard's own answer.

    vals, ids: [world, rows] -- each rank's local greedy choice (its value and its
    GLOBAL id), ranks in vocab order.  greedy_sample (crates/runtime/src/sampling.rs:29-52)
    scans from index 0 and moves only on a strictly greater value, so: the largest
    value wins, ties go to the lowest id (= the lowest rank, as shards are
    contiguous and in order), -0.0 equals +0.0, a NaN never wins -- except a NaN
    at global index 0, which the scan never leaves (rank 0 reports id 0 with a
    NaN value then, as the device argmax does for a NaN at its index 0).  The
    other shards must report their largest non-NaN value (TPHead maps a NaN at a
    shard's first element to -inf before its local argmax).
    """
    import torch
    nan0 = torch.isnan(vals[0]) & (ids[0] == 0)
    v = torch.where(torch.isnan(vals), torch.full_like(vals, float("-inf")), vals)
    best = torch.argmax(v, dim=0)  # first maximum: the lowest rank
    out = ids.gather(0, best[None]).squeeze(0)
    return torch.where(nan0, torch.zeros_like(out), out)


class TPHead:
    """Output head split by vocabulary rows over the ranks, with a cross-rank greedy pick.

    Each rank holds head rows [v0, v1) (the logits of its vocab shard), runs the
    quantized GEMV and the device argmax on them, and the ranks exchange one
    (value, id) pair per row (all_gather over `group`, NCCL on the GPU path);
    merge_argmax turns those into greedy_sample's answer over the whole vocab.
    The reference's caller: crates/runtime/src/sampling.rs:29.
    """

    def __init__(self, backend, ggml_type: int, shard_blocks, v0: int, v1: int, k: int, rank: int, world: int,
                 group=None):
        self.backend = backend
        self.v0, self.n = v0, v1 - v0
        self.rank, self.world, self.group = rank, world, group
        self.weight = backend.upload_quant(ggml_type, shard_blocks, self.n, k)

    def forward(self, h, rows: int, logits, ids_out) -> None:
        """h [rows, k] f32, logits [rows, n_local] scratch, ids_out [rows] int64: global greedy ids."""
        import torch
        import torch.distributed as dist
        be = self.backend
        be.linear_dev(self.weight, h, rows, logits)
        if self.v0 > 0:
            # greedy_sample's scan never leaves a NaN at ITS index 0; for a shard
            # that starts past global index 0 such a NaN must not hide the
            # shard's maximum, so it is taken as -inf here
            first = logits[:, :1]
            first.copy_(torch.where(torch.isnan(first), torch.full_like(first, float("-inf")), first))
        local = be.greedy_sample(logits).long()
        vals = logits.gather(1, local[:, None]).squeeze(1)
        gids = local + self.v0
        if self.world == 1:
            ids_out.copy_(gids)
            return
        gv = torch.empty(self.world, rows, dtype=vals.dtype, device=vals.device)
        gi = torch.empty(self.world, rows, dtype=gids.dtype, device=gids.device)
        dist.all_gather_into_tensor(gv, vals, group=self.group)
        dist.all_gather_into_tensor(gi, gids, group=self.group)
        ids_out.copy_(merge_argmax(gv, gi))
