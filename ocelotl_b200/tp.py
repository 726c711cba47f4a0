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
