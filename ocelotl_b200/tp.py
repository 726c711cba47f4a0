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


class TPLinear:
    """One rank's shard of a quantized linear layer on its own GPU.

    mode "out": y_local [rows, n_local] = x . W_shard^T (no communication).
    mode "in":  y [rows, n] = all_reduce_sum(x[:, k0:k1] . W_shard^T).
    """

    def __init__(self, backend, ggml_type: int, shard_blocks, n_local: int, k_local: int, mode: str,
                 group=None):
        if mode not in ("out", "in"):
            raise ValueError(mode)
        self.backend = backend
        self.mode = mode
        self.group = group
        self.n, self.k = n_local, k_local
        self.weight = backend.upload_quant(ggml_type, shard_blocks, n_local, k_local)

    def forward(self, x_local, rows: int, out) -> None:
        """x_local: this rank's input ([rows, k] for "out", [rows, k_local] for "in"), out [rows, n]."""
        self.backend.linear_dev(self.weight, x_local, rows, out)
        if self.mode == "in":
            import torch.distributed as dist
            if dist.is_initialized() and dist.get_world_size(self.group) > 1:
                dist.all_reduce(out, group=self.group)
