"""Hand-built Q8_0 weights for the gated-MLP cases (shared by CPU and GPU tests)."""
import struct

import numpy as np


def q8_0_unit_rows(n_rows: int, k: int, col_of_row) -> np.ndarray:
    """Q8_0 blocks of an [n_rows, k] weight that is 1.0 at (r, col_of_row(r)) and 0 elsewhere.

    Block = f16 scale d (1.0 = 0x3C00) + 32 int8 quants; value = d * q.
    """
    nb = k // 32
    out = np.zeros((n_rows, nb, 34), np.uint8)
    out[:, :, 0:2] = np.frombuffer(struct.pack("<H", 0x3C00), np.uint8)
    for r in range(n_rows):
        c = col_of_row(r)
        out[r, c // 32, 2 + c % 32] = 1
    return out.reshape(-1)


def doc_example():
    """The reference's documented mlp_gated_silu example (crates/kernels/src/mlp.rs:120-137),
    widened to Q8_0's 32-element blocks: x = [2, 0, ...], gate(x) = up(x) = x[0] for
    every intermediate unit, down sums unit 0, so every output is silu(2) * 2 ~= 3.5231884."""
    hidden = intermediate = 32
    gate = q8_0_unit_rows(intermediate, hidden, lambda r: 0)
    up = q8_0_unit_rows(intermediate, hidden, lambda r: 0)
    down = q8_0_unit_rows(hidden, intermediate, lambda r: 0)
    x = np.zeros((1, hidden), np.float32)
    x[0, 0] = 2.0
    return x, gate, up, down, hidden, intermediate
