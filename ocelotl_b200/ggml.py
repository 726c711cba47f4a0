"""GGUF tensor-type tags and block geometry for the quantized path.

Tags follow GgmlTensorType::from_raw (crates/loader/src/gguf_inspect.rs:172-206).
The reference returns no byte length for quantized tensors
(fixed_element_size, crates/loader/src/gguf_inspect.rs:208-219); `byte_len`
below is the block sizing the payload upload needs.
"""
from __future__ import annotations

from dataclasses import dataclass
from enum import IntEnum


class GgmlType(IntEnum):
    Q8_0 = 8
    Q4_K = 12
    Q6_K = 14


@dataclass(frozen=True)
class BlockGeometry:
    elems: int   # weights per block
    nbytes: int  # bytes per block


BLOCKS = {
    GgmlType.Q4_K: BlockGeometry(256, 144),
    GgmlType.Q6_K: BlockGeometry(256, 210),
    GgmlType.Q8_0: BlockGeometry(32, 34),
}


def geometry(t: int) -> BlockGeometry:
    from .errors import UnsupportedError
    try:
        return BLOCKS[GgmlType(t)]
    except (ValueError, KeyError):
        raise UnsupportedError("ggml_type", str(t), ["Q4_K(12)", "Q6_K(14)", "Q8_0(8)"]) from None


def byte_len(t: int, n_rows: int, k: int) -> int:
    """Bytes of an [n_rows, k] tensor of GGUF blocks (k a multiple of the block size)."""
    g = geometry(t)
    if k % g.elems:
        from .errors import UnsupportedError
        raise UnsupportedError(f"{GgmlType(t).name} in_features", str(k), [f"multiples of {g.elems}"])
    return n_rows * (k // g.elems) * g.nbytes
