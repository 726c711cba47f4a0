"""GGUF file reader for the quantized linear path: header, tensor table, payloads.

Restates the header walk of `inspect_gguf` (crates/loader/src/gguf_inspect.rs:224-414:
magic, version 3, metadata key/values with the same limits, tensor infos,
`general.alignment`, data_start = align(end of tensor infos), file_offset =
data_start + offset, range checks against the file length) and adds what the
reference leaves for later (its `fixed_element_size` returns None for quantized
types, :208-219): byte lengths for Q4_K / Q6_K / Q8_0, memory-mapped payload
access, and upload of a quantized tensor into the CUDA backend.

GGUF stores dims innermost first, so a linear weight [out, in] has
shape = [in, out]: k = shape[0], n_rows = prod(shape[1:]) (:294-320).
"""
from __future__ import annotations

import mmap
import struct
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

from .errors import InvalidRequestError, OcelotlError, UnsupportedError
from .ggml import BLOCKS, GgmlType

GGUF_MAGIC = b"GGUF"
SUPPORTED_VERSION = 3
MAX_METADATA_ENTRIES = 200_000
MAX_TENSORS = 2_000_000
MAX_METADATA_STRING_BYTES = 16 * 1024 * 1024
MAX_KEY_BYTES = 65_535
MAX_TENSOR_NAME_BYTES = 65_535
MAX_ARRAY_ELEMENTS = 2_000_000
MAX_ARRAY_DEPTH = 4
MAX_TENSOR_DIMS = 8
DEFAULT_ALIGNMENT = 32

# metadata value types
U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
_SCALAR = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<?",
           U64: "<Q", I64: "<q", F64: "<d"}
# fixed element sizes (F32, F16, I8, I16, I32, I64, F64, BF16) as in fixed_element_size
_FIXED = {0: 4, 1: 2, 24: 1, 25: 2, 26: 4, 27: 8, 28: 8, 30: 2}


class InvalidModelError(OcelotlError):
    """OcelotlError::InvalidModel(InvalidModelError{path, field, message})."""

    def __init__(self, path, field_name, message):
        self.path, self.field, self.message = path, field_name, message
        where = f" at `{path}`" if path else ""
        fld = f" (field `{field_name}`)" if field_name else ""
        super().__init__(f"invalid model artifact{where}{fld}: {message}")


@dataclass
class TensorEntry:
    name: str
    shape: list[int]
    tensor_type: int
    offset: int
    file_offset: int = 0
    byte_len: int | None = None

    @property
    def k(self) -> int:
        return self.shape[0]

    @property
    def n_rows(self) -> int:
        n = 1
        for d in self.shape[1:]:
            n *= d
        return n


@dataclass
class Manifest:
    path: Path
    version: int
    metadata: dict = field(default_factory=dict)
    tensors: list[TensorEntry] = field(default_factory=list)
    alignment: int = DEFAULT_ALIGNMENT
    data_start: int = 0
    file_len: int = 0

    def tensor(self, name: str) -> TensorEntry:
        for t in self.tensors:
            if t.name == name:
                return t
        raise InvalidRequestError("tensor", f"no tensor named `{name}` in {self.path}")


def tensor_byte_len(tensor_type: int, shape: list[int]) -> int | None:
    """Payload bytes of a tensor, or None for types this path does not size."""
    count = 1
    for d in shape:
        count *= d
    if tensor_type in _FIXED:
        return count * _FIXED[tensor_type]
    try:
        geo = BLOCKS[GgmlType(tensor_type)]
    except (ValueError, KeyError):
        return None
    if shape[0] % geo.elems:
        return None
    return count // geo.elems * geo.nbytes


class _Reader:
    def __init__(self, path: Path, buf: memoryview):
        self.path, self.buf, self.pos = path, buf, 0

    def take(self, n: int, what: str) -> memoryview:
        if self.pos + n > len(self.buf):
            raise InvalidModelError(self.path, what, f"GGUF file truncated while reading {what}")
        v = self.buf[self.pos:self.pos + n]
        self.pos += n
        return v

    def scalar(self, fmt: str, what: str):
        return struct.unpack(fmt, self.take(struct.calcsize(fmt), what))[0]

    def string(self, what: str, max_len: int) -> str:
        n = self.scalar("<Q", what)
        if n > max_len or n > MAX_METADATA_STRING_BYTES:
            raise InvalidModelError(self.path, what, f"GGUF {what} length {n} exceeds max {max_len}")
        try:
            return bytes(self.take(n, what)).decode("utf-8")
        except UnicodeDecodeError:
            raise InvalidModelError(self.path, what, f"GGUF {what} is not valid UTF-8") from None

    def value(self, vtype: int, depth: int, key: str):
        if vtype in _SCALAR:
            return self.scalar(_SCALAR[vtype], key)
        if vtype == STRING:
            return self.string("metadata string", MAX_METADATA_STRING_BYTES)
        if vtype == ARRAY:
            et = self.scalar("<I", "metadata array")
            n = self.scalar("<Q", "metadata array")
            if n > MAX_ARRAY_ELEMENTS:
                raise InvalidModelError(self.path, "metadata array",
                                        f"GGUF metadata array length {n} exceeds max {MAX_ARRAY_ELEMENTS}")
            if depth >= MAX_ARRAY_DEPTH:
                raise InvalidModelError(self.path, "metadata array",
                                        f"GGUF metadata array nesting exceeds max depth {MAX_ARRAY_DEPTH}")
            if et not in _SCALAR and et not in (STRING, ARRAY):
                raise InvalidModelError(self.path, key, f"unknown GGUF metadata type {et}")
            return [self.value(et, depth + 1, key) for _ in range(n)]
        raise InvalidModelError(self.path, key, f"unknown GGUF metadata type {vtype}")


def inspect(path) -> Manifest:
    """Parse the header and tensor table of a GGUF v3 file (no payload read)."""
    path = Path(path)
    try:
        data = path.read_bytes() if path.stat().st_size < (1 << 20) else None
    except OSError as e:
        raise OcelotlError(f"IO error on `{path}`: {e}") from e
    if data is None:
        with open(path, "rb") as f:
            mm = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
        buf = memoryview(mm)
    else:
        buf = memoryview(data)
    r = _Reader(path, buf)
    magic = bytes(r.take(4, "magic"))
    if magic != GGUF_MAGIC:
        raise InvalidModelError(path, "magic", f"invalid GGUF magic bytes: {list(magic)}")
    version = r.scalar("<I", "version")
    if version != SUPPORTED_VERSION:
        raise UnsupportedError("gguf_version", str(version), [str(SUPPORTED_VERSION)])
    n_tensors = r.scalar("<Q", "tensor_count")
    n_kv = r.scalar("<Q", "metadata_kv_count")
    if n_tensors > MAX_TENSORS:
        raise InvalidModelError(path, "tensor_count", f"GGUF tensor_count {n_tensors} exceeds max {MAX_TENSORS}")
    if n_kv > MAX_METADATA_ENTRIES:
        raise InvalidModelError(path, "metadata_kv_count",
                                f"GGUF metadata_kv_count {n_kv} exceeds max {MAX_METADATA_ENTRIES}")
    meta = {}
    for _ in range(n_kv):
        key = r.string("metadata key", MAX_KEY_BYTES)
        vtype = r.scalar("<I", key)
        meta[key] = r.value(vtype, 0, key)
    alignment = meta.get("general.alignment", DEFAULT_ALIGNMENT)
    if not isinstance(alignment, int) or alignment <= 0 or alignment & (alignment - 1):
        raise InvalidModelError(path, "general.alignment", f"GGUF alignment {alignment} is not a power of two")
    tensors = []
    for _ in range(n_tensors):
        name = r.string("tensor name", MAX_TENSOR_NAME_BYTES)
        nd = r.scalar("<I", name)
        if nd == 0 or nd > MAX_TENSOR_DIMS:
            raise InvalidModelError(path, name, f"GGUF tensor `{name}` has unsupported dimension count {nd}")
        shape = [r.scalar("<Q", name) for _ in range(nd)]
        if any(d == 0 for d in shape):
            raise InvalidModelError(path, name, f"GGUF tensor `{name}` has a zero dimension")
        ttype = r.scalar("<I", name)
        offset = r.scalar("<Q", name)
        if offset % alignment:
            raise InvalidModelError(path, name, f"GGUF tensor `{name}` offset {offset} is not aligned to "
                                                f"{alignment} bytes")
        tensors.append(TensorEntry(name, shape, ttype, offset, 0, tensor_byte_len(ttype, shape)))
    data_start = (r.pos + alignment - 1) // alignment * alignment
    file_len = len(buf)
    if data_start > file_len:
        raise InvalidModelError(path, "tensor_data",
                                f"GGUF tensor data section starts at {data_start}, beyond file length {file_len}")
    for t in tensors:
        t.file_offset = data_start + t.offset
        if t.file_offset > file_len:
            raise InvalidModelError(path, t.name, f"GGUF tensor `{t.name}` starts at file offset {t.file_offset}, "
                                                  f"beyond file length {file_len}")
        if t.byte_len is not None and t.file_offset + t.byte_len > file_len:
            raise InvalidModelError(path, t.name, f"GGUF tensor `{t.name}` byte range {t.file_offset}.."
                                                  f"{t.file_offset + t.byte_len} exceeds file length {file_len}")
    return Manifest(path, version, meta, tensors, alignment, data_start, file_len)


def read_payload(manifest: Manifest, name: str) -> np.ndarray:
    """The raw bytes of a tensor (memory-mapped, read-only uint8 view)."""
    t = manifest.tensor(name)
    if t.byte_len is None:
        raise UnsupportedError("gguf tensor payload", str(t.tensor_type), ["F32", "F16", "BF16", "Q4_K", "Q6_K",
                                                                            "Q8_0", "integer types"])
    return np.memmap(manifest.path, dtype=np.uint8, mode="r", offset=t.file_offset, shape=(t.byte_len,))


def upload_quant_tensor(backend, manifest: Manifest, name: str):
    """Read a Q4_K / Q6_K / Q8_0 weight from the file and upload it (repacked on the device)."""
    t = manifest.tensor(name)
    if t.tensor_type not in (GgmlType.Q4_K, GgmlType.Q6_K, GgmlType.Q8_0):
        raise UnsupportedError("quantized weight type", str(t.tensor_type), ["Q4_K(12)", "Q6_K(14)", "Q8_0(8)"])
    payload = np.ascontiguousarray(read_payload(manifest, name))
    return backend.upload_quant(t.tensor_type, payload, t.n_rows, t.k)
