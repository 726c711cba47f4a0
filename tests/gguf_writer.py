"""Minimal GGUF v3 writer for tests (the reference's own tests write synthetic
files the same way: crates/loader/src/gguf_inspect.rs:779-806)."""
import struct


def _s(b: bytes) -> bytes:
    return struct.pack("<Q", len(b)) + b


def write_gguf(path, tensors, metadata=None, alignment=None, version=3, magic=b"GGUF", bad_offset=False):
    """tensors: list of (name, shape (innermost first), ggml type, payload bytes)."""
    meta = list((metadata or {}).items())
    if alignment is not None:
        meta.append(("general.alignment", ("u32", alignment)))
    align = alignment or 32
    out = bytearray(magic + struct.pack("<I", version) + struct.pack("<QQ", len(tensors), len(meta)))
    for k, (kind, v) in meta:
        out += _s(k.encode())
        if kind == "u32":
            out += struct.pack("<II", 4, v)
        elif kind == "str":
            out += struct.pack("<I", 8) + _s(v.encode())
        elif kind == "f32arr":
            out += struct.pack("<IIQ", 9, 6, len(v)) + b"".join(struct.pack("<f", x) for x in v)
        else:
            raise ValueError(kind)
    offs, off = [], 0
    for name, shape, t, payload in tensors:
        offs.append(off)
        off += (len(payload) + align - 1) // align * align
    for (name, shape, t, payload), o in zip(tensors, offs):
        out += _s(name.encode()) + struct.pack("<I", len(shape)) + b"".join(struct.pack("<Q", d) for d in shape)
        out += struct.pack("<IQ", t, o + (1 if bad_offset else 0))
    out += b"\0" * ((-len(out)) % align)
    for (name, shape, t, payload), o in zip(tensors, offs):
        out += bytes(payload) + b"\0" * ((-len(payload)) % align)
    with open(path, "wb") as f:
        f.write(out)
