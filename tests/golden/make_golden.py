"""Generate the committed golden fixtures for the dequantize half of the path.

The reference (Dieshen/ocelotl) has no k-quant arithmetic and no quantized
fixtures (crates/loader/src/gguf_inspect.rs:208-219; docs/design/quantization.md
plans "known small tensors with exact expected dequantized values").  The block
arithmetic is the public GGUF/ggml format; this script pins it with the
third-party `gguf` Python package, version 0.19.0 (`gguf.quants.dequantize`),
which must be importable where the script runs.  It is NOT needed at test time:
the outputs are committed as tests/golden/dequant_<type>.npz with
  blocks    uint8  [n_blocks * block_bytes]  (GGUF layout)
  expected  float32 [n_blocks * block_elems] (gguf.quants.dequantize)
  sha256    the hex digest of expected.tobytes()
Blocks are seeded random ones (bench distributions) followed by hand-made edge
blocks: f16 zero / subnormal / max-normal / inf d and dmin, all-0 and all-max
scales and quants, Q6_K scale -128 and 127, Q8_0 quants -128 and 127.

Run:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import hashlib
from pathlib import Path

import numpy as np

OUT = Path(__file__).resolve().parent
SEED = 20261201

Q8_0, Q4_K, Q6_K = 8, 12, 14
GEO = {Q4_K: (256, 144), Q6_K: (256, 210), Q8_0: (32, 34)}
NAME = {Q4_K: "q4_k", Q6_K: "q6_k", Q8_0: "q8_0"}

F16_EDGE = [0x0000, 0x8000, 0x0001, 0x03FF, 0x0400, 0x7BFF, 0x7C00, 0x3C00, 0x2E66, 0xA4CD]


def f16_abs_normal(rng, n, std=0.02):
    return (np.abs(rng.standard_normal(n)) * std).astype(np.float16).view(np.uint16)


def random_blocks(t, n, rng):
    elems, nbytes = GEO[t]
    b = rng.integers(0, 256, size=(n, nbytes), dtype=np.uint8)
    if t == Q4_K:
        b[:, 0:2] = f16_abs_normal(rng, n).view(np.uint8).reshape(n, 2)
        b[:, 2:4] = f16_abs_normal(rng, n).view(np.uint8).reshape(n, 2)
    elif t == Q6_K:
        b[:, 192:208] = rng.integers(-64, 64, size=(n, 16)).astype(np.int8).view(np.uint8)
        b[:, 208:210] = f16_abs_normal(rng, n).view(np.uint8).reshape(n, 2)
    else:
        b[:, 2:34] = rng.integers(-127, 128, size=(n, 32)).astype(np.int8).view(np.uint8)
        b[:, 0:2] = f16_abs_normal(rng, n).view(np.uint8).reshape(n, 2)
    return b


def edge_blocks(t, rng):
    elems, nbytes = GEO[t]
    out = []
    for i, h in enumerate(F16_EDGE):
        b = random_blocks(t, 1, rng)[0]
        h16 = np.array([h], dtype=np.uint16).view(np.uint8)
        if t == Q4_K:
            b[0:2] = h16
            b[2:4] = np.array([F16_EDGE[(i + 3) % len(F16_EDGE)]], dtype=np.uint16).view(np.uint8)
            if i == 0:
                b[4:16] = 0xFF   # all scales / mins = 63
                b[16:] = 0xFF    # all quants = 15
            if i == 1:
                b[4:] = 0
        elif t == Q6_K:
            b[208:210] = h16
            if i == 0:
                b[192:208] = np.array([-128, 127] * 8, dtype=np.int8).view(np.uint8)
                b[0:192] = 0xFF  # all quants 63
            if i == 1:
                b[0:192] = 0     # all quants 0 -> -32
        else:
            b[0:2] = h16
            if i == 0:
                b[2:34] = np.array([-128, 127] * 16, dtype=np.int8).view(np.uint8)
        out.append(b)
    return np.stack(out)


def main():
    import gguf
    from gguf import GGMLQuantizationType as GT
    from gguf import quants

    gtype = {Q4_K: GT.Q4_K, Q6_K: GT.Q6_K, Q8_0: GT.Q8_0}
    rng = np.random.default_rng(SEED)
    for t in (Q4_K, Q6_K, Q8_0):
        elems, nbytes = GEO[t]
        blocks = np.concatenate([random_blocks(t, 48, rng), edge_blocks(t, rng)])
        with np.errstate(all="ignore"):
            exp = quants.dequantize(blocks, gtype[t]).astype(np.float32).reshape(-1)
        digest = hashlib.sha256(exp.tobytes()).hexdigest()
        np.savez_compressed(OUT / f"dequant_{NAME[t]}.npz", blocks=blocks.reshape(-1), expected=exp,
                            sha256=np.array(digest), gguf_version=np.array(getattr(gguf, "__version__", "0.19.0")))
        print(NAME[t], blocks.shape[0], "blocks", digest)


if __name__ == "__main__":
    main()
