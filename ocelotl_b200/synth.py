"""Seeded synthetic GGUF blocks and activations (benchmark / test inputs).

Distributions are the benchmark's: Q4_K d, dmin = f16(|N(0, 0.02)|), 6-bit
scales/mins i.i.d. U{0..63}, 4-bit quants U{0..15}; Q6_K d = f16(|N(0, 0.02)|),
int8 scales U{-64..63}, 6-bit quants U{0..63}; Q8_0 d = f16(|N(0, 0.02)|), int8
quants U{-127..127}; activations f32 N(0, 1).

Every bit of the packed Q4_K scale bytes and of the Q4_K / Q6_K quant bytes is
used by exactly one field, so uniform random bytes give exactly those i.i.d.
uniform fields; only d/dmin, the Q6_K scales and the Q8_0 quants are drawn
separately.  Generation runs with torch on the target device (CPU or CUDA), so
multi-GB weight sets are made in milliseconds on the GPU.  Streams are derived
from one u64 seed and the tensor name (splitmix64 of seed ^ fnv1a64(name)).
"""
from __future__ import annotations

import torch

from .ggml import GgmlType, geometry

_M64 = (1 << 64) - 1


def splitmix64(z: int) -> int:
    z = (z + 0x9E3779B97F4A7C15) & _M64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & _M64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & _M64
    return z ^ (z >> 31)


def fnv1a64(s: str) -> int:
    h = 0xCBF29CE484222325
    for b in s.encode():
        h = ((h ^ b) * 0x100000001B3) & _M64
    return h


def stream_seed(seed: int, name: str) -> int:
    return splitmix64((seed ^ fnv1a64(name)) & _M64) & ((1 << 63) - 1)


def _gen(seed: int, name: str, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(stream_seed(seed, name))
    return g


def _f16_abs_normal(n: int, std: float, g, device) -> torch.Tensor:
    v = (torch.randn(n, generator=g, device=device, dtype=torch.float32).abs() * std).to(torch.float16)
    return v.view(torch.uint8).view(n, 2)


def quant_blocks(ggml_type: int, n_rows: int, k: int, seed: int, name: str,
                 device="cpu") -> torch.Tensor:
    """GGUF blocks of an [n_rows, k] weight as a flat uint8 tensor on `device`."""
    geo = geometry(ggml_type)
    t = GgmlType(ggml_type)
    nb = n_rows * (k // geo.elems)
    g = _gen(seed, name, device)
    blk = torch.randint(0, 256, (nb, geo.nbytes), generator=g, device=device, dtype=torch.uint8)
    if t == GgmlType.Q4_K:
        blk[:, 0:2] = _f16_abs_normal(nb, 0.02, g, device)
        blk[:, 2:4] = _f16_abs_normal(nb, 0.02, g, device)
    elif t == GgmlType.Q6_K:
        sc = torch.randint(-64, 64, (nb, 16), generator=g, device=device, dtype=torch.int16)
        blk[:, 192:208] = sc.to(torch.int8).view(torch.uint8)
        blk[:, 208:210] = _f16_abs_normal(nb, 0.02, g, device)
    else:
        q = torch.randint(-127, 128, (nb, 32), generator=g, device=device, dtype=torch.int16)
        blk[:, 2:34] = q.to(torch.int8).view(torch.uint8)
        blk[:, 0:2] = _f16_abs_normal(nb, 0.02, g, device)
    return blk.reshape(-1)


def activations(rows: int, k: int, seed: int, name: str, device="cpu", dtype=torch.float32) -> torch.Tensor:
    g = _gen(seed, name, device)
    return torch.randn(rows, k, generator=g, device=device, dtype=torch.float32).to(dtype)
