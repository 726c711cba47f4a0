"""CPU oracle for the quantized-linear path -- TEST INFRASTRUCTURE ONLY.

ctypes wrapper of liboracle.so (oracle.c): the reference's f16 decode, the GGUF
block dequantization, linear_out_by_in (scalar, sequential k per output, no FMA)
and its AVX2 variant.  Only tests/, __graft_entry__.smoke() and bench.py's CPU
baseline leg use it; the product never imports it.

Parity status: the dequantization is pinned bit-for-bit to golden fixtures made
with gguf 0.19.0 (tests/golden/make_golden.py); the multiply is pinned to
hand-computed cases and to the tile/tail/threading properties the reference's
own tests check (crates/kernels/src/lib.rs:2650-3042).
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"

Q8_0, Q4_K, Q6_K = 8, 12, 14
BLOCK = {Q4_K: (256, 144), Q6_K: (256, 210), Q8_0: (32, 34)}

_lib = None


def build() -> Path:
    src = [HERE / "oracle.c", HERE / "oracle.h"]
    if not LIB_PATH.exists() or any(s.stat().st_mtime > LIB_PATH.stat().st_mtime for s in src):
        subprocess.run(["make", "-C", str(HERE), "liboracle.so"], check=True, capture_output=True)
    return LIB_PATH


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = C.CDLL(str(LIB_PATH))
        vp, sz = C.c_void_p, C.c_size_t
        L.orc_f16_to_f32.restype = C.c_float
        L.orc_f16_to_f32.argtypes = [C.c_uint16]
        L.orc_dequant.argtypes = [C.c_int, vp, sz, sz, vp]
        L.orc_linear_out_by_in.argtypes = [vp, sz, sz, vp, sz, vp, vp]
        L.orc_linear_out_by_in_avx2.argtypes = [vp, sz, sz, vp, sz, vp, vp]
        L.orc_q_linear.argtypes = [C.c_int, vp, vp, sz, sz, sz, vp, vp, C.c_int]
        L.orc_q_linear_avx2.argtypes = [C.c_int, vp, vp, sz, sz, sz, vp, vp, C.c_int]
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def f16_to_f32(bits: int) -> float:
    return lib().orc_f16_to_f32(bits)


def dequant(ggml_type: int, blocks, n_rows: int, k: int) -> np.ndarray:
    b = np.ascontiguousarray(np.asarray(blocks, dtype=np.uint8).reshape(-1))
    out = np.empty((n_rows, k), dtype=np.float32)
    if lib().orc_dequant(ggml_type, _p(b), n_rows, k, _p(out)):
        raise ValueError("oracle dequant: bad type or k")
    return out


def linear_out_by_in(x, rows, in_features, w, out_features, bias=None, avx2=False) -> np.ndarray:
    x, w = _f32(x), _f32(w)
    b = None if bias is None else _f32(bias)
    out = np.empty((rows, out_features), dtype=np.float32)
    fn = lib().orc_linear_out_by_in_avx2 if avx2 else lib().orc_linear_out_by_in
    if fn(_p(x), rows, in_features, _p(w), out_features, _p(b), _p(out)):
        raise RuntimeError("oracle linear failed (avx2 unavailable?)")
    return out


def q_linear(ggml_type, blocks, x, rows, in_features, out_features, bias=None, threads=1,
             avx2=False) -> np.ndarray:
    b8 = np.ascontiguousarray(np.asarray(blocks, dtype=np.uint8).reshape(-1))
    x = _f32(x)
    b = None if bias is None else _f32(bias)
    out = np.empty((rows, out_features), dtype=np.float32)
    fn = lib().orc_q_linear_avx2 if avx2 else lib().orc_q_linear
    if fn(ggml_type, _p(b8), _p(x), rows, in_features, out_features, _p(b), _p(out), threads):
        raise RuntimeError("oracle q_linear failed")
    return out


def silu_inplace(v: np.ndarray) -> np.ndarray:
    """silu(z) = z * (1 / (1 + exp(-z))) in f32 (crates/kernels/src/mlp.rs:77-86)."""
    v = np.asarray(v, dtype=np.float32)
    with np.errstate(over="ignore"):
        sig = np.float32(1.0) / (np.float32(1.0) + np.exp(-v))
    v *= sig
    return v


def q_gated(ggml_type, gate_blocks, up_blocks, x, rows, hidden, intermediate, threads=1) -> np.ndarray:
    """silu(x . gate^T) * (x . up^T): mlp_gated_silu up to the down projection
    (crates/kernels/src/mlp.rs:216-230), the matmuls as q_linear."""
    g = q_linear(ggml_type, gate_blocks, x, rows, hidden, intermediate, threads=threads)
    u = q_linear(ggml_type, up_blocks, x, rows, hidden, intermediate, threads=threads)
    silu_inplace(g)
    g *= u
    return g


def q_mlp_gated_silu(ggml_type, gate_blocks, up_blocks, down_type, down_blocks, x, rows, hidden, intermediate,
                     threads=1) -> tuple[np.ndarray, np.ndarray]:
    """(act, out) of mlp_gated_silu (crates/kernels/src/mlp.rs:139-240) on quantized weights."""
    act = q_gated(ggml_type, gate_blocks, up_blocks, x, rows, hidden, intermediate, threads=threads)
    out = q_linear(down_type, down_blocks, act, rows, intermediate, hidden, threads=threads)
    return act, out


def greedy_sample(logits) -> int:
    """greedy_sample (crates/runtime/src/sampling.rs:29-52): scan from index 0,
    move only on a strictly greater value.  Raises ValueError on no logits."""
    v = np.asarray(logits, dtype=np.float32).reshape(-1)
    if v.size == 0:
        raise ValueError("greedy_sample requires at least one logit")
    best_idx, best_val = 0, v[0]
    for i in range(1, v.size):
        if v[i] > best_val:
            best_idx, best_val = i, v[i]
    return best_idx


def greedy_sample_fast(logits) -> int:
    """Vectorised form of greedy_sample for large vocabularies (same answer):
    a NaN at index 0 is never displaced; otherwise NaNs never win and the first
    maximum is taken (-0.0 == +0.0 under numpy's comparison too)."""
    v = np.asarray(logits, dtype=np.float32).reshape(-1)
    if v.size == 0:
        raise ValueError("greedy_sample requires at least one logit")
    if np.isnan(v[0]):
        return 0
    w = np.where(np.isnan(v), -np.inf, v)
    return int(np.argmax(w))
