"""Accuracy criteria shared by the parity tests.

GEMV (f32 x, f32 accumulate): max_i |y_i - r_i| / max(|r_i|, FLOOR * rms(r)) <= 1e-3
where r is the CPU oracle (the reference's sequential-k f32 sum).  The floor
keeps outputs that cancel to ~0 from dominating: the oracle's own f32 rounding
is ~sqrt(K) * 2^-24 * rms(r), i.e. ~4e-6 rms at K=4096 and ~7e-6 rms at
K=14336, so a per-element relative test without a floor would fail the oracle
against an exact f64 sum.  FLOOR = 0.02 keeps that term below 4e-4.
bf16 GEMM (prefill): |y_i - r_i| / max(|r_i|, rms(r)) <= 2e-2 (GEMM_FLOOR = 1),
against the f32 product of the bf16-rounded activations and the exact f32
dequantized weights.  Here the weights themselves are rounded to bf16 (2^-9
relative) before the tensor cores see them, so an output that cancels to ~0
carries an absolute error of ~2^-9 * rms(r); a floor below rms would fail any
correct bf16 kernel on such outputs.
"""
import numpy as np

GEMV_RTOL = 1e-3
GEMM_RTOL = 2e-2
FLOOR = 0.02
GEMM_FLOOR = 1.0


def rel_err(y, r, floor=FLOOR):
    y = np.asarray(y, dtype=np.float64)
    r = np.asarray(r, dtype=np.float64)
    rms = np.sqrt(np.mean(r * r)) if r.size else 0.0
    den = np.maximum(np.abs(r), floor * rms)
    den = np.where(den == 0, 1.0, den)
    return float(np.max(np.abs(y - r) / den)) if r.size else 0.0


def normwise_err(y, r):
    y = np.asarray(y, dtype=np.float64)
    r = np.asarray(r, dtype=np.float64)
    m = np.max(np.abs(r))
    return float(np.max(np.abs(y - r)) / (m if m else 1.0))
