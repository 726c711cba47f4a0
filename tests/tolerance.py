"""Accuracy criteria shared by the parity tests.

GEMV (f32 x, f32 accumulate): max_i |y_i - r_i| / max(|r_i|, FLOOR * rms(r)) <= 1e-3
where r is the CPU oracle (the reference's sequential-k f32 sum).  The floor
keeps outputs that cancel to ~0 from dominating: the oracle's own f32 rounding
is ~sqrt(K) * 2^-24 * rms(r), i.e. ~4e-6 rms at K=4096 and ~7e-6 rms at
K=14336, so a per-element relative test without a floor would fail the oracle
against an exact f64 sum.  FLOOR = 0.02 keeps that term below 4e-4.
bf16 GEMM: the same formula with 2e-2, against the oracle run on the
bf16-rounded activations.
"""
import numpy as np

GEMV_RTOL = 1e-3
GEMM_RTOL = 2e-2
FLOOR = 0.02


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
