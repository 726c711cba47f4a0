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
Gated bf16 GEMM (act = silu(g) * u): each factor carries the GEMM's absolute
error ~eps * rms of its own column set, so the product's error is
~eps * (|silu(g)| * rms(u) + |u| * rms(g)); that (or |act| if larger) is the
denominator, the bound again GEMM_RTOL.  A floor at rms(act) alone fails a
correct kernel wherever a large gate meets a small up (|g| ~ 3.5 rms, |u| ~ 0.2
rms gives ~3e-2 for the exact f32 product of bf16-rounded weights).
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


def gated_rel_err(y, g, u):
    """max |y - silu(g) u| / max(|silu(g) u|, |silu(g)| rms(u) + |u| rms(g))."""
    y = np.asarray(y, dtype=np.float64)
    g = np.asarray(g, dtype=np.float64)
    u = np.asarray(u, dtype=np.float64)
    with np.errstate(over="ignore"):
        sg = g / (1.0 + np.exp(-g))
    r = sg * u
    den = np.maximum(np.abs(r), np.abs(sg) * np.sqrt(np.mean(u * u)) + np.abs(u) * np.sqrt(np.mean(g * g)))
    den = np.where(den == 0, 1.0, den)
    return float(np.max(np.abs(y - r) / den)) if r.size else 0.0


# ---- achieved errors, recorded by the parity tests -------------------------
# Every parity test records what it achieved, so the margin under each bound is
# visible: pytest prints the table at the end of the run (tests/conftest.py),
# and OCL_PARITY_LOG=<path> also writes it as JSON.
STRICT_FLOOR = 1e-3  # the stricter floor max(|r|, 1e-3 rms(r)), reported beside FLOOR
RECORDED: dict = {}


def record_err(name, value, **extra):
    RECORDED[name] = dict({"err": float(value)}, **{k: float(v) for k, v in extra.items()})


def gemv_err(name, y, r):
    """rel_err with FLOOR (the asserted one), recorded with the 1e-3-floor and normwise figures."""
    e = rel_err(y, r)
    record_err(name, e, err_floor_1e3=rel_err(y, r, floor=STRICT_FLOOR), normwise=normwise_err(y, r))
    return e


def gemm_err(name, y, r):
    """rel_err with GEMM_FLOOR (the asserted one), recorded with the normwise figure."""
    e = rel_err(y, r, floor=GEMM_FLOOR)
    record_err(name, e, err_floor_1e3=rel_err(y, r, floor=STRICT_FLOOR), normwise=normwise_err(y, r))
    return e


def gated_gemv_err(y, g, u, floor=FLOOR):
    """Error of act = silu(g) * u from the GEMV, held to GEMV_RTOL.

    g and u are the oracle's gate and up outputs.  The GEMV bound allows each of
    them an error of up to GEMV_RTOL * max(|v|, floor * rms(v)); propagated
    through silu(g) * u (first order: d act = silu'(g) u dg + silu(g) du) that is
    GEMV_RTOL times
        den = |silu'(g)| |u| max(|g|, floor rms(g)) + |silu(g)| max(|u|, floor rms(u)),
    so max |y - silu(g) u| / max(|silu(g) u|, den) <= GEMV_RTOL is the same
    1e-3 requirement as for a single projection, stated for the product.
    silu'(g) = sigmoid(g) (1 + g (1 - sigmoid(g))).  Where silu(g) underflows
    f32 (g below about -87) both den and the product are below f32's normal
    range, so den is kept at or above 2^-20 rms(act): f32 rounding noise of the
    f32 evaluation, far below the GEMV bound.
    """
    y = np.asarray(y, dtype=np.float64)
    g = np.asarray(g, dtype=np.float64)
    u = np.asarray(u, dtype=np.float64)
    with np.errstate(over="ignore"):
        sig = 1.0 / (1.0 + np.exp(-g))
    sg = g * sig
    dsg = sig * (1.0 + g * (1.0 - sig))
    r = sg * u
    rms = lambda v: np.sqrt(np.mean(v * v)) if v.size else 0.0  # noqa: E731
    den = np.abs(dsg) * np.abs(u) * np.maximum(np.abs(g), floor * rms(g)) + \
        np.abs(sg) * np.maximum(np.abs(u), floor * rms(u))
    den = np.maximum(np.maximum(np.abs(r), den), 2.0 ** -20 * rms(r))
    den = np.where(den == 0, 1.0, den)
    return float(np.max(np.abs(y - r) / den)) if r.size else 0.0
