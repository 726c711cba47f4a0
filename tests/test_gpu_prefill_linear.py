"""GPU: linear_d with many rows (prefill) runs ONE tcgen05 GEMM, checked against the CPU oracle.

The reference's linear_d takes f32 activations at any row count
(crates/kernels/src/lib.rs:193-217); Whisper's encoder calls it with rows =
audio_ctx >= 1500 (crates/models/src/whisper/primitives.rs:787-839).  From 64
rows on, ocl_q_linear rounds x to bf16 and runs the prefill GEMM (f32
accumulate, f32 out, bias added in the epilogue) instead of streaming the weight
once per 16 rows.  Its bound is the prefill one: max |y - r| / max(|r|, rms(r))
<= 2e-2, where r is the oracle (the reference's sequential-k f32 sum) on the
SAME bf16-rounded x.  Below the threshold the GEMV and its 1e-3 bound apply.
"""
import os

import numpy as np
import pytest
import torch

from tests.tolerance import GEMM_RTOL, GEMV_RTOL, gemm_err, gemv_err

pytestmark = pytest.mark.gpu
THREADS = max(1, min(32, os.cpu_count() or 1))


def _bf16_round(x: np.ndarray) -> np.ndarray:
    return torch.from_numpy(x).to(torch.bfloat16).float().numpy()


def _case(backend, oracle, t, n, k, rows, seed, check_rows=None, bias=True):
    from ocelotl_b200 import synth
    blocks = synth.quant_blocks(t, n, k, seed, f"pl{t}", device="cuda")
    w = backend.upload_quant(t, blocks, n, k)
    x = synth.activations(rows, k, seed, "plx").numpy()
    b = synth.activations(1, n, seed, "plb").numpy().reshape(-1) if bias else None
    y = torch.full((rows, n), float("nan"), device="cuda")
    backend.linear_dev(w, torch.from_numpy(x).cuda(), rows, y, torch.from_numpy(b).cuda() if bias else None)
    torch.cuda.synchronize()
    assert backend.take_device_errors() == (0, 0)
    sel = np.arange(rows) if check_rows is None else np.asarray(check_rows)
    got = y.cpu().numpy()[sel]
    return got, blocks.cpu().numpy(), x[sel], b


@pytest.mark.parametrize("t", [12, 14, 8])
@pytest.mark.parametrize("rows", [64, 200, 1500])
def test_linear_d_prefill_rows_use_gemm(backend, oracle, t, rows):
    n, k = 320, 1024
    got, blocks, x, b = _case(backend, oracle, t, n, k, rows, 31)
    ref = oracle.q_linear(t, blocks, _bf16_round(x), rows, k, n, bias=b, threads=THREADS)
    e = gemm_err(f"prefill_linear.t{t}.rows{rows}", got, ref)
    assert e <= GEMM_RTOL, e


@pytest.mark.parametrize("t,n,k", [(12, 4096, 4096), (14, 4096, 14336), (12, 6144, 4096)])
def test_linear_d_prefill_baseline_shape_vs_oracle(backend, oracle, t, n, k):
    """configs[2] shapes at M = 512, 48 of the rows checked against the CPU oracle."""
    rows = 512
    sel = np.random.default_rng(7).choice(rows, 48, replace=False)
    got, blocks, x, b = _case(backend, oracle, t, n, k, rows, 33, check_rows=sel, bias=False)
    ref = oracle.q_linear(t, blocks, _bf16_round(x), len(sel), k, n, threads=THREADS)
    e = gemm_err(f"prefill_linear.baseline.t{t}.{n}x{k}", got, ref)
    assert e <= GEMM_RTOL, e


def test_linear_d_below_threshold_keeps_gemv_accuracy(backend, oracle):
    n, k, rows = 320, 1024, 63
    got, blocks, x, b = _case(backend, oracle, 12, n, k, rows, 35)
    ref = oracle.q_linear(12, blocks, x, rows, k, n, bias=b, threads=THREADS)
    assert gemv_err("prefill_linear.rows63_gemv", got, ref) <= GEMV_RTOL


def test_gemm_threshold_can_be_disabled(backend, oracle):
    n, k, rows = 128, 512, 80
    backend.set_gemm_min_rows(0)
    try:
        got, blocks, x, b = _case(backend, oracle, 14, n, k, rows, 37)
    finally:
        backend.set_gemm_min_rows(64)
    ref = oracle.q_linear(14, blocks, x, rows, k, n, bias=b, threads=THREADS)
    assert gemv_err("prefill_linear.disabled_gemv", got, ref) <= GEMV_RTOL


def test_host_slices_prefill(backend, oracle):
    """linear_out_by_in (host slices) with many rows goes through the same GEMM."""
    from ocelotl_b200 import synth
    n, k, rows = 256, 768, 96
    blocks = synth.quant_blocks(12, n, k, 39, "plh")
    w = backend.upload_quant(12, blocks, n, k)
    x = synth.activations(rows, k, 39, "plhx").numpy()
    out = np.zeros(rows * n, np.float32)
    backend.linear_out_by_in(x, rows, k, w, n, None, out)
    ref = oracle.q_linear(12, blocks.numpy(), _bf16_round(x), rows, k, n, threads=THREADS)
    assert gemm_err("prefill_linear.host", out.reshape(rows, n), ref) <= GEMM_RTOL


def test_mlp_gated_silu_prefill(backend, oracle):
    """Many rows: gate+up as one gated GEMM (f32 act), then down as a GEMM on bf16(act)."""
    from ocelotl_b200 import synth
    from tests.tolerance import gated_rel_err
    hidden, inter, rows = 512, 768, 128
    gb = synth.quant_blocks(12, inter, hidden, 41, "pg")
    ub = synth.quant_blocks(12, inter, hidden, 41, "pu")
    db = synth.quant_blocks(14, hidden, inter, 41, "pd")
    g = backend.upload_quant(12, gb, inter, hidden)
    u = backend.upload_quant(12, ub, inter, hidden)
    d = backend.upload_quant(14, db, hidden, inter)
    pair = backend.pair_gated(g, u)
    x = synth.activations(rows, hidden, 41, "pgx").numpy()
    act = torch.empty(rows * inter, device="cuda")
    out = torch.empty(rows * hidden, device="cuda")
    backend.mlp_gated_silu(torch.from_numpy(x).cuda(), rows, hidden, inter, pair, None, d, act, None, out)
    backend.synchronize()
    xb = _bf16_round(x)
    gy = oracle.q_linear(12, gb.numpy(), xb, rows, hidden, inter, threads=THREADS)
    uy = oracle.q_linear(12, ub.numpy(), xb, rows, hidden, inter, threads=THREADS)
    a = act.cpu().numpy().reshape(rows, inter)
    ea = gated_rel_err(a, gy, uy)
    from tests.tolerance import record_err
    record_err("prefill_mlp.act", ea)
    assert ea <= GEMM_RTOL, ea
    ref_out = oracle.q_linear(14, db.numpy(), _bf16_round(a), rows, inter, hidden, threads=THREADS)
    assert gemm_err("prefill_mlp.out", out.cpu().numpy().reshape(rows, hidden), ref_out) <= GEMM_RTOL
