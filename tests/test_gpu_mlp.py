"""GPU: fused gated MLP (gate+up in one GEMV pass, silu*up epilogue, then down)
vs the CPU oracle, through the C ABI (crates/kernels/src/mlp.rs:139-240)."""
import numpy as np
import pytest
import torch

from tests.tolerance import GEMV_RTOL, gated_gemv_err, gemv_err, normwise_err, record_err, rel_err

pytestmark = pytest.mark.gpu


def _case(backend, t, td, hidden, inter, rows, seed):
    from ocelotl_b200 import synth
    gb = synth.quant_blocks(t, inter, hidden, seed, "gate")
    ub = synth.quant_blocks(t, inter, hidden, seed, "up")
    db = synth.quant_blocks(td, hidden, inter, seed, "down") if td else None
    x = synth.activations(rows, hidden, seed, "x").numpy()
    g = backend.upload_quant(t, gb, inter, hidden)
    u = backend.upload_quant(t, ub, inter, hidden)
    d = backend.upload_quant(td, db, hidden, inter) if td else None
    return gb.numpy(), ub.numpy(), None if db is None else db.numpy(), x, g, u, d


@pytest.mark.parametrize("t", [12, 14, 8])
@pytest.mark.parametrize("rows", [1, 2, 5, 16, 19])
@pytest.mark.parametrize("hidden,inter", [(512, 200), (1024, 768)])
def test_gated_gemv_matches_oracle(backend, oracle, t, rows, hidden, inter):
    gb, ub, _, x, g, u, _ = _case(backend, t, None, hidden, inter, rows, 11)
    pair = backend.pair_gated(g, u)
    xd = torch.from_numpy(x).cuda()
    act = torch.empty(rows, inter, device="cuda")
    backend.linear_gated(pair, xd, rows, act)
    backend.synchronize()
    gy = oracle.q_linear(t, gb, x, rows, hidden, inter, threads=8)
    uy = oracle.q_linear(t, ub, x, rows, hidden, inter, threads=8)
    e = gated_gemv_err(act.cpu().numpy(), gy, uy)
    record_err(f"gated_gemv.t{t}.rows{rows}.{hidden}x{inter}", e)
    assert e <= GEMV_RTOL, (t, rows, e)


@pytest.mark.parametrize("rows", [1, 8, 16])
def test_gated_gemv_llama_shape(backend, oracle, rows):
    """8B MLP: gate/up Q4_K [14336, 4096] (split-K at M > 2 exercises the partial path)."""
    hidden, inter = 4096, 14336
    gb, ub, _, x, g, u, _ = _case(backend, 12, None, hidden, inter, rows, 5)
    pair = backend.pair_gated(g, u)
    act = torch.empty(rows, inter, device="cuda")
    backend.linear_gated(pair, torch.from_numpy(x).cuda(), rows, act)
    backend.synchronize()
    gy = oracle.q_linear(12, gb, x, rows, hidden, inter, threads=16)
    uy = oracle.q_linear(12, ub, x, rows, hidden, inter, threads=16)
    e = gated_gemv_err(act.cpu().numpy(), gy, uy)
    record_err(f"gated_gemv.llama.rows{rows}", e)
    assert e <= GEMV_RTOL, e
    assert backend.take_device_errors() == (0, 0)


def test_gated_equals_separate_projections(backend):
    """The pair pass gives the same act as gate and up run separately then silu*up on torch."""
    from ocelotl_b200 import synth
    hidden, inter, rows = 2048, 1000, 4
    g = backend.upload_quant(12, synth.quant_blocks(12, inter, hidden, 3, "g"), inter, hidden)
    u = backend.upload_quant(12, synth.quant_blocks(12, inter, hidden, 3, "u"), inter, hidden)
    x = synth.activations(rows, hidden, 3, "x").cuda()
    gy = torch.empty(rows, inter, device="cuda")
    uy = torch.empty(rows, inter, device="cuda")
    backend.linear_dev(g, x, rows, gy)
    backend.linear_dev(u, x, rows, uy)
    act = torch.empty(rows, inter, device="cuda")
    backend.linear_gated(backend.pair_gated(g, u), x, rows, act)
    backend.synchronize()
    ref = (gy * torch.sigmoid(gy) * uy).cpu().numpy()
    assert rel_err(act.cpu().numpy(), ref) <= 1e-5


@pytest.mark.parametrize("t,td", [(12, 14), (14, 14), (8, 8)])
@pytest.mark.parametrize("rows", [1, 4])
def test_mlp_gated_silu_matches_oracle(backend, oracle, t, td, rows):
    hidden, inter = 1024, 2816
    gb, ub, db, x, g, u, d = _case(backend, t, td, hidden, inter, rows, 21)
    pair = backend.pair_gated(g, u)
    xd = torch.from_numpy(x).cuda()
    act = torch.empty(rows * inter, device="cuda")
    out = torch.empty(rows * hidden, device="cuda")
    backend.mlp_gated_silu(xd, rows, hidden, inter, pair, None, d, act, None, out)
    backend.synchronize()
    ref_act, ref_out = oracle.q_mlp_gated_silu(t, gb, ub, td, db, x, rows, hidden, inter, threads=8)
    a = act.cpu().numpy().reshape(rows, inter)
    gy = oracle.q_linear(t, gb, x, rows, hidden, inter, threads=8)
    uy = oracle.q_linear(t, ub, x, rows, hidden, inter, threads=8)
    e = gated_gemv_err(a, gy, uy)
    record_err(f"mlp_gated_silu.act.t{t}.rows{rows}", e)
    assert e <= GEMV_RTOL, e
    # the down projection alone, on the device's own act
    down_only = oracle.q_linear(td, db, a, rows, inter, hidden, threads=8)
    assert gemv_err(f"mlp_gated_silu.down.t{t}.rows{rows}", out.cpu().numpy().reshape(rows, hidden),
                    down_only) <= GEMV_RTOL
    # end to end the act error carries through down: normwise it stays at the GEMV bound
    ne = normwise_err(out.cpu().numpy().reshape(rows, hidden), ref_out)
    record_err(f"mlp_gated_silu.out_normwise.t{t}.rows{rows}", ne)
    assert ne <= GEMV_RTOL


def test_mlp_doc_example_host_slices(backend):
    """Reference doc example (mlp.rs:120-137) through the host-slice form with unpaired weights."""
    from tests.mlp_cases import doc_example
    x, gate, up, down, hidden, inter = doc_example()
    g = backend.upload_quant(8, gate, inter, hidden)
    u = backend.upload_quant(8, up, inter, hidden)
    d = backend.upload_quant(8, down, hidden, inter)
    gate_buf = np.zeros(inter, np.float32)
    out = np.zeros(hidden, np.float32)
    backend.mlp_gated_silu(x, 1, hidden, inter, g, u, d, gate_buf, None, out)
    assert np.allclose(gate_buf, 3.5231884, atol=1e-5)
    assert np.allclose(out, 3.5231884, atol=1e-5)


def test_mlp_errors(backend):
    from ocelotl_b200 import synth
    from ocelotl_b200.errors import KernelError, UnsupportedError
    g = backend.upload_quant(12, synth.quant_blocks(12, 64, 256, 1, "g"), 64, 256)
    u6 = backend.upload_quant(14, synth.quant_blocks(14, 64, 256, 1, "u"), 64, 256)
    u_wide = backend.upload_quant(12, synth.quant_blocks(12, 64, 512, 1, "u"), 64, 512)
    with pytest.raises(UnsupportedError):
        backend.pair_gated(g, u6)
    with pytest.raises(KernelError):
        backend.pair_gated(g, u_wide)
    pair = backend.pair_gated(g, g)
    x = torch.zeros(256, device="cuda")
    y = torch.zeros(64, device="cuda")
    with pytest.raises(KernelError):  # a pair is not a linear weight
        backend.linear_dev(pair, x, 1, y)
    with pytest.raises(KernelError):
        backend.mlp_gated_silu(x, 0, 256, 64, pair, None, g, y, None, x)
    with pytest.raises(KernelError):  # down must be [hidden, intermediate]
        backend.mlp_gated_silu(x, 1, 256, 64, pair, None, g, y, None, x)
