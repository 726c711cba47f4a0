"""GPU: prefill GEMM (tcgen05, bf16 x dequantized bf16 -> f32 accumulate -> bf16).

Reference: the bit-exact dequantized weight (checked against the oracle in
test_gpu_dequant) times the bf16-rounded activations, in f32 with torch -- the
plain fp32 reference of the same op.  Tolerance 2e-2 (tests/tolerance.py).
"""
import pytest
import torch

from tests.tolerance import GEMM_FLOOR, GEMM_RTOL, gated_rel_err, normwise_err, rel_err

pytestmark = pytest.mark.gpu


def run(backend, t, n, k, rows, seed=3):
    from ocelotl_b200 import synth
    w = backend.upload_quant(t, synth.quant_blocks(t, n, k, seed, f"g{t}", device="cuda"), n, k)
    x = synth.activations(rows, k, seed, "gx", device="cuda", dtype=torch.bfloat16).contiguous()
    y = backend.gemm_bf16(x, w)
    torch.cuda.synchronize()
    ref = x.float() @ backend.dequant(w.quant).t()
    assert backend.take_device_errors() == (0, 0)
    return y.float().cpu().numpy(), ref.cpu().numpy()


@pytest.mark.parametrize("t", [12, 14, 8])
@pytest.mark.parametrize("n,k,rows", [(128, 256, 128), (256, 1024, 256), (100, 768, 200), (384, 512, 64)])
def test_gemm_small(backend, t, n, k, rows):
    got, ref = run(backend, t, n, k, rows)
    e = rel_err(got, ref, floor=GEMM_FLOOR)
    assert e <= GEMM_RTOL, (e, normwise_err(got, ref))


@pytest.mark.parametrize("t,n,k,rows", [(12, 4096, 4096, 512), (14, 4096, 14336, 512), (12, 14336, 4096, 2048)])
def test_gemm_baseline_shapes(backend, t, n, k, rows):
    got, ref = run(backend, t, n, k, rows)
    e = rel_err(got, ref, floor=GEMM_FLOOR)
    assert e <= GEMM_RTOL, (e, normwise_err(got, ref))


def test_gemm_rejects_unaligned_k(backend):
    from ocelotl_b200 import UnsupportedError, synth
    w = backend.upload_quant(8, synth.quant_blocks(8, 32, 96, 1, "q8"), 32, 96)
    x = torch.zeros(64, 96, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(UnsupportedError):
        backend.gemm_bf16(x, w)


@pytest.mark.parametrize("t", [12, 14, 8])
@pytest.mark.parametrize("inter,k,rows", [(128, 256, 128), (200, 1024, 300), (14336, 4096, 512)])
def test_gemm_gated(backend, t, inter, k, rows):
    """Prefill gate+up over an interleaved pair with silu * up on the accumulators."""
    from ocelotl_b200 import synth
    g = backend.upload_quant(t, synth.quant_blocks(t, inter, k, 4, "gg", device="cuda"), inter, k)
    u = backend.upload_quant(t, synth.quant_blocks(t, inter, k, 4, "gu", device="cuda"), inter, k)
    pair = backend.pair_gated(g, u)
    x = synth.activations(rows, k, 4, "gx", device="cuda", dtype=torch.bfloat16).contiguous()
    act = backend.gemm_gated_bf16(pair, x)
    torch.cuda.synchronize()
    xf = x.float()
    gy, uy = xf @ backend.dequant(g.quant).t(), xf @ backend.dequant(u.quant).t()
    ref = (gy * torch.sigmoid(gy) * uy).cpu().numpy()
    assert backend.take_device_errors() == (0, 0)
    got = act.float().cpu().numpy()
    e = gated_rel_err(got, gy.cpu().numpy(), uy.cpu().numpy())
    assert e <= GEMM_RTOL, (e, normwise_err(got, ref))
