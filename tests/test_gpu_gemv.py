"""GPU: fused dequant-GEMV parity vs the CPU oracle, through the C ABI."""
import numpy as np
import pytest
import torch

from tests.tolerance import GEMV_RTOL, gemv_err, normwise_err, rel_err

pytestmark = pytest.mark.gpu

NAMES = {12: "Q4_K", 14: "Q6_K", 8: "Q8_0"}


def run_case(backend, oracle, t, n, k, rows, seed=1, bias=True, threads=8):
    from ocelotl_b200 import synth
    blocks = synth.quant_blocks(t, n, k, seed, f"w{t}")
    x = synth.activations(rows, k, seed, "x")
    b = synth.activations(1, n, seed, "b").reshape(-1) if bias else None
    w = backend.upload_quant(t, blocks, n, k)
    xd = backend.upload(x.numpy())
    out = backend.alloc(rows * n)
    bd = backend.upload(b.numpy()) if bias else None
    backend.linear_d(xd, rows, k, w, n, bd, out)
    got = out.to_host_owned().reshape(rows, n)
    ref = oracle.q_linear(t, blocks.numpy(), x.numpy(), rows, k, n,
                          bias=None if b is None else b.numpy(), threads=threads)
    return got, ref


@pytest.mark.parametrize("t", [12, 14, 8])
@pytest.mark.parametrize("rows", [1, 2, 3, 4, 5, 8, 11, 16])
def test_gemv_small_shapes(backend, oracle, t, rows):
    got, ref = run_case(backend, oracle, t, 100, 768, rows)
    e = gemv_err(f"gemv.small.{NAMES[t]}.rows{rows}", got, ref)
    assert e <= GEMV_RTOL, (NAMES[t], rows, e, normwise_err(got, ref))


@pytest.mark.parametrize("t", [12, 14, 8])
@pytest.mark.parametrize("rows", [17, 33])
def test_gemv_more_than_16_rows_is_chunked(backend, oracle, t, rows):
    got, ref = run_case(backend, oracle, t, 48, 512, rows, bias=False)
    assert rel_err(got, ref) <= GEMV_RTOL


@pytest.mark.parametrize("t,n,k", [(12, 4096, 4096), (14, 4096, 14336), (8, 1024, 4096), (12, 6144, 4096)])
@pytest.mark.parametrize("rows", [1, 16])
def test_gemv_baseline_shapes(backend, oracle, t, n, k, rows):
    got, ref = run_case(backend, oracle, t, n, k, rows, bias=False)
    e = gemv_err(f"gemv.baseline.{NAMES[t]}.{n}x{k}.rows{rows}", got, ref)
    assert e <= GEMV_RTOL, (NAMES[t], n, k, rows, e, normwise_err(got, ref))


def test_gemv_is_deterministic(backend):
    from ocelotl_b200 import synth
    n, k = 4096, 4096
    w = backend.upload_quant(12, synth.quant_blocks(12, n, k, 2, "w"), n, k)
    x = backend.upload(synth.activations(4, k, 2, "x").numpy())
    o1, o2 = backend.alloc(4 * n), backend.alloc(4 * n)
    backend.linear_d(x, 4, k, w, n, None, o1)
    backend.linear_d(x, 4, k, w, n, None, o2)
    assert torch.equal(o1.device, o2.device)


def test_linear_out_by_in_host_slices(backend, oracle):
    from ocelotl_b200 import synth
    n, k, rows = 200, 1024, 3
    blocks = synth.quant_blocks(14, n, k, 4, "w")
    x = synth.activations(rows, k, 4, "x").numpy()
    b = synth.activations(1, n, 4, "b").numpy().reshape(-1)
    w = backend.upload_quant(14, blocks, n, k)
    out = np.zeros(rows * n, np.float32)
    backend.linear_out_by_in(x, rows, k, w, n, b, out)
    ref = oracle.q_linear(14, blocks.numpy(), x, rows, k, n, bias=b)
    assert rel_err(out.reshape(rows, n), ref) <= GEMV_RTOL


def test_zero_and_large_activations(backend, oracle):
    from ocelotl_b200 import synth
    n, k = 64, 512
    blocks = synth.quant_blocks(12, n, k, 6, "w")
    w = backend.upload_quant(12, blocks, n, k)
    x = np.zeros((2, k), np.float32)
    x[1, :256] = 0.0
    x[1, 256:] = np.linspace(-3e4, 3e4, 256, dtype=np.float32)  # one block zero, one block large
    out = backend.alloc(2 * n)
    backend.linear_d(backend.upload(x), 2, k, w, n, None, out)
    got = out.to_host_owned().reshape(2, n)
    ref = oracle.q_linear(12, blocks.numpy(), x, 2, k, n)
    assert not got[0].any()
    assert rel_err(got[1], ref[1]) <= GEMV_RTOL


def test_nonfinite_activation_propagates(backend):
    from ocelotl_b200 import synth
    n, k = 32, 256
    w = backend.upload_quant(8, synth.quant_blocks(8, n, k, 1, "w"), n, k)
    x = np.ones((1, k), np.float32)
    x[0, 7] = np.inf
    out = backend.alloc(n)
    backend.linear_d(backend.upload(x), 1, k, w, n, None, out)
    assert not np.isfinite(out.to_host_owned()).any()


def test_shape_errors_are_kernel_errors(backend):
    from ocelotl_b200 import KernelError, synth
    n, k = 32, 256
    w = backend.upload_quant(12, synth.quant_blocks(12, n, k, 1, "w"), n, k)
    x = backend.alloc(k)
    with pytest.raises(KernelError) as e:
        backend.linear_d(x, 1, k, w, n, None, backend.alloc(n - 1))
    assert "out.len()" in str(e.value) and e.value.backend == "cuda-sm100a"
    with pytest.raises(KernelError):
        backend.linear_d(x, 1, k, w, n + 1, None, backend.alloc(n + 1))
    with pytest.raises(KernelError):
        backend.linear_d(x, 2, k, w, n, None, backend.alloc(2 * n))


def test_unsupported_before_launch(backend):
    from ocelotl_b200 import UnsupportedError
    with pytest.raises(UnsupportedError):
        backend.upload_quant(2, np.zeros(18, np.uint8), 1, 32)   # Q4_0 is not supported
    with pytest.raises(UnsupportedError):
        backend.upload_quant(12, np.zeros(144, np.uint8), 1, 300)  # K % 256 != 0
    with pytest.raises(UnsupportedError):
        backend.linear_d(backend.alloc(4), 1, 4, backend.alloc(4), 1, None, backend.alloc(1))  # f32 weight


@pytest.mark.parametrize("t,n,k", [(12, 1000, 2560), (14, 3000, 768), (8, 1000, 1184), (8, 4099, 4096),
                                   (12, 37, 65536), (14, 150, 2048)])
def test_gemv_single_row_balanced_ranges(backend, oracle, t, n, k):
    """Single row: record ranges cut row tiles across warps and CTAs (ragged n, k, bias)."""
    got, ref = run_case(backend, oracle, t, n, k, 1, seed=9)
    e = gemv_err(f"gemv.ragged.{NAMES[t]}.{n}x{k}", got, ref)
    assert e <= GEMV_RTOL, (NAMES[t], n, k, e, normwise_err(got, ref))
    assert backend.take_device_errors() == (0, 0)


def test_gemv_single_row_is_deterministic(backend):
    from ocelotl_b200 import synth
    n, k = 14336, 4096
    w = backend.upload_quant(12, synth.quant_blocks(12, n, k, 2, "w"), n, k)
    x = backend.upload(synth.activations(1, k, 2, "x").numpy())
    outs = [backend.alloc(n) for _ in range(3)]
    for o in outs:
        backend.linear_d(x, 1, k, w, n, None, o)
    assert torch.equal(outs[0].device, outs[1].device) and torch.equal(outs[0].device, outs[2].device)


@pytest.mark.parametrize("pinned", [False, True])
@pytest.mark.parametrize("rows", [1, 3, 20])
def test_linear_out_by_in_pinned_and_pageable(backend, oracle, pinned, rows):
    """Host-slice form: pinned buffers are used by the kernels in place, pageable ones are staged."""
    from ocelotl_b200 import synth
    n, k = 300, 1024
    blocks = synth.quant_blocks(12, n, k, 8, "w")
    w = backend.upload_quant(12, blocks, n, k)
    x = synth.activations(rows, k, 8, "x")
    b = synth.activations(1, n, 8, "b").reshape(-1)
    out = torch.zeros(rows * n)
    if pinned:
        x, b, out = x.pin_memory(), b.pin_memory(), out.pin_memory()
    backend.linear_out_by_in(x.numpy(), rows, k, w, n, b.numpy(), out.numpy())
    ref = oracle.q_linear(12, blocks.numpy(), x.numpy(), rows, k, n, bias=b.numpy())
    assert rel_err(out.numpy().reshape(rows, n), ref) <= GEMV_RTOL


def test_unaligned_activation_rows(backend, oracle):
    """x that starts 4 bytes past a 16-byte boundary (a view into a larger tensor)."""
    from ocelotl_b200 import synth
    n, k, rows = 256, 1024, 2
    blocks = synth.quant_blocks(14, n, k, 4, "w")
    w = backend.upload_quant(14, blocks, n, k)
    xs = synth.activations(rows, k, 4, "x")
    big = torch.zeros(rows * k + 1, device="cuda")
    big[1:] = xs.reshape(-1).cuda()
    x = big[1:]
    assert x.data_ptr() % 16 == 4
    for m in (1, rows):
        y = torch.empty(m, n, device="cuda")
        backend.linear_dev(w, x, m, y)
        backend.synchronize()
        ref = oracle.q_linear(14, blocks.numpy(), xs[:m].numpy(), m, k, n)
        assert rel_err(y.cpu().numpy(), ref) <= GEMV_RTOL

