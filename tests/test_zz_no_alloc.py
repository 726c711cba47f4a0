"""GPU: the allocation-free linear entry point, ocl_q_linear_noalloc.

Some callers cannot allocate GPU memory while they run: a plugin hosted inside
another engine's memory pool, code under a fixed memory budget, or a hot loop
that must never hit cudaMalloc (which may synchronise the device).  For them the
library offers ocl_q_linear_noalloc, which takes its scratch from a static
device array instead.  These tests call it through the C ABI and check that it
gives bit-identical results to ocl_q_linear (same kernels, same launch plan),
on consecutive calls that reuse the array, that no bounded wait gave up (its
counter lives in the same array and is read with
ocl_noalloc_take_device_errors), and that it refuses shapes beyond the array's
limit and a stream of another device.  The file is named so pytest collects it
last.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from tests.tolerance import GEMV_RTOL, rel_err

pytestmark = pytest.mark.gpu


def _noalloc(backend, w, x, rows, y, bias=None):
    lib = backend._lib
    q = w.quant
    return lib.ocl_q_linear_noalloc(int(q.ggml_type), C.c_void_p(q.device_ptr()), q.n_rows, q.k,
                                    C.c_void_p(x.data_ptr()), rows,
                                    C.c_void_p(bias.data_ptr()) if bias is not None else None,
                                    C.c_void_p(y.data_ptr()), None)


@pytest.mark.parametrize("t,n,k,rows", [(12, 4096, 4096, 1), (14, 4096, 14336, 3), (8, 1000, 4096, 17),
                                        (12, 320, 2048, 2)])
def test_noalloc_matches_linear_twice(backend, t, n, k, rows):
    from ocelotl_b200 import synth
    w = backend.upload_quant(t, synth.quant_blocks(t, n, k, 21, f"na{t}", device="cuda"), n, k)
    bias = synth.activations(1, n, 21, "na.b", device="cuda").reshape(-1).contiguous()
    for call in range(2):  # the second call sees the first call's leftovers in the static scratch
        x = synth.activations(rows, k, 100 + call, "na.x", device="cuda").contiguous()
        ref = torch.empty(rows, n, device="cuda")
        got = torch.full((rows, n), float("nan"), device="cuda")
        backend.linear_dev(w, x, rows, ref, bias)
        torch.cuda.synchronize()
        assert _noalloc(backend, w, x, rows, got, bias) == 0, backend._lib.ocl_last_error(None)
        torch.cuda.synchronize()
        g, r = got.cpu().numpy(), ref.cpu().numpy()
        assert np.isfinite(g).all()
        assert rel_err(g, r) <= GEMV_RTOL
        assert torch.equal(got, ref)  # same kernels and plan: the same bits
        tmo = C.c_uint(7)
        assert backend._lib.ocl_noalloc_take_device_errors(None, C.byref(tmo)) == 0
        assert tmo.value == 0


def test_noalloc_rejects_beyond_limit(backend):
    from ocelotl_b200 import synth
    n, k = 16, 16640  # in_features above the static scratch's 16384
    w = backend.upload_quant(12, synth.quant_blocks(12, n, k, 3, "big", device="cuda"), n, k)
    x = torch.zeros(1, k, device="cuda")
    y = torch.zeros(1, n, device="cuda")
    rc = _noalloc(backend, w, x, 1, y)
    assert rc == -2  # OCL_ERR_UNSUPPORTED, before any launch
    assert "16384" in backend._lib.ocl_last_error(None).decode()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_noalloc_rejects_a_stream_of_another_device(backend):
    from ocelotl_b200 import synth
    n, k = 64, 256
    w = backend.upload_quant(12, synth.quant_blocks(12, n, k, 3, "dev", device="cuda"), n, k)
    x = torch.zeros(1, k, device="cuda")
    y = torch.zeros(1, n, device="cuda")
    other = torch.cuda.Stream(device=1)
    q = w.quant
    rc = backend._lib.ocl_q_linear_noalloc(int(q.ggml_type), C.c_void_p(q.device_ptr()), n, k,
                                           C.c_void_p(x.data_ptr()), 1, None, C.c_void_p(y.data_ptr()),
                                           C.c_void_p(other.cuda_stream))
    assert rc == -1  # OCL_ERR_INVALID, before any launch
    assert "stream" in backend._lib.ocl_last_error(None).decode()
