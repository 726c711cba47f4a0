"""CPU: the C-ABI library loads and exports exactly what include/ocelotl_cuda.h declares.

No compute is called (there is no GPU here); only symbol presence and the
ctypes signature table are checked, plus the error path of ocl_cuda_init on a
machine without a CUDA device.
"""
import ctypes as C
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "ocelotl_cuda.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"OCL_API\s+[\w\s\*]+?\b(ocl_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from ocelotl_b200.build import build
    build()
    from ocelotl_b200 import _lib
    return _lib.load()


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert "ocl_q_linear" in syms and "ocl_q_upload" in syms and "ocl_q_linear_noalloc" in syms
    assert len(syms) >= 20


def test_library_exports_every_declared_symbol(lib):
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, missing


def test_ctypes_table_matches_header():
    from ocelotl_b200 import _lib
    assert sorted(_lib.SIGNATURES) == declared_symbols()


def test_backend_id_and_abi_version(lib):
    assert lib.ocl_backend_id() == b"cuda-sm100a"
    assert lib.ocl_abi_version() == 1


def test_init_without_gpu_fails_cleanly(lib):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    ctx = C.c_void_p()
    rc = lib.ocl_cuda_init(0, C.byref(ctx))
    assert rc != 0 and not ctx.value
    assert lib.ocl_last_error(None)


def test_unsupported_noalloc_rejected_before_any_cuda_call(lib):
    # K not a multiple of the block size: refused on the host, no device touched
    rc = lib.ocl_q_linear_noalloc(12, C.c_void_p(16), 16, 300, C.c_void_p(16), 1, None, C.c_void_p(16), None)
    assert rc == -2
    assert b"in_features" in lib.ocl_last_error(None)
