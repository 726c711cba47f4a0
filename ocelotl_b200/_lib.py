"""ctypes binding of libocelotl_cuda.so (the C ABI in include/ocelotl_cuda.h).

The library is built in-tree by ocelotl_b200/build.py.  There is no fallback:
if it is missing, `load()` raises, so a GPU run can never silently take a CPU
path.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libocelotl_cuda.so"

OCL_OK = 0
OCL_ERR_INVALID = -1
OCL_ERR_UNSUPPORTED = -2
OCL_ERR_CUDA = -3
OCL_ERR_OOM = -4
OCL_ERR_TIMEOUT = -5

_vp = C.c_void_p
_sz = C.c_size_t

# name -> (restype, argtypes); every symbol include/ocelotl_cuda.h declares.
SIGNATURES = {
    "ocl_cuda_init": (C.c_int, [C.c_int, C.POINTER(_vp)]),
    "ocl_cuda_destroy": (None, [_vp]),
    "ocl_last_error": (C.c_char_p, [_vp]),
    "ocl_set_stream": (C.c_int, [_vp, _vp]),
    "ocl_synchronize": (C.c_int, [_vp]),
    "ocl_set_pdl": (C.c_int, [_vp, C.c_int]),
    "ocl_set_gemm_min_rows": (C.c_int, [_vp, _sz]),
    "ocl_backend_id": (C.c_char_p, []),
    "ocl_abi_version": (C.c_int, []),
    "ocl_q_upload": (C.c_int, [_vp, C.c_int, _vp, _sz, _sz, C.c_int, C.POINTER(_vp)]),
    "ocl_q_upload_device": (C.c_int, [_vp, C.c_int, _vp, _sz, _sz, C.POINTER(_vp)]),
    "ocl_q_free": (C.c_int, [_vp]),
    "ocl_q_info": (C.c_int, [_vp, C.POINTER(C.c_int), C.POINTER(_sz), C.POINTER(_sz), C.POINTER(_sz)]),
    "ocl_q_device_ptr": (_vp, [_vp]),
    "ocl_q_dequant": (C.c_int, [_vp, _vp, _vp]),
    "ocl_q_download_gguf": (C.c_int, [_vp, _vp, _vp]),
    "ocl_q_linear": (C.c_int, [_vp, _vp, _vp, _sz, _sz, _sz, _vp, _vp]),
    "ocl_q_linear_noalloc": (C.c_int, [C.c_int, _vp, _sz, _sz, _vp, _sz, _vp, _vp, _vp]),
    "ocl_tp_comm_create": (C.c_int, [_vp, C.c_int, C.c_int, _sz, _sz, C.POINTER(_vp), _vp]),
    "ocl_tp_comm_open": (C.c_int, [_vp, _vp, _vp]),
    "ocl_tp_comm_destroy": (C.c_int, [_vp]),
    "ocl_tp_comm_packets": (_vp, [_vp]),
    "ocl_noalloc_take_device_errors": (C.c_int, [_vp, C.POINTER(C.c_uint)]),
    "ocl_q_linear_allreduce": (C.c_int, [_vp, _vp, _vp, _vp, _sz, _sz, _sz, _vp, _vp]),
    "ocl_q_linear_host": (C.c_int, [_vp, _vp, _vp, _sz, _sz, _sz, _vp, _vp]),
    "ocl_q_gemm_bf16": (C.c_int, [_vp, _vp, _vp, _sz, _sz, _sz, _vp]),
    "ocl_q_pair_gated": (C.c_int, [_vp, _vp, _vp, C.POINTER(_vp)]),
    "ocl_q_linear_gated": (C.c_int, [_vp, _vp, _vp, _sz, _sz, _sz, _vp]),
    "ocl_q_mlp_gated_silu": (C.c_int, [_vp, _vp, _vp, _vp, _sz, _sz, _sz, _vp, _vp]),
    "ocl_q_gemm_gated_bf16": (C.c_int, [_vp, _vp, _vp, _sz, _sz, _sz, _vp]),
    "ocl_argmax_f32": (C.c_int, [_vp, _vp, _sz, _sz, _vp]),
    "ocl_q_embed_rows": (C.c_int, [_vp, _vp, _vp, _sz, _vp]),
    "ocl_take_device_errors": (C.c_int, [_vp, C.POINTER(C.c_uint), C.POINTER(C.c_uint)]),
}

_lib = None


def load() -> C.CDLL:
    """Load the library (once) and attach signatures.  Raises if it is absent."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m ocelotl_b200.build` "
                "(the quantized path has no CPU fallback)")
        lib = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib
