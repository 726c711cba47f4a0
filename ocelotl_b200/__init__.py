"""ocelotl_b200: B200 (sm_100a) backend for Ocelotl's GGUF-quantized linear path.

Fused Q4_K / Q6_K / Q8_0 dequantize-and-multiply behind the reference's
`KernelBackend` boundary (crates/kernels/src/lib.rs:84-495).  Kernels are
hand-written CUDA in csrc/, exposed through the C ABI in include/ocelotl_cuda.h;
`CudaKernelBackend` is the host-side mirror of the reference's trait.
"""
from .errors import InvalidRequestError, KernelError, OcelotlError, UnsupportedError  # noqa: F401
from .ggml import GgmlType, byte_len  # noqa: F401


def __getattr__(name):
    # the backend pulls in torch + the CUDA library; import it lazily
    if name in ("CudaKernelBackend", "DeviceTensor", "QuantBuffer"):
        from . import backend
        return getattr(backend, name)
    raise AttributeError(name)
