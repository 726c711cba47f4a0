"""Host-side mirror of the reference's `KernelBackend` for quantized weights.

`CudaKernelBackend` is what `ocelotl-kernels` would register as its CUDA backend
(crates/kernels/src/lib.rs:84-495): the same method names, argument meaning and
error behaviour, for a weight that is a resident GGUF-quantized tensor.  All
compute goes through the C ABI in include/ocelotl_cuda.h (libocelotl_cuda.so);
torch is used only to own device memory and streams.

Reference interfaces mirrored:
  * linear_out_by_in (host slices)    crates/kernels/src/lib.rs:107-116, 1939-1967
  * linear_d (device-resident)        crates/kernels/src/lib.rs:193-217
  * upload / alloc                    crates/kernels/src/lib.rs:176-184
  * DeviceTensor / DeviceBuffer       crates/kernels/src/tensor.rs:45-268
  * shape validation messages         crates/kernels/src/lib.rs:2443-2494
  * downcast of the weight buffer     crates/kernels/src/cubecl_backend.rs:245-293, 2413-2439
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from .errors import KernelError, UnsupportedError
from .ggml import GgmlType, byte_len, geometry

BACKEND_ID = "cuda-sm100a"


def _kernel_err(message: str) -> KernelError:
    return KernelError(BACKEND_ID, message)


class QuantBuffer:
    """A GGUF-quantized weight resident in HBM (the CUDA `DeviceBuffer`).

    `len_f32()` is the logical element count (n_rows * k) so the reference's
    length checks hold; `to_host()` returns the dequantized f32 values, so the
    trait's default readback path stays correct; `write_from_host` is
    unsupported for quantized buffers.
    """

    def __init__(self, backend: "CudaKernelBackend", handle: int, ggml_type: int, n_rows: int, k: int,
                 gated: bool = False):
        self._backend = backend
        self._handle = C.c_void_p(handle)
        self.ggml_type = GgmlType(ggml_type)
        self.n_rows = n_rows
        self.k = k
        self.gated = gated  # interleaved gate/up pair (n_rows each); only the gated-MLP calls take it

    # DeviceBuffer surface -------------------------------------------------
    def backend_id(self) -> str:
        return BACKEND_ID

    def len_f32(self) -> int:
        return (2 if self.gated else 1) * self.n_rows * self.k

    def to_host(self) -> np.ndarray:
        return self._backend.dequant(self).cpu().numpy().reshape(-1)

    def write_from_host(self, src) -> None:
        raise UnsupportedError("write_from_host on a quantized buffer", self.ggml_type.name, ["f32 buffers"])

    # extras -----------------------------------------------------------------
    @property
    def handle(self) -> C.c_void_p:
        if not self._handle:
            raise _kernel_err("quantized buffer used after free")
        return self._handle

    def device_bytes(self) -> int:
        n = C.c_size_t()
        self._backend._lib.ocl_q_info(self.handle, None, None, None, C.byref(n))
        return n.value

    def device_ptr(self) -> int:
        return self._backend._lib.ocl_q_device_ptr(self.handle)

    def to_gguf(self) -> np.ndarray:
        """The weight written back out as GGUF blocks (layout round trip)."""
        out = np.empty(byte_len(self.ggml_type, self.n_rows, self.k), dtype=np.uint8)
        self._backend._check(self._backend._lib.ocl_q_download_gguf(
            self._backend._ctx, self.handle, out.ctypes.data_as(C.c_void_p)))
        return out

    def free(self) -> None:
        if self._handle:
            self._backend._lib.ocl_q_free(self._handle)
            self._handle = C.c_void_p()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


@dataclass
class DeviceTensor:
    """f32 tensor on host (`numpy`) or device (`torch`, cuda), or a quantized weight."""

    host: np.ndarray | None = None
    device: torch.Tensor | None = None
    quant: QuantBuffer | None = None

    @staticmethod
    def from_host(v) -> "DeviceTensor":
        return DeviceTensor(host=np.ascontiguousarray(v, dtype=np.float32).reshape(-1))

    def len_f32(self) -> int:
        if self.quant is not None:
            return self.quant.len_f32()
        if self.device is not None:
            return self.device.numel()
        return int(self.host.size)

    def to_host_owned(self) -> np.ndarray:
        if self.quant is not None:
            return self.quant.to_host()
        if self.device is not None:
            return self.device.detach().cpu().numpy().reshape(-1).copy()
        return self.host.copy()

    def write_from_host_slice(self, src) -> None:
        src = np.ascontiguousarray(src, dtype=np.float32).reshape(-1)
        if src.size != self.len_f32():
            raise _kernel_err(f"write_from_host len {src.size} does not match buffer len {self.len_f32()}")
        if self.quant is not None:
            self.quant.write_from_host(src)
        elif self.device is not None:
            self.device.copy_(torch.from_numpy(src).view(self.device.shape))
        else:
            self.host[:] = src

    def try_as_device_buffer(self):
        if self.quant is not None:
            return self.quant
        if self.device is not None:
            return self.device
        raise _kernel_err("tensor is host-resident; expected a device buffer")


class CudaKernelBackend:
    """The B200 (sm_100a) backend for GGUF-quantized linear layers."""

    def __init__(self, device: int = 0):
        self._lib = _lib.load()
        ctx = C.c_void_p()
        rc = self._lib.ocl_cuda_init(device, C.byref(ctx))
        if rc != _lib.OCL_OK:
            msg = self._lib.ocl_last_error(None).decode()
            raise (UnsupportedError("device", message=msg) if rc == _lib.OCL_ERR_UNSUPPORTED else _kernel_err(msg))
        self._ctx = ctx
        self.device_index = device
        self.torch_device = torch.device("cuda", device)

    def __del__(self):
        try:
            if self._ctx:
                self._lib.ocl_cuda_destroy(self._ctx)
                self._ctx = C.c_void_p()
        except Exception:
            pass

    # -- plumbing -------------------------------------------------------------
    def name(self) -> str:
        return BACKEND_ID

    def cpu_thread_pool(self):
        return None

    def _check(self, rc: int) -> None:
        if rc == _lib.OCL_OK:
            return
        msg = self._lib.ocl_last_error(self._ctx).decode()
        if rc == _lib.OCL_ERR_UNSUPPORTED:
            raise UnsupportedError("", message=msg)
        raise _kernel_err(msg)

    def set_stream(self, stream: torch.cuda.Stream | None) -> None:
        self._check(self._lib.ocl_set_stream(self._ctx, C.c_void_p(stream.cuda_stream if stream else 0)))

    def use_current_stream(self) -> None:
        """Launch on torch's current stream of this device."""
        self.set_stream(torch.cuda.current_stream(self.torch_device))

    def synchronize(self) -> None:
        self._check(self._lib.ocl_synchronize(self._ctx))

    # -- tensors --------------------------------------------------------------
    def upload(self, host) -> DeviceTensor:
        a = np.ascontiguousarray(host, dtype=np.float32).reshape(-1)
        return DeviceTensor(device=torch.from_numpy(a).to(self.torch_device))

    def alloc(self, length: int) -> DeviceTensor:
        return DeviceTensor(device=torch.zeros(length, dtype=torch.float32, device=self.torch_device))

    def upload_quant(self, ggml_type: int, blocks, n_rows: int, k: int) -> DeviceTensor:
        """Upload GGUF blocks (host bytes / numpy uint8 / torch uint8 on host or this device)."""
        geometry(ggml_type)  # Unsupported before anything else
        expected = byte_len(ggml_type, n_rows, k)
        h = C.c_void_p()
        if isinstance(blocks, torch.Tensor) and blocks.is_cuda:
            if blocks.dtype != torch.uint8 or not blocks.is_contiguous() or blocks.numel() != expected:
                raise _kernel_err(f"upload_quant blocks must be {expected} contiguous uint8 bytes")
            self._check(self._lib.ocl_q_upload_device(self._ctx, int(ggml_type), C.c_void_p(blocks.data_ptr()),
                                                      n_rows, k, C.byref(h)))
        else:
            if isinstance(blocks, torch.Tensor):
                blocks = blocks.numpy()
            arr = np.frombuffer(blocks, dtype=np.uint8) if isinstance(blocks, (bytes, bytearray)) else \
                np.ascontiguousarray(blocks, dtype=np.uint8).reshape(-1)
            if arr.size != expected:
                raise _kernel_err(f"upload_quant blocks len {arr.size} does not match {GgmlType(ggml_type).name} "
                                  f"[{n_rows}, {k}] = {expected} bytes")
            self._check(self._lib.ocl_q_upload(self._ctx, int(ggml_type), arr.ctypes.data_as(C.c_void_p),
                                               n_rows, k, 0, C.byref(h)))
        return DeviceTensor(quant=QuantBuffer(self, h.value, ggml_type, n_rows, k))

    def dequant(self, w: QuantBuffer) -> torch.Tensor:
        out = torch.empty(w.n_rows, w.k, dtype=torch.float32, device=self.torch_device)
        self._check(self._lib.ocl_q_dequant(self._ctx, w.handle, C.c_void_p(out.data_ptr())))
        self.synchronize()
        return out

    # -- validation (crates/kernels/src/lib.rs:2443-2494) ----------------------
    @staticmethod
    def _validate(x_len, rows, in_features, w_len, out_features, bias_len, out_len, op="linear_out_by_in"):
        if x_len != rows * in_features:
            raise _kernel_err(f"{op} x.len()={x_len} does not match rows*in_features="
                              f"{rows}*{in_features}={rows * in_features}")
        if w_len != out_features * in_features:
            raise _kernel_err(f"{op} weight.len()={w_len} does not match out_features*in_features="
                              f"{out_features}*{in_features}={out_features * in_features}")
        if bias_len is not None and bias_len != out_features:
            raise _kernel_err(f"{op} bias.len()={bias_len} does not match out_features={out_features}")
        if out_len != rows * out_features:
            raise _kernel_err(f"{op} out.len()={out_len} does not match rows*out_features="
                              f"{rows}*{out_features}={rows * out_features}")

    @staticmethod
    def _quant_weight(weight) -> QuantBuffer:
        q = weight.quant if isinstance(weight, DeviceTensor) else weight
        if not isinstance(q, QuantBuffer):
            raise UnsupportedError("linear weight dtype", "f32", ["Q4_K", "Q6_K", "Q8_0 device buffers"])
        return q

    # -- the hot path -----------------------------------------------------------
    def linear_d(self, x: DeviceTensor, rows: int, in_features: int, weight: DeviceTensor, out_features: int,
                 bias: DeviceTensor | None, out: DeviceTensor) -> None:
        """Device-resident quantized linear: out = x . W^T (+ bias), all on this device."""
        w = self._quant_weight(weight)
        self._validate(x.len_f32(), rows, in_features, w.len_f32(), out_features,
                       None if bias is None else bias.len_f32(), out.len_f32(), op="linear_d")
        xd, od = x.try_as_device_buffer(), out.try_as_device_buffer()
        bd = None if bias is None else bias.try_as_device_buffer()
        for t in (xd, od) + ((bd,) if bd is not None else ()):
            if not isinstance(t, torch.Tensor) or t.dtype != torch.float32 or not t.is_contiguous() \
                    or t.device != self.torch_device:
                raise _kernel_err("linear_d operands must be contiguous f32 tensors on " + str(self.torch_device))
        self._check(self._lib.ocl_q_linear(self._ctx, w.handle, C.c_void_p(xd.data_ptr()), rows, in_features,
                                           out_features, C.c_void_p(bd.data_ptr()) if bd is not None else None,
                                           C.c_void_p(od.data_ptr())))

    def linear_out_by_in(self, x, rows: int, in_features: int, weight, out_features: int, bias, out) -> None:
        """Host-slice form: x, bias, out are host f32 arrays; weight is resident."""
        w = self._quant_weight(weight)
        x = np.ascontiguousarray(x, dtype=np.float32)
        if not (isinstance(out, np.ndarray) and out.dtype == np.float32 and out.flags.c_contiguous):
            raise _kernel_err("linear_out_by_in out must be a contiguous f32 numpy array")
        b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
        self._validate(x.size, rows, in_features, w.len_f32(), out_features, None if b is None else b.size,
                       out.size)
        # raw addresses: the argtypes are void*, and ndarray.ctypes.data_as costs microseconds a call
        rc = self._lib.ocl_q_linear_host(
            self._ctx, w.handle, x.__array_interface__["data"][0], rows, in_features, out_features,
            b.__array_interface__["data"][0] if b is not None else None, out.__array_interface__["data"][0])
        if rc:
            self._check(rc)

    def gemm_bf16(self, x: torch.Tensor, weight, out: torch.Tensor | None = None) -> torch.Tensor:
        """Prefill: bf16 [rows, in] . W^T -> bf16 [rows, out] on tcgen05 tensor cores."""
        w = self._quant_weight(weight)
        if x.dtype != torch.bfloat16 or x.dim() != 2 or not x.is_contiguous() or x.device != self.torch_device:
            raise _kernel_err("gemm_bf16 x must be a contiguous 2-D bf16 tensor on " + str(self.torch_device))
        rows, in_features = x.shape
        if out is None:
            out = torch.empty(rows, w.n_rows, dtype=torch.bfloat16, device=self.torch_device)
        if tuple(out.shape) != (rows, w.n_rows) or out.dtype != torch.bfloat16 or not out.is_contiguous():
            raise _kernel_err(f"gemm_bf16 out must be a contiguous bf16 [{rows}, {w.n_rows}] tensor")
        self._check(self._lib.ocl_q_gemm_bf16(self._ctx, w.handle, C.c_void_p(x.data_ptr()), rows, in_features,
                                              w.n_rows, C.c_void_p(out.data_ptr())))
        return out

    def embed_rows(self, table, ids: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """Q8_0 embedding gather of rows `ids` (int32 on this device) -> f32 [len(ids), k]."""
        w = self._quant_weight(table)
        if ids.dtype != torch.int32 or not ids.is_contiguous() or ids.device != self.torch_device:
            raise _kernel_err("embed_rows ids must be a contiguous int32 tensor on " + str(self.torch_device))
        if out is None:
            out = torch.empty(ids.numel(), w.k, dtype=torch.float32, device=self.torch_device)
        self._check(self._lib.ocl_q_embed_rows(self._ctx, w.handle, C.c_void_p(ids.data_ptr()), ids.numel(),
                                               C.c_void_p(out.data_ptr())))
        return out

    def take_device_errors(self) -> tuple[int, int]:
        """(out-of-range embedding ids, device waits that timed out) since the last call.

        The C call also returns OCL_ERR_TIMEOUT when waits timed out; here the
        counts are returned either way (check_device_errors raises instead).
        """
        bad, tmo = C.c_uint(), C.c_uint()
        rc = self._lib.ocl_take_device_errors(self._ctx, C.byref(bad), C.byref(tmo))
        if rc != _lib.OCL_ERR_TIMEOUT:
            self._check(rc)
        return bad.value, tmo.value

    def check_device_errors(self) -> None:
        """Raise KernelError if a bounded device wait gave up since the last check."""
        bad, tmo = C.c_uint(), C.c_uint()
        self._check(self._lib.ocl_take_device_errors(self._ctx, C.byref(bad), C.byref(tmo)))

    def take_bad_ids(self) -> int:
        return self.take_device_errors()[0]

    def linear_allreduce(self, comm, weight, x: torch.Tensor, rows: int, out: torch.Tensor,
                         bias: torch.Tensor | None = None) -> None:
        """Row-split linear with the cross-rank sum fused into the GEMV (see ocelotl_b200.tp.TPComm)."""
        w = self._quant_weight(weight)
        self._check(self._lib.ocl_q_linear_allreduce(
            self._ctx, comm.handle, w.handle, C.c_void_p(x.data_ptr()), rows, w.k, w.n_rows,
            C.c_void_p(bias.data_ptr()) if bias is not None else None, C.c_void_p(out.data_ptr())))

    def set_gemm_min_rows(self, rows: int) -> None:
        """Rows at which linear_d switches to the bf16 tcgen05 GEMM (2e-2 bound); 0 = never."""
        self._check(self._lib.ocl_set_gemm_min_rows(self._ctx, rows))

    def set_pdl(self, enable: bool) -> None:
        self._check(self._lib.ocl_set_pdl(self._ctx, 1 if enable else 0))

    def linear_dev(self, weight, x: torch.Tensor, rows: int, out: torch.Tensor,
                   bias: torch.Tensor | None = None) -> None:
        """linear_d on raw contiguous f32 torch tensors of this device (no checks beyond the C ABI's)."""
        w = self._quant_weight(weight)
        self._check(self._lib.ocl_q_linear(self._ctx, w.handle, C.c_void_p(x.data_ptr()), rows, w.k, w.n_rows,
                                           C.c_void_p(bias.data_ptr()) if bias is not None else None,
                                           C.c_void_p(out.data_ptr())))

    # -- fused gated MLP (crates/kernels/src/mlp.rs:139-240) ---------------------
    def pair_gated(self, gate, up) -> DeviceTensor:
        """Interleave a gate and an up weight (same type and shape) into one pair buffer."""
        g, u = self._quant_weight(gate), self._quant_weight(up)
        h = C.c_void_p()
        self._check(self._lib.ocl_q_pair_gated(self._ctx, g.handle, u.handle, C.byref(h)))
        return DeviceTensor(quant=QuantBuffer(self, h.value, g.ggml_type, g.n_rows, g.k, gated=True))

    def linear_gated(self, gate_up, x: torch.Tensor, rows: int, act: torch.Tensor) -> None:
        """act [rows, intermediate] = silu(x . gate^T) * (x . up^T), one pass over the pair."""
        w = self._quant_weight(gate_up)
        self._check(self._lib.ocl_q_linear_gated(self._ctx, w.handle, C.c_void_p(x.data_ptr()), rows, w.k,
                                                 w.n_rows, C.c_void_p(act.data_ptr())))

    def gemm_gated_bf16(self, gate_up, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """Prefill: bf16 [rows, hidden] -> bf16 silu(x . gate^T) * (x . up^T) on tcgen05 tensor cores."""
        w = self._quant_weight(gate_up)
        if x.dtype != torch.bfloat16 or x.dim() != 2 or not x.is_contiguous() or x.device != self.torch_device:
            raise _kernel_err("gemm_gated_bf16 x must be a contiguous 2-D bf16 tensor on " + str(self.torch_device))
        rows = x.shape[0]
        if out is None:
            out = torch.empty(rows, w.n_rows, dtype=torch.bfloat16, device=self.torch_device)
        if tuple(out.shape) != (rows, w.n_rows) or out.dtype != torch.bfloat16 or not out.is_contiguous():
            raise _kernel_err(f"gemm_gated_bf16 out must be a contiguous bf16 [{rows}, {w.n_rows}] tensor")
        self._check(self._lib.ocl_q_gemm_gated_bf16(self._ctx, w.handle, C.c_void_p(x.data_ptr()), rows, x.shape[1],
                                                    w.n_rows, C.c_void_p(out.data_ptr())))
        return out

    def mlp_gated_silu(self, x, rows: int, hidden: int, intermediate: int, gate_w, up_w, down_w,
                       gate_buf, up_buf, out) -> None:
        """KernelBackend::mlp_gated_silu (crates/kernels/src/lib.rs:150) on quantized weights.

        gate_w is either a pair from `pair_gated` (then up_w is None) or a plain
        gate weight with up_w its partner, paired for this call only.  x / gate_buf
        / out are either contiguous f32 tensors on this device or host f32 numpy
        arrays (then copied in and out).  gate_buf ends holding silu(gate) * up,
        as in the reference; up_buf is accepted for signature parity and left
        untouched (the fused pass never materialises up).
        """
        if rows == 0:
            raise _kernel_err("mlp_gated_silu seq_len must be non-zero")
        if hidden == 0:
            raise _kernel_err("mlp_gated_silu hidden must be non-zero")
        if intermediate == 0:
            raise _kernel_err("mlp_gated_silu intermediate must be non-zero")
        temp = None
        gw = self._quant_weight(gate_w)
        if not gw.gated:
            if up_w is None:
                raise _kernel_err("mlp_gated_silu up_w is required unless gate_w is a gate/up pair")
            temp = self.pair_gated(gw, up_w)
            gw = temp.quant
        elif up_w is not None and self._quant_weight(up_w) is not gw:
            raise _kernel_err("mlp_gated_silu gate_w is already a gate/up pair; pass up_w=None")
        dw = self._quant_weight(down_w)
        host = not isinstance(x, torch.Tensor)
        sizes = {"x": rows * hidden, "gate_buf": rows * intermediate, "out": rows * hidden}
        for name, t in (("x", x), ("gate_buf", gate_buf), ("out", out)):
            n = t.numel() if isinstance(t, torch.Tensor) else np.asarray(t).size
            if n != sizes[name]:
                raise _kernel_err(f"mlp_gated_silu {name} length {n} does not match {sizes[name]}")
        try:
            if host:
                xd = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32).reshape(-1)).to(self.torch_device)
                ad = torch.empty(rows * intermediate, dtype=torch.float32, device=self.torch_device)
                od = torch.empty(rows * hidden, dtype=torch.float32, device=self.torch_device)
                torch.cuda.synchronize(self.torch_device)  # the copy-in ran on torch's stream
            else:
                xd, ad, od = x, gate_buf, out
                for t in (xd, ad, od):
                    if t.dtype != torch.float32 or not t.is_contiguous() or t.device != self.torch_device:
                        raise _kernel_err("mlp_gated_silu operands must be contiguous f32 tensors on "
                                          + str(self.torch_device))
            self._check(self._lib.ocl_q_mlp_gated_silu(
                self._ctx, gw.handle, dw.handle, C.c_void_p(xd.data_ptr()), rows, hidden, intermediate,
                C.c_void_p(ad.data_ptr()), C.c_void_p(od.data_ptr())))
            if host:
                self.synchronize()
                np.copyto(gate_buf.reshape(-1), ad.cpu().numpy())
                np.copyto(out.reshape(-1), od.cpu().numpy())
        finally:
            if temp is not None:
                self.synchronize()
                temp.quant.free()

    # -- greedy sampling (crates/runtime/src/sampling.rs:29) ----------------------
    def greedy_sample(self, logits, out: torch.Tensor | None = None):
        """Argmax per row of f32 logits with greedy_sample's tie and NaN rules.

        logits: a contiguous f32 tensor on this device ([vocab] or [rows, vocab]),
        returning int32 ids on the device; or a host f32 array of one row,
        returning the id as an int (copied in and out).
        """
        if not isinstance(logits, torch.Tensor):
            arr = np.ascontiguousarray(logits, dtype=np.float32).reshape(-1)
            if arr.size == 0:
                raise _kernel_err("greedy_sample requires at least one logit")
            ids = self.greedy_sample(torch.from_numpy(arr).to(self.torch_device))
            return int(ids.cpu()[0])
        if logits.dtype != torch.float32 or not logits.is_contiguous() or logits.device != self.torch_device:
            raise _kernel_err("greedy_sample logits must be a contiguous f32 tensor on " + str(self.torch_device))
        rows, vocab = (1, logits.numel()) if logits.dim() == 1 else (logits.shape[0], logits.shape[-1])
        if out is None:
            out = torch.empty(rows, dtype=torch.int32, device=self.torch_device)
        self._check(self._lib.ocl_argmax_f32(self._ctx, C.c_void_p(logits.data_ptr()), rows, vocab,
                                             C.c_void_p(out.data_ptr())))
        return out
