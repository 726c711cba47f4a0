/*
 * ocelotl_cuda.h -- C ABI of the B200 (sm_100a) quantized-linear backend.
 *
 * This is the drop-in boundary for Ocelotl's quantized linear-layer hot path.
 * A host-side backend (the Rust `CudaKernelBackend` a maintainer would add to
 * `ocelotl-kernels`, or the Python mirror in ocelotl_b200/backend.py) binds these
 * entry points.  Plain pointers and sizes only; device pointers are CUDA device
 * addresses on the context's device; `stream` arguments are cudaStream_t passed as
 * void* (NULL = the context's stream).
 *
 * Error convention (crates/core/src/lib.rs:14-30,75-80 and
 * crates/kernels/src/lib.rs:2443-2494): every call returns OCL_OK (0) or a
 * negative status.  OCL_ERR_UNSUPPORTED maps to OcelotlError::Unsupported and is
 * returned BEFORE any launch (unknown ggml type, K not a multiple of the block
 * size); OCL_ERR_INVALID maps to OcelotlError::Kernel for shape / length / null
 * pointer mismatches; OCL_ERR_CUDA and OCL_ERR_OOM map to OcelotlError::Kernel
 * with backend "cuda-sm100a".  ocl_last_error() returns the message of the last
 * failing call on that context (thread-safe per context).
 *
 * Thread safety: the reference trait is Send + Sync (crates/kernels/src/lib.rs:84);
 * a context serialises its calls with a mutex, so one context may be shared
 * across host threads.  Use one context per stream for concurrency.
 */
#ifndef OCELOTL_CUDA_H
#define OCELOTL_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define OCL_ABI_VERSION 1

#if defined(__GNUC__)
#define OCL_API __attribute__((visibility("default")))
#else
#define OCL_API
#endif

/* Status codes. */
enum {
    OCL_OK = 0,
    OCL_ERR_INVALID = -1,     /* shape / length / pointer mismatch -> KernelError */
    OCL_ERR_UNSUPPORTED = -2, /* type / shape outside the supported set -> Unsupported */
    OCL_ERR_CUDA = -3,        /* CUDA runtime failure -> KernelError */
    OCL_ERR_OOM = -4,         /* device allocation failed -> KernelError */
    OCL_ERR_TIMEOUT = -5      /* a bounded device-side wait gave up -> KernelError */
};

/* GGUF tensor-type tags, crates/loader/src/gguf_inspect.rs:178,182,184. */
enum { OCL_Q8_0 = 8, OCL_Q4_K = 12, OCL_Q6_K = 14 };

/* Device layouts of a quantized weight.
 *  OCL_LAYOUT_GGUF:    the GGUF super-blocks as stored in the file, row-major
 *                      [n_rows, k/block_elems] blocks (input format only).
 *  OCL_LAYOUT_TILED16: the repacked layout every kernel reads: 16-row tiles, each
 *                      tile's blocks regrouped so that one coalesced 16-byte load
 *                      per lane yields tensor-core operand fragments (the exact byte
 *                      map is documented in ocelotl_b200/csrc/layout.cuh).  Same byte
 *                      count as GGUF for N a multiple of 16. */
enum { OCL_LAYOUT_GGUF = 0, OCL_LAYOUT_TILED16 = 1 };

typedef struct ocl_ctx ocl_ctx;   /* one device + stream + scratch */
typedef struct ocl_qbuf ocl_qbuf; /* a quantized weight resident in HBM */
typedef struct ocl_tpcomm ocl_tpcomm; /* tensor-parallel peer buffers of one rank */

/* ---- context ------------------------------------------------------------ */

/* Create a context on CUDA device `device` (Device::Gpu{ordinal},
 * crates/core/src/lib.rs:437-441).  Replaces the backend construction done in
 * crates/kernels/src/cubecl_backend.rs:46-69 for the CubeCL backend. */
OCL_API int ocl_cuda_init(int device, ocl_ctx** out);
OCL_API void ocl_cuda_destroy(ocl_ctx* ctx);
/* Message of the last failing call on `ctx` ("" if none).  With ctx == NULL,
 * the message of the last failing context-free call (ocl_cuda_init,
 * ocl_q_linear_noalloc) on this thread. */
OCL_API const char* ocl_last_error(const ocl_ctx* ctx);
/* Set the stream later calls launch on (NULL = legacy default stream). */
OCL_API int ocl_set_stream(ocl_ctx* ctx, void* stream);
OCL_API int ocl_synchronize(ocl_ctx* ctx);
/* Launch with programmatic dependent launch (default on): a GEMV's weight
 * stream starts while the previous kernel on the stream finishes; it reads its
 * activations only after that kernel completed. */
OCL_API int ocl_set_pdl(ocl_ctx* ctx, int enable);
/* Rows at which ocl_q_linear / ocl_q_linear_host / the gated calls switch
 * from the GEMV to the bf16 tcgen05 GEMM (default 64; 0 = always the GEMV,
 * keeping the 1e-3 GEMV accuracy at any rows). */
OCL_API int ocl_set_gemm_min_rows(ocl_ctx* ctx, size_t rows);
/* Backend id used in KernelError{backend}: "cuda-sm100a". */
OCL_API const char* ocl_backend_id(void);
OCL_API int ocl_abi_version(void);

/* ---- quantized weights (DeviceBuffer for a quantized tensor) ------------ */

/* Upload `n_rows` rows of `k` weights stored as GGUF blocks of `ggml_type`
 * (host memory, `layout` = OCL_LAYOUT_GGUF) and repack them on the device into
 * OCL_LAYOUT_TILED16.  This is the payload upload that the GGUF loader feeds
 * (crates/loader/src/gguf_inspect.rs:119-130 gives file_offset/byte_len; the
 * reference stops at the header).  Owns the device allocation until
 * ocl_q_free (the Rust Drop of CudaQuantBuffer). */
OCL_API int ocl_q_upload(ocl_ctx* ctx, int ggml_type, const void* host_blocks, size_t n_rows, size_t k,
                 int layout, ocl_qbuf** out);
/* Same, from GGUF blocks already in device memory (no host copy). */
OCL_API int ocl_q_upload_device(ocl_ctx* ctx, int ggml_type, const void* dev_blocks, size_t n_rows,
                        size_t k, ocl_qbuf** out);
OCL_API int ocl_q_free(ocl_qbuf* w);
/* Shape and size of a resident weight.  len_f32 = n_rows * k (DeviceBuffer::len_f32,
 * crates/kernels/src/tensor.rs:45-68). */
OCL_API int ocl_q_info(const ocl_qbuf* w, int* ggml_type, size_t* n_rows, size_t* k, size_t* device_bytes);
/* Device address of the repacked bytes (for callers that rotate copies). */
OCL_API const void* ocl_q_device_ptr(const ocl_qbuf* w);

/* Dequantize to f32 [n_rows, k] in device memory; bit-exact with the GGUF
 * block arithmetic.  Backs DeviceBuffer::to_host for a quantized buffer. */
OCL_API int ocl_q_dequant(ocl_ctx* ctx, const ocl_qbuf* w, float* out_dev);
/* Write the weight back out as GGUF blocks (host memory): a round trip of the
 * repacked layout. */
OCL_API int ocl_q_download_gguf(ocl_ctx* ctx, const ocl_qbuf* w, void* host_blocks);

/* ---- the hot path -------------------------------------------------------- */

/* y[r, o] = bias[o] + sum_k x[r, k] * W[o, k], x f32 [rows, in_features],
 * y f32 [rows, out_features], bias f32 [out_features] or NULL; all device
 * pointers.  W is the resident quantized weight with n_rows == out_features and
 * k == in_features.  Replaces KernelBackend::linear_d for a quantized weight
 * (crates/kernels/src/lib.rs:193-217) and, via ocl_q_linear_host, the slice form
 * linear_out_by_in (crates/kernels/src/lib.rs:107-116, 1939-1967).
 * rows 1..8 run the dequant-GEMV as one launch (HBM-bound); more rows below the
 * context's GEMM threshold (64 by default, ocl_set_gemm_min_rows) are processed
 * in 8-row groups by the same kernel (measured faster than 16-row launches).  GEMV accuracy: the products of the integer quants
 * with x are computed exactly (x split into three int8 planes per 256-k block,
 * i.e. ~21 significant bits), scaled and accumulated in f32; max relative error
 * vs the f32 CPU oracle <= 1e-3.
 * rows >= the threshold (prefill, e.g. Whisper's encoder at rows = audio_ctx,
 * crates/models/src/whisper/primitives.rs:787-839) with in_features a multiple
 * of 256 run ONE tcgen05 GEMM instead, so the weight is streamed once: x is
 * rounded to bf16 on the device, the weight tiles are dequantized to bf16, the
 * products accumulate in f32 and y (+ bias) is written in f32.  Accuracy then:
 * max |y - r| / max(|r|, rms(r)) <= 2e-2 vs the f32 oracle on the bf16-rounded
 * x, the prefill bound.  The bf16 copy of x lives in a context buffer grown on
 * demand (rows * in_features * 2 bytes). */
OCL_API int ocl_q_linear(ocl_ctx* ctx, const ocl_qbuf* w, const float* x_dev, size_t rows,
                 size_t in_features, size_t out_features, const float* bias_dev, float* y_dev);

/* Same with host buffers (x, bias, y in host memory), on the context stream,
 * synchronising before it returns.  The slice-based linear_out_by_in.
 * Returns OCL_ERR_TIMEOUT (KernelError) when a bounded device wait of this call
 * gave up (the context's timeout counter is then cleared; waits of earlier
 * device-pointer calls are reported by ocl_take_device_errors).
 * Page-locked (pinned) buffers are read and written by the kernels in place
 * through unified addressing; pageable ones are copied through a device staging
 * area kept by the context.  (Environment OCL_HOST_ZEROCOPY=0 forces staging.) */
OCL_API int ocl_q_linear_host(ocl_ctx* ctx, const ocl_qbuf* w, const float* x_host, size_t rows,
                      size_t in_features, size_t out_features, const float* bias_host,
                      float* y_host);

/* ---- tensor parallelism (one process per GPU) ----------------------------- */
/* The reference has no multi-device code (Device::Gpu{ordinal} names one GPU,
 * crates/core/src/lib.rs:437-441); these entry points are new.
 * ocl_tp_comm_create allocates this rank's receive buffer (packet slots, 2 x
 * world x max_elems x 8 bytes, plus 256 bytes of launch counters; max_groups is
 * kept for ABI stability and must be non-zero, it no longer sizes anything) and
 * writes its 64-byte CUDA IPC handle to ipc_handle_out; the caller gathers all
 * ranks' handles (in rank order, e.g. with torch.distributed all_gather) and
 * passes them to ocl_tp_comm_open, which maps the peers' buffers (NVLink /
 * NVSwitch peer memory).  A handle equal to this rank's own maps that slot back
 * onto this rank's buffer (loopback, used to exercise the bounded wait without a
 * second process). */
OCL_API int ocl_tp_comm_create(ocl_ctx* ctx, int rank, int world, size_t max_elems, size_t max_groups,
                               ocl_tpcomm** out, void* ipc_handle_out);
OCL_API int ocl_tp_comm_open(ocl_ctx* ctx, ocl_tpcomm* comm, const void* ipc_handles);
OCL_API int ocl_tp_comm_destroy(ocl_tpcomm* comm);
/* Device address of this rank's packet slots, u64 [2 parities][world][max_elems]:
 * slot [par][p][e] holds (value bits | launch tag << 32) as rank p last stored
 * it for output element e.  For tests of the packet protocol. */
OCL_API unsigned long long* ocl_tp_comm_packets(ocl_tpcomm* comm);
/* Row-split quantized linear with the all-reduce fused into the GEMV: each rank
 * holds W[:, k0:k1] and x[:, k0:k1]; every rank's y receives the sum over ranks
 * (plus bias), identical bits on every rank.  Each output value goes to every
 * rank as one 8-byte packet (value, launch tag) -- no flags, no fences -- and
 * each rank waits (bounded, ~1 s; a timeout is counted by
 * ocl_take_device_errors and leaves y unwritten) until every rank's packet for
 * its outputs has arrived.  Launch e stores tag e + 1; a waiter accepts any tag
 * at or past its own.  Every rank must issue the same sequence of these calls. */
OCL_API int ocl_q_linear_allreduce(ocl_ctx* ctx, ocl_tpcomm* comm, const ocl_qbuf* w, const float* x_dev,
                                   size_t rows, size_t in_features, size_t out_features, const float* bias_dev,
                                   float* y_dev);

/* Allocation-free variant of ocl_q_linear, for callers that cannot allocate
 * GPU memory on the hot path: code running inside someone else's memory pool
 * or under a strict no-allocation budget, plugins that may not call cudaMalloc
 * (it can synchronise the device and stall the host), and hosts that must know
 * their memory footprint up front.  No counterpart in the reference.
 * It takes no context: `w_tiled_dev` is a weight already in OCL_LAYOUT_TILED16
 * on the current device (e.g. ocl_q_device_ptr of an uploaded weight),
 * x / bias / y are device pointers, and it launches on `stream` (cudaStream_t,
 * NULL = default stream) on the current device.  Its scratch (activation planes,
 * split-K partial sums and counters) is one static 4 MiB device array that
 * every GPU loading this library holds until exit; in_features above 16384 or
 * shapes whose partial sums exceed that array are rejected with
 * OCL_ERR_UNSUPPORTED before any launch.  The first call on a device looks up
 * that array's device address (no allocation); make the first call before any
 * stream capture.  All calls share the array, so calls that overlap on the GPU
 * (different streams or devices' contexts racing on one device) race on it:
 * serialise them on one stream.  `stream` must belong to the current device
 * (OCL_ERR_INVALID otherwise).  Below ocl_q_linear's GEMM threshold the
 * results are bit-identical to its (same kernels, same 8-row groups, same
 * plans); this entry point never switches to the prefill GEMM.  Errors:
 * ocl_last_error(NULL).  A bounded device wait that gives up is counted in the
 * same array; read it with ocl_noalloc_take_device_errors. */
OCL_API int ocl_q_linear_noalloc(int ggml_type, const void* w_tiled_dev, size_t n_rows, size_t k,
                                 const float* x_dev, size_t rows, const float* bias_dev, float* y_dev,
                                 void* stream);
/* Read and clear the wait-timeout counter that ocl_q_linear_noalloc calls on
 * the current device accumulate (a copy on `stream`, then a stream
 * synchronisation; no allocation).  Returns OCL_ERR_TIMEOUT when it was
 * non-zero. */
OCL_API int ocl_noalloc_take_device_errors(void* stream, unsigned int* timeouts);

/* Prefill: y bf16 [rows, out_features] = x bf16 [rows, in_features] . W^T, f32
 * accumulate on tcgen05 tensor cores (weights dequantized to bf16 tiles in
 * shared memory).  Tolerance vs the f32 oracle on the same bf16-rounded x:
 * 2e-2 relative.  bf16 values are passed as uint16_t bit patterns. */
OCL_API int ocl_q_gemm_bf16(ocl_ctx* ctx, const ocl_qbuf* w, const uint16_t* x_dev, size_t rows,
                    size_t in_features, size_t out_features, uint16_t* y_dev);

/* Fused gated MLP (crates/kernels/src/mlp.rs:139-240, KernelBackend::mlp_gated_silu
 * at crates/kernels/src/lib.rs:150).  The reference multiplies by f32 gate_w /
 * up_w [hidden, intermediate] and down_w [intermediate, hidden]; here they are
 * GGUF quantized weights, GGUF-shaped (rows = out features, k = in features).
 *
 * ocl_q_pair_gated: a new buffer holding gate and up (same type and shape) as
 * interleaved 16-row tiles, so one GEMV pass streams both against one copy of
 * x.  The inputs stay valid and owned by the caller; free the pair with
 * ocl_q_free.  A pair is accepted only by the gated calls below.
 *
 * ocl_q_linear_gated: act f32 [rows, intermediate] = silu(x . gate^T) * (x . up^T),
 * silu(z) = z / (1 + exp(-z)), in one launch over the pair.
 *
 * ocl_q_mlp_gated_silu: out f32 [rows, hidden] = act . down^T after
 * ocl_q_linear_gated; act_dev is the caller's [rows, intermediate] scratch (the
 * reference's gate_buf, which likewise ends holding silu(gate) * up).  Errors
 * follow the reference's checks: zero seq_len / hidden / intermediate and shape
 * mismatches are OCL_ERR_INVALID.  Tolerance as ocl_q_linear per projection.
 *
 * ocl_q_gemm_gated_bf16: prefill form, act bf16 [rows, intermediate] for bf16 x
 * [rows, hidden] (hidden a multiple of 256, x 16-byte aligned): one tcgen05
 * GEMM over the pair, silu * up applied to the f32 accumulators before the
 * bf16 store. */
OCL_API int ocl_q_pair_gated(ocl_ctx* ctx, const ocl_qbuf* gate, const ocl_qbuf* up, ocl_qbuf** out);
OCL_API int ocl_q_linear_gated(ocl_ctx* ctx, const ocl_qbuf* gate_up, const float* x_dev, size_t rows,
                               size_t hidden, size_t intermediate, float* act_dev);
OCL_API int ocl_q_mlp_gated_silu(ocl_ctx* ctx, const ocl_qbuf* gate_up, const ocl_qbuf* down, const float* x_dev,
                                 size_t rows, size_t hidden, size_t intermediate, float* act_dev, float* out_dev);
OCL_API int ocl_q_gemm_gated_bf16(ocl_ctx* ctx, const ocl_qbuf* gate_up, const uint16_t* x_dev, size_t rows,
                                  size_t hidden, size_t intermediate, uint16_t* act_dev);

/* Greedy sampling (crates/runtime/src/sampling.rs:29 greedy_sample) on the
 * device: ids_dev[r] = argmax of logits_dev row r ([rows, vocab] f32), the
 * lowest index among equal maxima, -0.0 equal to +0.0, NaN never chosen --
 * except that a NaN at index 0 makes the answer 0, as the reference's scan
 * does.  vocab == 0 is OCL_ERR_INVALID ("greedy_sample requires at least one
 * logit"); rows <= 65535.  Bit-exact with the reference. */
OCL_API int ocl_argmax_f32(ocl_ctx* ctx, const float* logits_dev, size_t rows, size_t vocab, int32_t* ids_dev);

/* Q8_0 embedding gather: out f32 [n_ids, k] = dequantized rows ids[i] of `table`
 * (ids int32 in device memory), bit-exact with the GGUF block arithmetic.  The
 * ids are only known on the device, so an id outside [0, n_rows) cannot fail the
 * call without a synchronisation: its row is written as zeros and a per-context
 * device counter is bumped; ocl_take_device_errors reads and clears it. */
OCL_API int ocl_q_embed_rows(ocl_ctx* ctx, const ocl_qbuf* table, const int32_t* ids_dev, size_t n_ids,
                     float* out_dev);
/* Read and clear the context's device-side error counters (synchronises the
 * stream): embedding ids that were out of range, and bounded device waits that
 * gave up (a GEMV whose shared-memory stream stalled for ~1 s, or a fused
 * all-reduce whose peers did not signal in ~1 s; that output is then
 * incomplete).  Either pointer may be NULL.  Returns OCL_ERR_TIMEOUT (after
 * filling both counters) when any wait gave up, so that a caller checking only
 * the status still sees the failure (KernelError in the reference's terms,
 * crates/core/src/lib.rs:75-80). */
OCL_API int ocl_take_device_errors(ocl_ctx* ctx, unsigned int* bad_ids, unsigned int* timeouts);

#ifdef __cplusplus
}
#endif
#endif
