// api.cu -- the C ABI (include/ocelotl_cuda.h): context, weight upload, the
// quantized linear entry points.  Host-side validation mirrors
// validate_linear_out_by_in (crates/kernels/src/lib.rs:2443-2494) and the
// "unsupported before launch" rule of the reference's kernel design.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/ocelotl_cuda.h"
#include "internal.cuh"

struct ocl_ctx {
    int device = 0;
    int sms = 148;
    cudaStream_t stream = nullptr;
    std::mutex mu;
    std::string err;
    void* scratch = nullptr;  // x planes for the GEMV
    unsigned long long* amax_slots = nullptr;  // argmax: per-row best key, zero between launches
    unsigned int* amax_counters = nullptr;     // argmax: per-row CTA arrivals, zero between launches
    char* io = nullptr;       // device staging of the host-slice calls (x, bias, y), grown on demand
    size_t io_bytes = 0;
    size_t scratch_bytes = 0;
    float* part = nullptr;  // cross-CTA split-K partial sums
    size_t part_bytes = 0;
    unsigned int* counters = nullptr;  // split-K arrival counters, zero between launches
    size_t counter_count = 0;
    bool pdl = true;  // launch with programmatic dependent launch
    unsigned int* dev_flags = nullptr;  // [0] bad embedding ids, [1] bounded waits that gave up
    unsigned int* host_flags = nullptr;      // pinned, mapped: [0] set by a GEMV of a host-slice call whose wait gave up,
                                             // [1] the GEMM route's copy of dev_flags[1]
    unsigned int* host_flags_dev = nullptr;  // the device address of host_flags
    uint16_t* xbf = nullptr;  // bf16 copy of x for the prefill GEMM form, grown on demand
    size_t xbf_bytes = 0;
    size_t gemm_min_rows = 64;  // rows at which ocl_q_linear switches to the tcgen05 GEMM (0 = never)
};

struct ocl_tpcomm {
    int device = 0, world = 1, rank = 0;
    int64_t max_elems = 0, max_groups = 0;
    void* buf = nullptr;  // this rank's buffer
    size_t bytes = 0;
    void* peer[ocl::kTpMax] = {};  // every rank's buffer as mapped here (own = buf)
    bool open = false;
};

struct ocl_qbuf {
    int device = 0;
    int type = 0;
    size_t n_rows = 0, k = 0, bytes = 0;
    void* dev = nullptr;
    bool gated = false;  // interleaved gate/up row tiles; n_rows = gate (= up) rows
};

namespace {

thread_local std::string g_init_err;

int fail(ocl_ctx* ctx, int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    if (ctx) ctx->err = buf;
    else g_init_err = buf;
    return code;
}

int cuda_fail(ocl_ctx* ctx, cudaError_t e, const char* what) {
    return fail(ctx, e == cudaErrorMemoryAllocation ? OCL_ERR_OOM : OCL_ERR_CUDA, "%s: %s (%s)", what,
                cudaGetErrorString(e), cudaGetErrorName(e));
}

#define OCL_CUDA(ctx, call, what)                                  \
    do {                                                           \
        cudaError_t e_ = (call);                                   \
        if (e_ != cudaSuccess) return cuda_fail((ctx), e_, (what)); \
    } while (0)

const char* type_name(int t) {
    return t == OCL_Q4_K ? "Q4_K" : t == OCL_Q6_K ? "Q6_K" : t == OCL_Q8_0 ? "Q8_0" : "?";
}

// Unsupported type / K before any launch.
int check_type_k(ocl_ctx* ctx, int type, size_t k) {
    if (type != OCL_Q4_K && type != OCL_Q6_K && type != OCL_Q8_0)
        return fail(ctx, OCL_ERR_UNSUPPORTED,
                    "unsupported feature `ggml_type` (requested `%d`): supported = [Q4_K(12), Q6_K(14), Q8_0(8)]",
                    type);
    const size_t be = (size_t)ocl::block_elems(type);
    if (k == 0 || k % be != 0)
        return fail(ctx, OCL_ERR_UNSUPPORTED,
                    "unsupported feature `%s in_features` (requested `%zu`): supported = [multiples of %zu]",
                    type_name(type), k, be);
    return OCL_OK;
}

size_t tiled_bytes(int type, size_t n_rows, size_t k) {
    return (n_rows + 15) / 16 * (k / (size_t)ocl::rec_k(type)) * (size_t)ocl::rec_bytes(type);
}

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

// Device staging for ocl_q_linear_host.  A per-call cudaMallocAsync /
// cudaFreeAsync pair returned its memory to the driver at every stream
// synchronisation (the default pool keeps nothing), which cost ~0.5 ms a call.
int ensure_io(ocl_ctx* ctx, size_t bytes) {
    if (ctx->io_bytes >= bytes) return OCL_OK;
    if (ctx->io) {
        OCL_CUDA(ctx, cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
        cudaFree(ctx->io);
        ctx->io = nullptr;
        ctx->io_bytes = 0;
    }
    OCL_CUDA(ctx, cudaMalloc((void**)&ctx->io, bytes), "cudaMalloc(io staging)");
    ctx->io_bytes = bytes;
    return OCL_OK;
}

bool zero_copy_enabled() {
    static const bool on = [] {
        const char* f = getenv("OCL_HOST_ZEROCOPY");  // 0 forces the staged copies
        return f ? atoi(f) != 0 : true;
    }();
    return on;
}

// Device address of a page-locked host buffer, or nullptr for pageable memory.
const float* mapped(const float* host) {
    cudaPointerAttributes at{};
    if (cudaPointerGetAttributes(&at, host) != cudaSuccess) {
        cudaGetLastError();  // clear
        return nullptr;
    }
    if (at.type != cudaMemoryTypeHost || !at.devicePointer) return nullptr;
    return (const float*)at.devicePointer;
}

int ensure_scratch(ocl_ctx* ctx, size_t bytes) {
    if (ctx->scratch_bytes >= bytes) return OCL_OK;
    if (ctx->scratch) {
        // a previous launch may still read the old planes
        OCL_CUDA(ctx, cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
        cudaFree(ctx->scratch);
        ctx->scratch = nullptr;
        ctx->scratch_bytes = 0;
    }
    OCL_CUDA(ctx, cudaMalloc(&ctx->scratch, bytes), "cudaMalloc(scratch)");
    ctx->scratch_bytes = bytes;
    return OCL_OK;
}

int ensure_split_buffers(ocl_ctx* ctx, const ocl::GemvPlan& pl) {
    const size_t pb = pl.part_floats * sizeof(float);
    if (pb > ctx->part_bytes) {
        if (ctx->part) {
            OCL_CUDA(ctx, cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
            cudaFree(ctx->part);
            ctx->part = nullptr;
            ctx->part_bytes = 0;
        }
        OCL_CUDA(ctx, cudaMalloc(&ctx->part, pb), "cudaMalloc(split-K partials)");
        ctx->part_bytes = pb;
    }
    if (pl.ks > 1 && (size_t)pl.groups > ctx->counter_count) {
        if (ctx->counters) {
            OCL_CUDA(ctx, cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
            cudaFree(ctx->counters);
            ctx->counters = nullptr;
            ctx->counter_count = 0;
        }
        const size_t cnt = (size_t)pl.groups < 4096 ? 4096 : (size_t)pl.groups;
        OCL_CUDA(ctx, cudaMalloc(&ctx->counters, cnt * sizeof(unsigned int)), "cudaMalloc(split-K counters)");
        OCL_CUDA(ctx, cudaMemsetAsync(ctx->counters, 0, cnt * sizeof(unsigned int), ctx->stream), "memset counters");
        ctx->counter_count = cnt;
    }
    return OCL_OK;
}

int check_linear_shapes(ocl_ctx* ctx, const ocl_qbuf* w, size_t rows, size_t in_features, size_t out_features) {
    if (!w) return fail(ctx, OCL_ERR_INVALID, "linear_d weight is null");
    if (w->gated)
        return fail(ctx, OCL_ERR_INVALID, "linear_d weight is a gate/up pair; use ocl_q_linear_gated / ocl_q_mlp_gated_silu");
    if (w->device != ctx->device)
        return fail(ctx, OCL_ERR_INVALID, "weight lives on device %d but the context is on device %d", w->device,
                    ctx->device);
    if (w->k != in_features)
        return fail(ctx, OCL_ERR_INVALID, "linear_d weight in_features=%zu does not match in_features=%zu", w->k,
                    in_features);
    if (w->n_rows != out_features)
        return fail(ctx, OCL_ERR_INVALID, "linear_d weight out_features=%zu does not match out_features=%zu",
                    w->n_rows, out_features);
    if (rows == 0) return fail(ctx, OCL_ERR_INVALID, "linear_d rows must be > 0");
    return OCL_OK;
}

int ensure_xbf(ocl_ctx* ctx, size_t bytes) {
    if (ctx->xbf_bytes >= bytes) return OCL_OK;
    if (ctx->xbf) {
        OCL_CUDA(ctx, cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
        cudaFree(ctx->xbf);
        ctx->xbf = nullptr;
        ctx->xbf_bytes = 0;
    }
    OCL_CUDA(ctx, cudaMalloc((void**)&ctx->xbf, bytes), "cudaMalloc(bf16 activations)");
    ctx->xbf_bytes = bytes;
    return OCL_OK;
}

// Many rows (prefill): one tcgen05 GEMM over bf16-rounded x instead of
// rows/16 GEMV passes that would each stream the whole weight.
bool use_gemm(const ocl_ctx* ctx, const ocl_qbuf* w, size_t rows) {
    return ctx->gemm_min_rows > 0 && rows >= ctx->gemm_min_rows && w->k % 256 == 0;
}

int q_gemm_f32_locked(ocl_ctx* ctx, const ocl_qbuf* w, const float* x, size_t rows, const float* bias, float* y,
                      bool gated) {
    const size_t k = w->k, n = w->n_rows;
    int rc = ensure_xbf(ctx, rows * k * 2 + 256);
    if (rc) return rc;
    OCL_CUDA(ctx, ocl::launch_cast_bf16(x, ctx->xbf, (int64_t)(rows * k), ctx->stream), "bf16 cast launch");
    const int64_t n_gemm = gated ? (int64_t)((n + 15) / 16) * 32 : (int64_t)n;
    OCL_CUDA(ctx,
             ocl::launch_qgemm(w->type, w->dev, (int64_t)rows, n_gemm, (int64_t)k, ctx->xbf, nullptr, ctx->dev_flags,
                               ctx->stream, gated ? (int64_t)n : 0, y, bias),
             "prefill gemm launch");
    return OCL_OK;
}

// y = x . W^T (+bias) for device pointers, any rows (16-row groups).  host_err:
// mapped host word the GEMVs set when a bounded wait gives up (host-slice calls).
int q_linear_locked(ocl_ctx* ctx, const ocl_qbuf* w, const float* x, size_t rows, const float* bias, float* y,
                    unsigned int* host_err = nullptr) {
    const size_t k = w->k, n = w->n_rows;
    if (use_gemm(ctx, w, rows)) return q_gemm_f32_locked(ctx, w, x, rows, bias, y, false);
    int rc = ensure_scratch(ctx, ocl::xplanes_bytes((int64_t)k));
    if (rc) return rc;
    const ocl::XPlanes planes = ocl::xplanes_carve(ctx->scratch, (int64_t)k);
    const size_t G = ocl::kGemvGroupRows;
    for (size_t r0 = 0; r0 < rows; r0 += G) {
        const int m = (int)((rows - r0) < G ? (rows - r0) : G);
        const ocl::GemvPlan pl = ocl::plan_gemv(w->type, (int64_t)n, (int64_t)k, m, ctx->sms);
        rc = ensure_split_buffers(ctx, pl);
        if (rc) return rc;
        OCL_CUDA(ctx, ocl::launch_xsplit(x + r0 * k, m, (int64_t)k, planes, ctx->pdl, ctx->stream, w->type),
                 "x split launch");
        OCL_CUDA(ctx,
                 ocl::launch_gemv(w->type, w->dev, (int64_t)n, (int64_t)k, planes, m, bias, y + r0 * n, pl, ctx->part,
                                  ctx->counters, ctx->dev_flags, ctx->pdl, ctx->stream, nullptr, host_err),
                 "gemv launch");
    }
    return OCL_OK;
}

// act [rows, n_gate] = silu(x . Wg^T) * (x . Wu^T) over an interleaved pair.
int q_gated_locked(ocl_ctx* ctx, const ocl_qbuf* w, const float* x, size_t rows, float* act) {
    const size_t k = w->k, n = w->n_rows;
    if (use_gemm(ctx, w, rows)) return q_gemm_f32_locked(ctx, w, x, rows, nullptr, act, true);
    int rc = ensure_scratch(ctx, ocl::xplanes_bytes((int64_t)k));
    if (rc) return rc;
    const ocl::XPlanes planes = ocl::xplanes_carve(ctx->scratch, (int64_t)k);
    const size_t G = ocl::kGemvGroupRows;
    for (size_t r0 = 0; r0 < rows; r0 += G) {
        const int m = (int)((rows - r0) < G ? (rows - r0) : G);
        const ocl::GemvPlan pl = ocl::plan_gemv_gated(w->type, (int64_t)n, (int64_t)k, m, ctx->sms);
        rc = ensure_split_buffers(ctx, pl);
        if (rc) return rc;
        OCL_CUDA(ctx, ocl::launch_xsplit(x + r0 * k, m, (int64_t)k, planes, ctx->pdl, ctx->stream, w->type),
                 "x split launch");
        OCL_CUDA(ctx,
                 ocl::launch_gemv_gated(w->type, w->dev, (int64_t)n, (int64_t)k, planes, m, act + r0 * n, pl,
                                        ctx->part, ctx->counters, ctx->dev_flags, ctx->pdl, ctx->stream),
                 "gated gemv launch");
    }
    return OCL_OK;
}

int check_gated_shapes(ocl_ctx* ctx, const ocl_qbuf* gu, size_t rows, size_t hidden, size_t intermediate) {
    if (!gu) return fail(ctx, OCL_ERR_INVALID, "mlp_gated_silu gate/up weight is null");
    if (!gu->gated) return fail(ctx, OCL_ERR_INVALID, "mlp_gated_silu weight is not a gate/up pair (ocl_q_pair_gated)");
    if (gu->device != ctx->device)
        return fail(ctx, OCL_ERR_INVALID, "weight lives on device %d but the context is on device %d", gu->device,
                    ctx->device);
    if (rows == 0) return fail(ctx, OCL_ERR_INVALID, "mlp_gated_silu seq_len must be non-zero");
    if (hidden == 0) return fail(ctx, OCL_ERR_INVALID, "mlp_gated_silu hidden must be non-zero");
    if (intermediate == 0) return fail(ctx, OCL_ERR_INVALID, "mlp_gated_silu intermediate must be non-zero");
    if (gu->k != hidden)
        return fail(ctx, OCL_ERR_INVALID, "mlp_gated_silu gate_w in_features=%zu does not match hidden=%zu", gu->k,
                    hidden);
    if (gu->n_rows != intermediate)
        return fail(ctx, OCL_ERR_INVALID, "mlp_gated_silu gate_w out_features=%zu does not match intermediate=%zu",
                    gu->n_rows, intermediate);
    return OCL_OK;
}

// A kernel of this call gave up a bounded wait: clear the device counter and
// report it as KernelError.
int take_timeouts(ocl_ctx* ctx, const char* op) {
    unsigned int n = 0;
    cudaError_t e = cudaMemcpyAsync(&n, ctx->dev_flags + 1, 4, cudaMemcpyDeviceToHost, ctx->stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(ctx->dev_flags + 1, 0, 4, ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "clear timeout counter");
    ctx->host_flags[0] = ctx->host_flags[1] = 0;
    return fail(ctx, OCL_ERR_TIMEOUT,
                "%s: %u bounded device wait(s) gave up (~1 s each); the output of the affected row groups is "
                "incomplete", op, n);
}

}  // namespace

namespace ocl {
// Message for ocl_last_error(NULL) from entry points that take no context.
void set_thread_error(const char* msg) { g_init_err = msg; }
}  // namespace ocl

extern "C" {

const char* ocl_backend_id(void) { return "cuda-sm100a"; }
int ocl_abi_version(void) { return OCL_ABI_VERSION; }

int ocl_cuda_init(int device, ocl_ctx** out) {
    if (!out) return fail(nullptr, OCL_ERR_INVALID, "ocl_cuda_init: out is null");
    *out = nullptr;
    int count = 0;
    cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess) return cuda_fail(nullptr, e, "cudaGetDeviceCount");
    if (device < 0 || device >= count)
        return fail(nullptr, OCL_ERR_INVALID, "device ordinal %d out of range (%d devices)", device, count);
    cudaDeviceProp prop;
    e = cudaGetDeviceProperties(&prop, device);
    if (e != cudaSuccess) return cuda_fail(nullptr, e, "cudaGetDeviceProperties");
    if (prop.major != 10 || prop.minor != 0)
        return fail(nullptr, OCL_ERR_UNSUPPORTED,
                    "unsupported feature `device` (requested `sm_%d%d`): supported = [sm_100a (B200)]", prop.major,
                    prop.minor);
    DeviceGuard guard(device);
    ocl_ctx* ctx = new ocl_ctx();
    ctx->device = device;
    ctx->sms = prop.multiProcessorCount;
    e = cudaMalloc(&ctx->dev_flags, 64);
    if (e == cudaSuccess) e = cudaMemset(ctx->dev_flags, 0, 64);
    if (e == cudaSuccess) e = cudaHostAlloc((void**)&ctx->host_flags, 64, cudaHostAllocMapped);
    if (e == cudaSuccess) e = cudaHostGetDevicePointer((void**)&ctx->host_flags_dev, ctx->host_flags, 0);
    if (e != cudaSuccess) {
        if (ctx->dev_flags) cudaFree(ctx->dev_flags);
        delete ctx;
        return cuda_fail(nullptr, e, "context allocation");
    }
    *out = ctx;
    return OCL_OK;
}

void ocl_cuda_destroy(ocl_ctx* ctx) {
    if (!ctx) return;
    {
        DeviceGuard guard(ctx->device);
        cudaStreamSynchronize(ctx->stream);
        if (ctx->scratch) cudaFree(ctx->scratch);
        if (ctx->io) cudaFree(ctx->io);
        if (ctx->amax_slots) cudaFree(ctx->amax_slots);
        if (ctx->amax_counters) cudaFree(ctx->amax_counters);
        if (ctx->part) cudaFree(ctx->part);
        if (ctx->counters) cudaFree(ctx->counters);
        if (ctx->dev_flags) cudaFree(ctx->dev_flags);
        if (ctx->host_flags) cudaFreeHost(ctx->host_flags);
        if (ctx->xbf) cudaFree(ctx->xbf);
    }
    delete ctx;
}

const char* ocl_last_error(const ocl_ctx* ctx) { return ctx ? ctx->err.c_str() : g_init_err.c_str(); }

int ocl_set_stream(ocl_ctx* ctx, void* stream) {
    if (!ctx) return OCL_ERR_INVALID;
    std::lock_guard<std::mutex> lk(ctx->mu);
    ctx->stream = (cudaStream_t)stream;
    return OCL_OK;
}

int ocl_synchronize(ocl_ctx* ctx) {
    if (!ctx) return OCL_ERR_INVALID;
    std::lock_guard<std::mutex> lk(ctx->mu);
    DeviceGuard guard(ctx->device);
    OCL_CUDA(ctx, cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
    return OCL_OK;
}

static int upload_impl(ocl_ctx* ctx, int type, const void* src, bool src_on_device, size_t n_rows, size_t k,
                       ocl_qbuf** out) {
    if (!ctx) return OCL_ERR_INVALID;
    std::lock_guard<std::mutex> lk(ctx->mu);
    if (!out) return fail(ctx, OCL_ERR_INVALID, "ocl_q_upload: out is null");
    *out = nullptr;
    int rc = check_type_k(ctx, type, k);
    if (rc) return rc;
    if (n_rows == 0) return fail(ctx, OCL_ERR_INVALID, "ocl_q_upload: n_rows must be > 0");
    if (!src) return fail(ctx, OCL_ERR_INVALID, "ocl_q_upload: blocks pointer is null");
    DeviceGuard guard(ctx->device);
    const size_t gguf_bytes = n_rows * (k / (size_t)ocl::block_elems(type)) * (size_t)ocl::block_bytes(type);
    const size_t bytes = tiled_bytes(type, n_rows, k);
    ocl_qbuf* w = new ocl_qbuf();
    w->device = ctx->device;
    w->type = type;
    w->n_rows = n_rows;
    w->k = k;
    w->bytes = bytes;
    cudaError_t e = cudaMalloc(&w->dev, bytes);
    if (e != cudaSuccess) {
        delete w;
        return cuda_fail(ctx, e, "cudaMalloc(weight)");
    }
    const void* dsrc = src;
    void* staging = nullptr;
    if (!src_on_device) {
        e = cudaMalloc(&staging, gguf_bytes);
        if (e == cudaSuccess) e = cudaMemcpyAsync(staging, src, gguf_bytes, cudaMemcpyHostToDevice, ctx->stream);
        dsrc = staging;
    }
    if (e == cudaSuccess) e = ocl::launch_repack(type, dsrc, (int64_t)n_rows, (int64_t)k, w->dev, ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    if (staging) cudaFree(staging);
    if (e != cudaSuccess) {
        cudaFree(w->dev);
        delete w;
        return cuda_fail(ctx, e, "weight upload/repack");
    }
    *out = w;
    return OCL_OK;
}

int ocl_q_upload(ocl_ctx* ctx, int type, const void* host_blocks, size_t n_rows, size_t k, int layout,
                 ocl_qbuf** out) {
    if (ctx && layout != OCL_LAYOUT_GGUF) {
        std::lock_guard<std::mutex> lk(ctx->mu);
        return fail(ctx, OCL_ERR_UNSUPPORTED,
                    "unsupported feature `upload layout` (requested `%d`): supported = [GGUF(0)]", layout);
    }
    return upload_impl(ctx, type, host_blocks, false, n_rows, k, out);
}

int ocl_q_upload_device(ocl_ctx* ctx, int type, const void* dev_blocks, size_t n_rows, size_t k, ocl_qbuf** out) {
    return upload_impl(ctx, type, dev_blocks, true, n_rows, k, out);
}

int ocl_q_free(ocl_qbuf* w) {
    if (!w) return OCL_OK;
    DeviceGuard guard(w->device);
    if (w->dev) cudaFree(w->dev);
    delete w;
    return OCL_OK;
}

int ocl_q_info(const ocl_qbuf* w, int* type, size_t* n_rows, size_t* k, size_t* device_bytes) {
    if (!w) return OCL_ERR_INVALID;
    if (type) *type = w->type;
    if (n_rows) *n_rows = w->n_rows;
    if (k) *k = w->k;
    if (device_bytes) *device_bytes = w->bytes;
    return OCL_OK;
}

const void* ocl_q_device_ptr(const ocl_qbuf* w) { return w ? w->dev : nullptr; }

int ocl_q_dequant(ocl_ctx* ctx, const ocl_qbuf* w, float* out_dev) {
    if (!ctx) return OCL_ERR_INVALID;
    std::lock_guard<std::mutex> lk(ctx->mu);
    if (!w || !out_dev) return fail(ctx, OCL_ERR_INVALID, "ocl_q_dequant: null argument");
    if (w->gated) return fail(ctx, OCL_ERR_UNSUPPORTED, "unsupported feature `dequant of a gate/up pair`");
    DeviceGuard guard(ctx->device);
    OCL_CUDA(ctx, ocl::launch_dequant(w->type, w->dev, (int64_t)w->n_rows, (int64_t)w->k, out_dev, ctx->stream),
             "dequant launch");
    return OCL_OK;
}

int ocl_q_download_gguf(ocl_ctx* ctx, const ocl_qbuf* w, void* host_blocks) {
    if (!ctx) return OCL_ERR_INVALID;
    std::lock_guard<std::mutex> lk(ctx->mu);
    if (!w || !host_blocks) return fail(ctx, OCL_ERR_INVALID, "ocl_q_download_gguf: null argument");
    if (w->gated) return fail(ctx, OCL_ERR_UNSUPPORTED, "unsupported feature `download of a gate/up pair`");
    DeviceGuard guard(ctx->device);
    const size_t bytes = w->n_rows * (w->k / (size_t)ocl::block_elems(w->type)) * (size_t)ocl::block_bytes(w->type);
    void* tmp = nullptr;
    OCL_CUDA(ctx, cudaMalloc(&tmp, bytes), "cudaMalloc(download)");
    cudaError_t e = ocl::launch_unpack(w->type, w->dev, (int64_t)w->n_rows, (int64_t)w->k, tmp, ctx->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(host_blocks, tmp, bytes, cudaMemcpyDeviceToHost, ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    cudaFree(tmp);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "download");
    return OCL_OK;
}

int ocl_q_linear(ocl_ctx* ctx, const ocl_qbuf* w, const float* x_dev, size_t rows, size_t in_features,
                 size_t out_features, const float* bias_dev, float* y_dev) {
    if (!ctx) return OCL_ERR_INVALID;
    std::lock_guard<std::mutex> lk(ctx->mu);
    int rc = check_linear_shapes(ctx, w, rows, in_features, out_features);
    if (rc) return rc;
    if (!x_dev || !y_dev) return fail(ctx, OCL_ERR_INVALID, "linear_d x/out pointer is null");
    DeviceGuard guard(ctx->device);
    return q_linear_locked(ctx, w, x_dev, rows, bias_dev, y_dev);
}

int ocl_q_linear_host(ocl_ctx* ctx, const ocl_qbuf* w, const float* x_host, size_t rows, size_t in_features,
                      size_t out_features, const float* bias_host, float* y_host) {
    if (!ctx) return OCL_ERR_INVALID;
    std::lock_guard<std::mutex> lk(ctx->mu);
    int rc = check_linear_shapes(ctx, w, rows, in_features, out_features);
    if (rc) return rc;
    if (!x_host || !y_host) return fail(ctx, OCL_ERR_INVALID, "linear_out_by_in x/out pointer is null");
    DeviceGuard guard(ctx->device);
    const size_t xb = rows * in_features * 4, yb = rows * out_features * 4, bb = bias_host ? out_features * 4 : 0;
    // Page-locked host buffers are read and written by the kernels in place
    // (mapped through unified addressing): no staging copies, no copy-engine
    // round trips.  Pageable buffers go through the device staging area.
    const float* xd = zero_copy_enabled() ? mapped(x_host) : nullptr;
    float* yd = zero_copy_enabled() ? const_cast<float*>(mapped(y_host)) : nullptr;
    const float* bd = (bias_host && zero_copy_enabled()) ? mapped(bias_host) : nullptr;
    rc = ensure_io(ctx, xb + yb + bb + 512);
    if (rc) return rc;
    char* buf = ctx->io;
    cudaError_t e = cudaSuccess;
    if (!xd) {
        e = cudaMemcpyAsync(buf, x_host, xb, cudaMemcpyHostToDevice, ctx->stream);
        xd = (const float*)buf;
    }
    float* y_stage = (float*)(buf + ((xb + 255) & ~(size_t)255));
    if (bias_host && !bd && e == cudaSuccess) {
        float* b_stage = (float*)((char*)y_stage + ((yb + 255) & ~(size_t)255));
        e = cudaMemcpyAsync(b_stage, bias_host, bb, cudaMemcpyHostToDevice, ctx->stream);
        bd = b_stage;
    }
    const bool y_mapped = yd != nullptr;
    if (!y_mapped) yd = y_stage;
    // A GEMV whose bounded wait gives up sets host_flags[0] with a plain store
    // to this mapped word, read after the synchronisation below (a 4-byte copy
    // of the device counter instead cost ~9 us a call).  The GEMM route (many
    // rows) copies the device counter into host_flags[1] instead.
    volatile unsigned int* hf = ctx->host_flags;
    hf[0] = hf[1] = 0;
    const bool gemm_route = use_gemm(ctx, w, rows);
    if (e == cudaSuccess) {
        rc = q_linear_locked(ctx, w, xd, rows, bd, yd, ctx->host_flags_dev);
        if (rc == OCL_OK && !y_mapped) e = cudaMemcpyAsync(y_host, yd, yb, cudaMemcpyDeviceToHost, ctx->stream);
        if (rc == OCL_OK && e == cudaSuccess && gemm_route)
            e = cudaMemcpyAsync(ctx->host_flags + 1, ctx->dev_flags + 1, 4, cudaMemcpyDeviceToHost, ctx->stream);
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    if (rc) return rc;
    if (e != cudaSuccess) return cuda_fail(ctx, e, "linear_out_by_in host path");
    if (hf[0] != 0 || hf[1] != 0) return take_timeouts(ctx, "linear_out_by_in");
    return OCL_OK;
}

int ocl_q_embed_rows(ocl_ctx* ctx, const ocl_qbuf* table, const int32_t* ids_dev, size_t n_ids, float* out_dev) {
    if (!ctx) return OCL_ERR_INVALID;
    std::lock_guard<std::mutex> lk(ctx->mu);
    if (!table || !ids_dev || !out_dev) return fail(ctx, OCL_ERR_INVALID, "embed_rows: null argument");
    if (table->type != OCL_Q8_0)
        return fail(ctx, OCL_ERR_UNSUPPORTED, "unsupported feature `embedding type` (requested `%s`): supported = [Q8_0]",
                    type_name(table->type));
    if (n_ids == 0) return OCL_OK;
    DeviceGuard guard(ctx->device);
    OCL_CUDA(ctx,
             ocl::launch_embed(table->dev, (int64_t)table->n_rows, (int64_t)table->k, ids_dev, (int64_t)n_ids, out_dev,
                               ctx->dev_flags, ctx->stream),
             "embed launch");
    return OCL_OK;
}

int ocl_take_device_errors(ocl_ctx* ctx, unsigned int* bad_ids, unsigned int* timeouts) {
    if (!ctx) return OCL_ERR_INVALID;
    std::lock_guard<std::mutex> lk(ctx->mu);
    DeviceGuard guard(ctx->device);
    unsigned int h[2] = {0, 0};
    OCL_CUDA(ctx, cudaMemcpyAsync(h, ctx->dev_flags, 8, cudaMemcpyDeviceToHost, ctx->stream), "read flags");
    OCL_CUDA(ctx, cudaMemsetAsync(ctx->dev_flags, 0, 8, ctx->stream), "clear flags");
    OCL_CUDA(ctx, cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
    if (bad_ids) *bad_ids = h[0];
    if (timeouts) *timeouts = h[1];
    if (h[1] != 0)
        return fail(ctx, OCL_ERR_TIMEOUT,
                    "%u bounded device wait(s) gave up since the last check (~1 s each); the outputs of the "
                    "affected launches are incomplete", h[1]);
    return OCL_OK;
}

int ocl_tp_comm_create(ocl_ctx* ctx, int rank, int world, size_t max_elems, size_t max_groups, ocl_tpcomm** out,
                       void* ipc_handle_out) {
    if (!ctx) return OCL_ERR_INVALID;
    std::lock_guard<std::mutex> lk(ctx->mu);
    if (!out || !ipc_handle_out) return fail(ctx, OCL_ERR_INVALID, "tp_comm_create: null output pointer");
    *out = nullptr;
    if (world < 2 || world > ocl::kTpMax || rank < 0 || rank >= world)
        return fail(ctx, OCL_ERR_UNSUPPORTED, "unsupported feature `tensor-parallel world` (requested `%d`, rank %d): "
                    "supported = [2..%d]", world, rank, ocl::kTpMax);
    if (max_elems == 0 || max_groups == 0) return fail(ctx, OCL_ERR_INVALID, "tp_comm_create: zero capacity");
    DeviceGuard guard(ctx->device);
    ocl_tpcomm* c = new ocl_tpcomm();
    c->device = ctx->device;
    c->world = world;
    c->rank = rank;
    c->max_elems = (int64_t)max_elems;
    c->max_groups = (int64_t)max_groups;
    c->bytes = ocl::tp_buffer_bytes(world, c->max_elems);
    cudaError_t e = cudaMalloc(&c->buf, c->bytes);
    if (e == cudaSuccess) e = cudaMemset(c->buf, 0, c->bytes);
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(reinterpret_cast<cudaIpcMemHandle_t*>(ipc_handle_out), c->buf);
    if (e != cudaSuccess) {
        if (c->buf) cudaFree(c->buf);
        delete c;
        return cuda_fail(ctx, e, "tp_comm_create");
    }
    c->peer[rank] = c->buf;
    *out = c;
    return OCL_OK;
}

int ocl_tp_comm_open(ocl_ctx* ctx, ocl_tpcomm* c, const void* handles) {
    if (!ctx) return OCL_ERR_INVALID;
    std::lock_guard<std::mutex> lk(ctx->mu);
    if (!c || !handles) return fail(ctx, OCL_ERR_INVALID, "tp_comm_open: null argument");
    DeviceGuard guard(ctx->device);
    const cudaIpcMemHandle_t* hs = static_cast<const cudaIpcMemHandle_t*>(handles);
    cudaIpcMemHandle_t own;
    OCL_CUDA(ctx, cudaIpcGetMemHandle(&own, c->buf), "tp_comm_open: own handle");
    for (int p = 0; p < c->world; ++p) {
        if (p == c->rank) continue;
        if (memcmp(&hs[p], &own, sizeof own) == 0) {  // loopback: a peer slot mapped onto this rank's buffer
            c->peer[p] = c->buf;
            continue;
        }
        void* ptr = nullptr;
        cudaError_t e = cudaIpcOpenMemHandle(&ptr, hs[p], cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) return cuda_fail(ctx, e, "tp_comm_open: cudaIpcOpenMemHandle");
        c->peer[p] = ptr;
    }
    c->open = true;
    return OCL_OK;
}

int ocl_tp_comm_destroy(ocl_tpcomm* c) {
    if (!c) return OCL_OK;
    DeviceGuard guard(c->device);
    cudaDeviceSynchronize();
    for (int p = 0; p < c->world; ++p)
        if (p != c->rank && c->peer[p] && c->peer[p] != c->buf) cudaIpcCloseMemHandle(c->peer[p]);
    if (c->buf) cudaFree(c->buf);
    delete c;
    return OCL_OK;
}

unsigned long long* ocl_tp_comm_packets(ocl_tpcomm* c) {
    if (!c || !c->buf) return nullptr;
    return reinterpret_cast<unsigned long long*>(static_cast<char*>(c->buf) + ocl::kTpCtlBytes);
}

int ocl_q_linear_allreduce(ocl_ctx* ctx, ocl_tpcomm* c, const ocl_qbuf* w, const float* x_dev, size_t rows,
                           size_t in_features, size_t out_features, const float* bias_dev, float* y_dev) {
    if (!ctx) return OCL_ERR_INVALID;
    std::lock_guard<std::mutex> lk(ctx->mu);
    int rc = check_linear_shapes(ctx, w, rows, in_features, out_features);
    if (rc) return rc;
    if (!c || !c->open) return fail(ctx, OCL_ERR_INVALID, "linear_allreduce: communicator not opened");
    if (c->device != ctx->device) return fail(ctx, OCL_ERR_INVALID, "linear_allreduce: communicator on another device");
    if (!x_dev || !y_dev) return fail(ctx, OCL_ERR_INVALID, "linear_allreduce x/out pointer is null");
    DeviceGuard guard(ctx->device);
    const size_t k = w->k, n = w->n_rows;
    rc = ensure_scratch(ctx, ocl::xplanes_bytes((int64_t)k));
    if (rc) return rc;
    const ocl::XPlanes planes = ocl::xplanes_carve(ctx->scratch, (int64_t)k);
    ocl::TpArgs tp;
    tp.world = c->world;
    tp.rank = c->rank;
    tp.max_elems = c->max_elems;
    for (int p = 0; p < c->world; ++p)
        tp.pkt[p] = reinterpret_cast<unsigned long long*>(static_cast<char*>(c->peer[p]) + ocl::kTpCtlBytes);
    tp.ctl = static_cast<unsigned int*>(c->buf);
    for (size_t r0 = 0; r0 < rows; r0 += ocl::kGemvGroupRows) {
        const int m = (int)((rows - r0) < (size_t)ocl::kGemvGroupRows ? (rows - r0) : ocl::kGemvGroupRows);
        ocl::GemvPlan pl = ocl::plan_gemv(w->type, (int64_t)n, (int64_t)k, m, ctx->sms);
        if (!ocl::plan_single_split(pl, w->type, m))
            return fail(ctx, OCL_ERR_UNSUPPORTED, "unsupported feature `fused all-reduce shape` (requested `%zu x %zu`):"
                        " supported = [activation planes of the full K within shared memory]", n, k);
        if ((int64_t)m * (int64_t)n > c->max_elems)
            return fail(ctx, OCL_ERR_INVALID, "linear_allreduce: %d x %zu outputs exceed the communicator capacity "
                        "(%lld elements)", m, n, (long long)c->max_elems);
        OCL_CUDA(ctx, ocl::launch_xsplit(x_dev + r0 * k, m, (int64_t)k, planes, ctx->pdl, ctx->stream, w->type),
                 "x split launch");
        OCL_CUDA(ctx,
                 ocl::launch_gemv(w->type, w->dev, (int64_t)n, (int64_t)k, planes, m, bias_dev, y_dev + r0 * n, pl,
                                  ctx->part, ctx->counters, ctx->dev_flags, ctx->pdl, ctx->stream, &tp),
                 "fused linear + all-reduce launch");
    }
    return OCL_OK;
}

int ocl_q_pair_gated(ocl_ctx* ctx, const ocl_qbuf* gate, const ocl_qbuf* up, ocl_qbuf** out) {
    if (!ctx) return OCL_ERR_INVALID;
    std::lock_guard<std::mutex> lk(ctx->mu);
    if (!out) return fail(ctx, OCL_ERR_INVALID, "ocl_q_pair_gated: out is null");
    *out = nullptr;
    if (!gate || !up) return fail(ctx, OCL_ERR_INVALID, "ocl_q_pair_gated: null weight");
    if (gate->gated || up->gated) return fail(ctx, OCL_ERR_INVALID, "ocl_q_pair_gated: input is already a pair");
    if (gate->type != up->type)
        return fail(ctx, OCL_ERR_UNSUPPORTED, "unsupported feature `gate/up of different types` (requested `%s/%s`)",
                    type_name(gate->type), type_name(up->type));
    if (gate->n_rows != up->n_rows || gate->k != up->k)
        return fail(ctx, OCL_ERR_INVALID, "gate [%zu x %zu] and up [%zu x %zu] shapes differ", gate->n_rows, gate->k,
                    up->n_rows, up->k);
    if (gate->device != ctx->device || up->device != ctx->device)
        return fail(ctx, OCL_ERR_INVALID, "gate/up weights are not on the context's device %d", ctx->device);
    DeviceGuard guard(ctx->device);
    const size_t n_rt = (gate->n_rows + 15) / 16, tile = gate->bytes / n_rt;
    ocl_qbuf* w = new ocl_qbuf();
    w->device = ctx->device;
    w->type = gate->type;
    w->n_rows = gate->n_rows;
    w->k = gate->k;
    w->bytes = 2 * gate->bytes;
    w->gated = true;
    cudaError_t e = cudaMalloc(&w->dev, w->bytes);
    if (e != cudaSuccess) {
        delete w;
        return cuda_fail(ctx, e, "cudaMalloc(gate/up pair)");
    }
    // row tile t of gate -> tile 2t, of up -> tile 2t+1
    e = cudaMemcpy2DAsync(w->dev, 2 * tile, gate->dev, tile, tile, n_rt, cudaMemcpyDeviceToDevice, ctx->stream);
    if (e == cudaSuccess)
        e = cudaMemcpy2DAsync((char*)w->dev + tile, 2 * tile, up->dev, tile, tile, n_rt, cudaMemcpyDeviceToDevice,
                              ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) {
        cudaFree(w->dev);
        delete w;
        return cuda_fail(ctx, e, "gate/up interleave");
    }
    *out = w;
    return OCL_OK;
}

int ocl_q_linear_gated(ocl_ctx* ctx, const ocl_qbuf* gate_up, const float* x_dev, size_t rows, size_t hidden,
                       size_t intermediate, float* act_dev) {
    if (!ctx) return OCL_ERR_INVALID;
    std::lock_guard<std::mutex> lk(ctx->mu);
    int rc = check_gated_shapes(ctx, gate_up, rows, hidden, intermediate);
    if (rc) return rc;
    if (!x_dev || !act_dev) return fail(ctx, OCL_ERR_INVALID, "linear_gated x/act pointer is null");
    DeviceGuard guard(ctx->device);
    return q_gated_locked(ctx, gate_up, x_dev, rows, act_dev);
}

int ocl_q_mlp_gated_silu(ocl_ctx* ctx, const ocl_qbuf* gate_up, const ocl_qbuf* down, const float* x_dev, size_t rows,
                         size_t hidden, size_t intermediate, float* act_dev, float* out_dev) {
    if (!ctx) return OCL_ERR_INVALID;
    std::lock_guard<std::mutex> lk(ctx->mu);
    int rc = check_gated_shapes(ctx, gate_up, rows, hidden, intermediate);
    if (rc) return rc;
    if (!down) return fail(ctx, OCL_ERR_INVALID, "mlp_gated_silu down_w is null");
    if (down->gated) return fail(ctx, OCL_ERR_INVALID, "mlp_gated_silu down_w is a gate/up pair");
    if (down->device != ctx->device)
        return fail(ctx, OCL_ERR_INVALID, "down_w lives on device %d but the context is on device %d", down->device,
                    ctx->device);
    if (down->k != intermediate || down->n_rows != hidden)
        return fail(ctx, OCL_ERR_INVALID,
                    "mlp_gated_silu down_w [%zu x %zu] does not match shape %zux%zu (out x in)", down->n_rows, down->k,
                    hidden, intermediate);
    if (!x_dev || !act_dev || !out_dev) return fail(ctx, OCL_ERR_INVALID, "mlp_gated_silu x/act/out pointer is null");
    DeviceGuard guard(ctx->device);
    rc = q_gated_locked(ctx, gate_up, x_dev, rows, act_dev);
    if (rc) return rc;
    return q_linear_locked(ctx, down, act_dev, rows, nullptr, out_dev);
}

int ocl_set_gemm_min_rows(ocl_ctx* ctx, size_t rows) {
    if (!ctx) return OCL_ERR_INVALID;
    std::lock_guard<std::mutex> lk(ctx->mu);
    ctx->gemm_min_rows = rows;
    return OCL_OK;
}

int ocl_set_pdl(ocl_ctx* ctx, int enable) {
    if (!ctx) return OCL_ERR_INVALID;
    std::lock_guard<std::mutex> lk(ctx->mu);
    ctx->pdl = enable != 0;
    return OCL_OK;
}

int ocl_q_gemm_bf16(ocl_ctx* ctx, const ocl_qbuf* w, const uint16_t* x_dev, size_t rows, size_t in_features,
                    size_t out_features, uint16_t* y_dev) {
    if (!ctx) return OCL_ERR_INVALID;
    std::lock_guard<std::mutex> lk(ctx->mu);
    int rc = check_linear_shapes(ctx, w, rows, in_features, out_features);
    if (rc) return rc;
    if (in_features % 256 != 0)
        return fail(ctx, OCL_ERR_UNSUPPORTED,
                    "unsupported feature `q_gemm_bf16 in_features` (requested `%zu`): supported = [multiples of 256]",
                    in_features);
    if (!x_dev || !y_dev) return fail(ctx, OCL_ERR_INVALID, "q_gemm_bf16 x/out pointer is null");
    if (((uintptr_t)x_dev & 15) != 0)
        return fail(ctx, OCL_ERR_INVALID, "q_gemm_bf16 x must be 16-byte aligned");
    DeviceGuard guard(ctx->device);
    OCL_CUDA(ctx,
             ocl::launch_qgemm(w->type, w->dev, (int64_t)rows, (int64_t)out_features, (int64_t)in_features, x_dev,
                               y_dev, ctx->dev_flags, ctx->stream),
             "q_gemm launch");
    return OCL_OK;
}

int ocl_q_gemm_gated_bf16(ocl_ctx* ctx, const ocl_qbuf* gate_up, const uint16_t* x_dev, size_t rows, size_t hidden,
                          size_t intermediate, uint16_t* act_dev) {
    if (!ctx) return OCL_ERR_INVALID;
    std::lock_guard<std::mutex> lk(ctx->mu);
    int rc = check_gated_shapes(ctx, gate_up, rows, hidden, intermediate);
    if (rc) return rc;
    if (hidden % 256 != 0)
        return fail(ctx, OCL_ERR_UNSUPPORTED,
                    "unsupported feature `q_gemm_gated_bf16 hidden` (requested `%zu`): supported = [multiples of 256]",
                    hidden);
    if (!x_dev || !act_dev) return fail(ctx, OCL_ERR_INVALID, "q_gemm_gated_bf16 x/act pointer is null");
    if (((uintptr_t)x_dev & 15) != 0) return fail(ctx, OCL_ERR_INVALID, "q_gemm_gated_bf16 x must be 16-byte aligned");
    DeviceGuard guard(ctx->device);
    const int64_t n_int = (int64_t)((intermediate + 15) / 16) * 32;
    OCL_CUDA(ctx,
             ocl::launch_qgemm(gate_up->type, gate_up->dev, (int64_t)rows, n_int, (int64_t)hidden, x_dev, act_dev,
                               ctx->dev_flags, ctx->stream, (int64_t)intermediate),
             "q_gemm_gated launch");
    return OCL_OK;
}

int ocl_argmax_f32(ocl_ctx* ctx, const float* logits_dev, size_t rows, size_t vocab, int32_t* ids_dev) {
    if (!ctx) return OCL_ERR_INVALID;
    std::lock_guard<std::mutex> lk(ctx->mu);
    if (vocab == 0) return fail(ctx, OCL_ERR_INVALID, "greedy_sample requires at least one logit");
    if (rows == 0) return OCL_OK;
    if (!logits_dev || !ids_dev) return fail(ctx, OCL_ERR_INVALID, "argmax: null argument");
    if (rows > (size_t)ocl::kArgmaxRowsMax || vocab > 0x7FFFFFFFu)
        return fail(ctx, OCL_ERR_UNSUPPORTED,
                    "unsupported feature `argmax shape` (requested `%zu x %zu`): supported = [rows <= %d, vocab < 2^31]",
                    rows, vocab, ocl::kArgmaxRowsMax);
    DeviceGuard guard(ctx->device);
    if (!ctx->amax_slots) {
        OCL_CUDA(ctx, cudaMalloc((void**)&ctx->amax_slots, ocl::kArgmaxRowsMax * sizeof(unsigned long long)),
                 "cudaMalloc(argmax slots)");
        OCL_CUDA(ctx, cudaMalloc((void**)&ctx->amax_counters, ocl::kArgmaxRowsMax * sizeof(unsigned int)),
                 "cudaMalloc(argmax counters)");
        OCL_CUDA(ctx, cudaMemsetAsync(ctx->amax_slots, 0, ocl::kArgmaxRowsMax * sizeof(unsigned long long), ctx->stream),
                 "memset argmax slots");
        OCL_CUDA(ctx, cudaMemsetAsync(ctx->amax_counters, 0, ocl::kArgmaxRowsMax * sizeof(unsigned int), ctx->stream),
                 "memset argmax counters");
    }
    OCL_CUDA(ctx,
             ocl::launch_argmax(logits_dev, (int64_t)rows, (int64_t)vocab, ids_dev, ctx->amax_slots,
                                ctx->amax_counters, ctx->stream),
             "argmax launch");
    return OCL_OK;
}

}  // extern "C"
