// noalloc.cu -- ocl_q_linear_noalloc: the quantized GEMV without any device
// allocation, for callers that may not allocate GPU memory on their hot path.
//
// The kernels are the same as ocl_q_linear's (activation split + streaming
// GEMV); only their scratch comes from a file-scope static device array of
// kScratchBytes instead of a context's cudaMalloc'd buffers.  Its layout:
//   [0, kPlanesBytes)                      activation planes (in_features <= kMaxK)
//   [kPlanesBytes, +kCounterBytes)         split-K arrival counters + error flags
//   [kPlanesBytes + kCounterBytes, end)    split-K partial sums
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "../../include/ocelotl_cuda.h"
#include "internal.cuh"

namespace ocl {
void set_thread_error(const char* msg);
}

namespace {

constexpr int64_t kMaxK = 16384;
constexpr size_t kScratchBytes = 4u << 20;
constexpr size_t kPlanesBytes = (ocl::xplanes_bytes(kMaxK) + 255) / 256 * 256;
constexpr size_t kMaxGroups = 4096;
constexpr size_t kCounterBytes = (kMaxGroups + 64) * sizeof(unsigned int);  // counters, then 2 error flags
constexpr size_t kPartBytes = kScratchBytes - kPlanesBytes - kCounterBytes;
static_assert(kPlanesBytes + kCounterBytes < kScratchBytes, "scratch layout");

// The scratch.  Host code must not pass this name to a kernel: on the host it
// only stands in for the symbol; its device address comes from
// cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_scratch[kScratchBytes];

struct DeviceSlot {
    bool ready = false;
    unsigned char* scratch = nullptr;  // device address of g_scratch on this device
    int sms = 0;
};
constexpr int kMaxDevices = 64;
DeviceSlot g_slots[kMaxDevices];
std::mutex g_mu;

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    ocl::set_thread_error(buf);
    return code;
}

// Once per device, with that device current: look up the array's device address.
int setup(int dev, DeviceSlot*& out) {
    if (dev < 0 || dev >= kMaxDevices) return fail(OCL_ERR_INVALID, "q_linear_noalloc: device %d out of range", dev);
    std::lock_guard<std::mutex> lk(g_mu);
    DeviceSlot& s = g_slots[dev];
    if (!s.ready) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_scratch);
        if (e != cudaSuccess)
            return fail(OCL_ERR_CUDA, "q_linear_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
        int sms = 0;
        e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess)
            return fail(OCL_ERR_CUDA, "q_linear_noalloc: cudaDeviceGetAttribute: %s", cudaGetErrorString(e));
        s.scratch = static_cast<unsigned char*>(p);
        s.sms = sms;
        s.ready = true;
    }
    out = &s;
    return OCL_OK;
}

}  // namespace

extern "C" int ocl_q_linear_noalloc(int type, const void* w, size_t n_rows, size_t k, const float* x, size_t rows,
                                    const float* bias, float* y, void* stream) {
    if (type != OCL_Q4_K && type != OCL_Q6_K && type != OCL_Q8_0)
        return fail(OCL_ERR_UNSUPPORTED,
                    "unsupported feature `ggml_type` (requested `%d`): supported = [Q4_K(12), Q6_K(14), Q8_0(8)]",
                    type);
    const size_t be = (size_t)ocl::block_elems(type);
    if (k == 0 || k % be != 0)
        return fail(OCL_ERR_UNSUPPORTED, "unsupported feature `in_features` (requested `%zu`): supported = "
                    "[multiples of %zu]", k, be);
    if ((int64_t)k > kMaxK)
        return fail(OCL_ERR_UNSUPPORTED, "unsupported feature `q_linear_noalloc in_features` (requested `%zu`): "
                    "supported = [<= %lld, the size of its static scratch]", k, (long long)kMaxK);
    if (!w || !x || !y) return fail(OCL_ERR_INVALID, "q_linear_noalloc: weight / x / y pointer is null");
    if (n_rows == 0 || rows == 0) return fail(OCL_ERR_INVALID, "q_linear_noalloc: n_rows and rows must be > 0");
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail(OCL_ERR_CUDA, "q_linear_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
    DeviceSlot* slot = nullptr;
    int rc = setup(dev, slot);
    if (rc) return rc;

    // Check every 16-row group's geometry before launching anything.
    for (size_t r0 = 0; r0 < rows; r0 += ocl::kGemvGroupRows) {  // the same row groups as ocl_q_linear
        const int m = (int)((rows - r0) < (size_t)ocl::kGemvGroupRows ? (rows - r0) : ocl::kGemvGroupRows);
        const ocl::GemvPlan pl = ocl::plan_gemv(type, (int64_t)n_rows, (int64_t)k, m, slot->sms);
        if (pl.part_floats * sizeof(float) > kPartBytes || (pl.ks > 1 && (size_t)pl.groups > kMaxGroups))
            return fail(OCL_ERR_UNSUPPORTED, "unsupported feature `q_linear_noalloc shape` (requested `%zu x %zu, "
                        "%d rows`): supported = [split-K partial sums within its %zu-byte static scratch]",
                        n_rows, k, m, kPartBytes);
    }

    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (s) {  // the scratch address below belongs to the current device
        int sdev = -1;
        e = cudaStreamGetDevice(s, &sdev);
        if (e != cudaSuccess) return fail(OCL_ERR_CUDA, "q_linear_noalloc: cudaStreamGetDevice: %s", cudaGetErrorString(e));
        if (sdev != dev)
            return fail(OCL_ERR_INVALID, "q_linear_noalloc: stream belongs to device %d but device %d is current", sdev,
                        dev);
    }
    unsigned char* base = slot->scratch;
    const ocl::XPlanes planes = ocl::xplanes_carve(base, (int64_t)k);
    unsigned int* counters = reinterpret_cast<unsigned int*>(base + kPlanesBytes);
    unsigned int* flags = counters + kMaxGroups;
    float* part = reinterpret_cast<float*>(base + kPlanesBytes + kCounterBytes);
    // The array keeps the previous call's contents: counters must start at zero
    // (a launch that gave up a wait can leave them raised).  The error flags
    // after them are kept until ocl_noalloc_take_device_errors reads them.
    e = cudaMemsetAsync(counters, 0, kMaxGroups * sizeof(unsigned int), s);
    if (e != cudaSuccess) return fail(OCL_ERR_CUDA, "q_linear_noalloc: clearing counters: %s", cudaGetErrorString(e));
    for (size_t r0 = 0; r0 < rows; r0 += ocl::kGemvGroupRows) {  // the same row groups as ocl_q_linear
        const int m = (int)((rows - r0) < (size_t)ocl::kGemvGroupRows ? (rows - r0) : ocl::kGemvGroupRows);
        const ocl::GemvPlan pl = ocl::plan_gemv(type, (int64_t)n_rows, (int64_t)k, m, slot->sms);
        e = ocl::launch_xsplit(x + r0 * k, m, (int64_t)k, planes, false, s, type);
        if (e == cudaSuccess)
            e = ocl::launch_gemv(type, w, (int64_t)n_rows, (int64_t)k, planes, m, bias, y + r0 * n_rows, pl, part,
                                 counters, flags, false, s);
        if (e != cudaSuccess) return fail(OCL_ERR_CUDA, "q_linear_noalloc: launch: %s", cudaGetErrorString(e));
    }
    return OCL_OK;
}

extern "C" int ocl_noalloc_take_device_errors(void* stream, unsigned int* timeouts) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail(OCL_ERR_CUDA, "noalloc_take_device_errors: cudaGetDevice: %s", cudaGetErrorString(e));
    DeviceSlot* slot = nullptr;
    int rc = setup(dev, slot);
    if (rc) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    unsigned int* flags = reinterpret_cast<unsigned int*>(slot->scratch + kPlanesBytes) + kMaxGroups;
    unsigned int h[2] = {0, 0};
    e = cudaMemcpyAsync(h, flags, sizeof h, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(flags, 0, sizeof h, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return fail(OCL_ERR_CUDA, "noalloc_take_device_errors: %s", cudaGetErrorString(e));
    if (timeouts) *timeouts = h[1];
    if (h[1] != 0)
        return fail(OCL_ERR_TIMEOUT, "q_linear_noalloc: %u bounded device wait(s) gave up since the last check; the "
                    "outputs of the affected calls are incomplete", h[1]);
    return OCL_OK;
}
