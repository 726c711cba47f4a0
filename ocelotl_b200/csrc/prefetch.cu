// prefetch.cu -- pull a quantized weight into L2 ahead of the GEMV that reads it.
//
// A decode step is a chain of dependent GEMVs; each call spends a few
// microseconds between its predecessor finishing and its own streaming
// starting (activation split, kernel hand-off), during which HBM sits idle.
// The weights themselves do not depend on anything, so the NEXT projection's
// weight can be brought into L2 while the current one runs: a small kernel on a
// side stream issues bulk L2 prefetches (cp.async.bulk.prefetch.L2, no
// shared-memory destination, no completion to wait for) over the weight's
// bytes.  The GEMV then finds its records in L2.  A prefetch is only a hint: it
// changes no result, needs no ordering against any other work, and a weight
// that is evicted again before it is read is simply read from HBM.
#include <cuda_runtime.h>

#include <cstdint>

#include "internal.cuh"

namespace ocl {

namespace {

constexpr uint32_t kChunk = 32768;  // bytes per bulk prefetch

__global__ void __launch_bounds__(128) prefetch_l2_kernel(const uint8_t* __restrict__ p, uint64_t bytes) {
    const uint64_t n_chunks = (bytes + kChunk - 1) / kChunk;
    for (uint64_t c = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; c < n_chunks;
         c += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t off = c * kChunk;
        const uint32_t sz = (uint32_t)((bytes - off) < kChunk ? (bytes - off) : kChunk);
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p + off), "r"(sz) : "memory");
    }
}

}  // namespace

cudaError_t launch_prefetch_l2(const void* p, uint64_t bytes, cudaStream_t s) {
    // bulk copies want 16-byte aligned addresses and sizes; weights are cudaMalloc'd
    // and every record size is a multiple of 16, so only a foreign pointer trips this
    if ((reinterpret_cast<uintptr_t>(p) & 15) != 0 || (bytes & 15) != 0) return cudaErrorInvalidValue;
    if (bytes == 0) return cudaSuccess;
    const uint64_t n_chunks = (bytes + kChunk - 1) / kChunk;
    const unsigned blocks = (unsigned)((n_chunks + 127) / 128 < 16 ? (n_chunks + 127) / 128 : 16);
    prefetch_l2_kernel<<<blocks, 128, 0, s>>>(static_cast<const uint8_t*>(p), bytes);
    return cudaGetLastError();
}

}  // namespace ocl
