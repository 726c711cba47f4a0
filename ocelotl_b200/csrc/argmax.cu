// argmax.cu -- greedy sampling over f32 logits on the device.
//
// Semantics of greedy_sample (crates/runtime/src/sampling.rs:29-52): a scan
// from index 0 that moves only on a strictly greater value, so
//   * ties go to the lowest index,
//   * NaN never wins (every comparison with it is false) -- unless logits[0] is
//     NaN, which then can never be displaced: the answer is 0,
//   * -0.0 and +0.0 compare equal.
// Here each row is cut into chunks; every CTA reduces its chunk to one 64-bit
// key (order-preserving bits of the value << 32 | ~index, NaN skipped, -0.0
// folded to +0.0) and atomically maxes it into the row's slot, so the largest
// value and, among equals, the smallest index win.  The last CTA of a row to
// arrive (arrival counter) writes the id, applies the logits[0]-is-NaN rule and
// resets the slot and the counter for the next launch.
#include <cuda_runtime.h>

#include "internal.cuh"

namespace ocl {

namespace {

constexpr int kThreads = 256, kPerThread = 16, kChunk = kThreads * kPerThread;

__device__ __forceinline__ unsigned long long key_of(float v, uint32_t idx) {
    uint32_t b = __float_as_uint(v == 0.0f ? 0.0f : v);  // -0.0 -> +0.0
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);       // monotone in v
    return ((unsigned long long)b << 32) | (unsigned long long)(0xFFFFFFFFu - idx);
}

__global__ void __launch_bounds__(kThreads) argmax_kernel(const float* __restrict__ logits, int64_t vocab,
                                                          int32_t* __restrict__ ids,
                                                          unsigned long long* __restrict__ slots,
                                                          unsigned int* __restrict__ counters) {
    const int64_t row = blockIdx.y;
    const float* x = logits + row * vocab;
    const int64_t c0 = (int64_t)blockIdx.x * kChunk;
    unsigned long long best = 0;  // below every non-NaN key
    const bool vec = ((reinterpret_cast<uintptr_t>(x) & 15) == 0);
#pragma unroll
    for (int j = 0; j < kPerThread / 4; ++j) {
        const int64_t i = c0 + ((int64_t)j * kThreads + threadIdx.x) * 4;
        float v[4];
        if (vec && i + 4 <= vocab) {
            const float4 q = __ldcs(reinterpret_cast<const float4*>(x + i));
            v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
        } else {
#pragma unroll
            for (int e = 0; e < 4; ++e) v[e] = i + e < vocab ? x[i + e] : __int_as_float(0x7fc00000);
        }
#pragma unroll
        for (int e = 0; e < 4; ++e)
            if (!isnan(v[e])) {
                const unsigned long long k = key_of(v[e], (uint32_t)(i + e));
                best = k > best ? k : best;
            }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const unsigned long long k = __shfl_xor_sync(0xffffffffu, best, o);
        best = k > best ? k : best;
    }
    __shared__ unsigned long long warp_best[kThreads / 32];
    __shared__ bool last;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) warp_best[warp] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < kThreads / 32; ++w) best = warp_best[w] > best ? warp_best[w] : best;
        if (best) atomicMax(slots + row, best);
        __threadfence();
        last = atomicAdd(counters + row, 1u) == gridDim.x - 1;
        if (last) {
            __threadfence();
            const unsigned long long k = atomicExch(slots + row, 0ull);  // read and reset
            int32_t id = (int32_t)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull));
            if (isnan(x[0]) || k == 0) id = 0;
            ids[row] = id;
            counters[row] = 0;
        }
    }
}

}  // namespace

cudaError_t launch_argmax(const float* logits, int64_t rows, int64_t vocab, int32_t* ids,
                          unsigned long long* slots, unsigned int* counters, cudaStream_t s) {
    if (rows <= 0 || vocab <= 0 || rows > 65535) return cudaErrorInvalidValue;
    const dim3 grid((unsigned)((vocab + kChunk - 1) / kChunk), (unsigned)rows);
    argmax_kernel<<<grid, kThreads, 0, s>>>(logits, vocab, ids, slots, counters);
    return cudaGetLastError();
}

}  // namespace ocl
