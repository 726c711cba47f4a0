// internal.cuh -- declarations shared by the CUDA translation units.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

#include "layout.cuh"

namespace ocl {

// Activation planes produced by the x-split kernel and read by the GEMV kernels.
// x[m, k] = xs[m, k/256] * (xq[3m, k] + xq[3m+1, k] / 2^7 + xq[3m+2, k] / 2^14)
// up to 2^-21 of the block's largest magnitude.  Column c = 3m + s of xq holds
// split s of activation row m; s16 / s32 hold exact per-16 / per-32 sums of each
// column (used for the Q6_K "-32" offset and the Q4_K "-dmin*m" term).
struct XPlanes {
    int8_t* xq;    // [kColsMax][kx]
    int32_t* s16;  // [kColsMax][kx/16]
    int32_t* s32;  // [kColsMax][kx/32]
    float* xs;     // [kRowsMax][kx/256]
    int8_t* p32;   // [kColsMax][kx/256][16]: per-32 sums as lo (0..63) / hi bytes, sum = lo + 64*hi
    int8_t* p16;   // [kColsMax][kx/256][32]: per-16 sums, same split
    int kx;        // K rounded up to a multiple of 256
};

constexpr int kMaxDevices = 64;  // per-device host-side caches
constexpr int kRowsMax = 16;            // activation rows per GEMV launch
constexpr int kColsMax = 3 * kRowsMax;  // int8 planes per launch
// Rows per GEMV launch when a call has more: 8.  Measured (8B layer, same box):
// 16 rows as one launch 208 us, as two 8-row launches 185 us (12 rows: 183 vs
// 166; 9: 144 vs 140); the 16-row form's staged planes allow one CTA per SM
// and its instruction count grows with the plane columns, so streaming the
// weights twice costs less.  6-row groups lost (253 us at 16 rows).
constexpr int kGemvGroupRows = 8;

// Bytes of scratch the x planes need for a given K.
constexpr size_t xplanes_bytes(int64_t k) {
    return (size_t)kColsMax * ((k + 255) / 256 * 256)     // xq
           + (size_t)kColsMax * ((k + 255) / 256 * 16) * 4  // s16
           + (size_t)kColsMax * ((k + 255) / 256 * 8) * 4   // s32
           + (size_t)kRowsMax * ((k + 255) / 256) * 4       // xs
           + (size_t)kColsMax * ((k + 255) / 256) * 48      // p32 + p16
           + 6 * 256;                                       // alignment slack
}
// Carve the planes out of one scratch allocation (256-byte aligned pieces).
XPlanes xplanes_carve(void* base, int64_t k);

cudaError_t launch_repack(int type, const void* src, int64_t n_rows, int64_t k, void* dst, cudaStream_t s);
cudaError_t launch_dequant(int type, const void* tiles, int64_t n_rows, int64_t k, float* out, cudaStream_t s);
cudaError_t launch_unpack(int type, const void* tiles, int64_t n_rows, int64_t k, void* dst, cudaStream_t s);
cudaError_t launch_embed(const void* tiles, int64_t n_rows, int64_t k, const int32_t* ids, int64_t n_ids,
                         float* out, unsigned int* bad, cudaStream_t s);

// x [rows<=16, k] f32 -> planes (waits for the previous kernel when `pdl`).
// `type` (the GEMV's weight type) limits the plane sums written to the ones its
// GEMV reads; -1 writes all of them.
cudaError_t launch_xsplit(const float* x, int rows, int64_t k, const XPlanes& p, bool pdl, cudaStream_t s,
                          int type = -1);

// Launch geometry of one GEMV.
struct GemvPlan {
    int nt;             // n8 tiles of activation planes (3*rows/8 rounded up); 0 = single-row layout
    int64_t n_rt;       // 16-row tiles
    int64_t groups;     // CTAs along N (8/kw row tiles each)
    int kw;             // warps per row tile inside a CTA (K split in shared memory)
    int n_units;        // 256-k units along K
    int ks;             // K splits across CTAs
    int umax;           // units in the largest CTA range
    size_t smem;        // dynamic shared memory per CTA
    size_t part_floats; // cross-CTA partial sums (0 when ks == 1)
};
GemvPlan plan_gemv(int type, int64_t n, int64_t k, int rows, int sms);
// Plan for a gate/up pair stored as interleaved row tiles (tile 2t = gate tile
// t, tile 2t+1 = up tile t; n_gate outputs): every CTA holds whole pairs.
GemvPlan plan_gemv_gated(int type, int64_t n_gate, int64_t k, int rows, int sms);
// Same plan without a cross-CTA K split (required by the fused all-reduce);
// false if the CTA's activation planes then no longer fit in shared memory.
bool plan_single_split(GemvPlan& pl, int type, int rows);

// Tensor-parallel all-reduce fused into the GEMV epilogue (row-split layers).
// Every rank owns one buffer: {epoch, CTAs done} (256 bytes), then packet slots
// u64 [2 parities][world][max_elems]; peers' buffers are mapped into this
// process (CUDA IPC over NVLink), so pkt[p] is rank p's slots as seen from here.
constexpr int kTpMax = 8;
struct TpArgs {
    int world = 1, rank = 0;
    int64_t max_elems = 0;
    unsigned long long* pkt[kTpMax] = {};
    unsigned int* ctl = nullptr;  // local: [0] epoch, [1] CTAs done this launch
};
// A packet's tag `v` has reached launch tag `tag` (tags grow by one per launch;
// the signed difference keeps the test right across 2^32 wrap).
__host__ __device__ inline bool tp_flag_reached(unsigned int v, unsigned int tag) {
    return (int)(v - tag) >= 0;
}
constexpr size_t kTpCtlBytes = 256;
inline size_t tp_buffer_bytes(int world, int64_t max_elems) {
    return kTpCtlBytes + (size_t)2 * world * max_elems * 8;
}

struct GemvArgs {
    const uint8_t* W;
    int64_t n, k, n_rt;
    int n_units, nblk, ks, rt_per_cta, umax;
    XPlanes p;
    int rows;
    const float* bias;
    float* y;
    float* part;             // [ks][rows][n] when ks > 1
    unsigned int* counters;  // [groups], zero between launches
    unsigned int* err;       // [0] bad embedding ids, [1] bounded waits that gave up
    TpArgs tp;               // world > 1: sum the rows over ranks in the epilogue (ks must be 1)
    int gated;               // 1: interleaved gate/up tiles, y = silu(gate) * up over n = n_gate outputs
    unsigned int* host_err;  // non-null: a mapped pinned host word set to 1 when a wait gives up
};

// y [rows<=16, n] = planes . W^T (+ bias), geometry from plan_gemv.  `pdl`
// launches with programmatic dependent launch (the kernel waits for its
// predecessor before reading the planes).
cudaError_t launch_gemv(int type, const void* tiles, int64_t n, int64_t k, const XPlanes& p, int rows,
                        const float* bias, float* y, const GemvPlan& pl, float* part, unsigned int* counters,
                        unsigned int* err, bool pdl, cudaStream_t s, const TpArgs* tp = nullptr,
                        unsigned int* host_err = nullptr);
// act [rows<=16, n_gate] = silu(planes . Wg^T) * (planes . Wu^T) over an
// interleaved gate/up weight, geometry from plan_gemv_gated.
cudaError_t launch_gemv_gated(int type, const void* tiles, int64_t n_gate, int64_t k, const XPlanes& p, int rows,
                              float* act, const GemvPlan& pl, float* part, unsigned int* counters, unsigned int* err,
                              bool pdl, cudaStream_t s);

// Greedy argmax per row of f32 logits (greedy_sample semantics); slots and
// counters [rows] must be zero and are left zero.
constexpr int kArgmaxRowsMax = 65535;
cudaError_t launch_argmax(const float* logits, int64_t rows, int64_t vocab, int32_t* ids,
                          unsigned long long* slots, unsigned int* counters, cudaStream_t s);

// Prefill GEMM: y bf16 [M, N] = x bf16 [M, K] . W^T on tcgen05 (K a multiple of 256).
// gated_n_out > 0: W is an interleaved gate/up pair with N = 2 * 16 * row tiles
// of each, and y bf16 [M, gated_n_out] = silu(x . gate^T) * (x . up^T).
// yf != nullptr: f32 output instead of bf16 (y unused), plus bias[n] when given
// (non-gated): the form ocl_q_linear uses for many rows.
cudaError_t launch_qgemm(int type, const void* tiles, int64_t M, int64_t N, int64_t K, const uint16_t* x,
                         uint16_t* y, unsigned int* err, cudaStream_t s, int64_t gated_n_out = 0,
                         float* yf = nullptr, const float* bias = nullptr);
// x f32 [n] -> bf16 bits, round to nearest even.
cudaError_t launch_cast_bf16(const float* x, uint16_t* xb, int64_t n, cudaStream_t s);

}  // namespace ocl
