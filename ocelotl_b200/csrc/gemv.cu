// gemv.cu -- decode-time (M = 1..16) fused dequantize-and-multiply.
//
// y[m, n] = bias[n] + sum_k x[m, k] * W[n, k] with W in TILED16 records.
//
// Design (B200, HBM-bound):
//  * Weights stream from HBM exactly once with coalesced 16-byte loads
//    (ld.global.nc.L1::no_allocate), one record (16 rows x 256 k) per warp step,
//    the next record's loads issued before the current one is consumed.
//  * The GGUF quants are small integers, so the inner products run on the
//    tensor cores as exact int8 x int8 -> int32 MMAs (mma.sync m16n8k32 /
//    m16n8k16, ~1.1 POPS on B200): each lane's 16-byte chunk IS its A fragment
//    (after a nibble mask), no shared-memory staging.  Activations come as three
//    int8 planes per row (see XPlanes), so the integer sums are exact and the
//    only rounding happens in the per-super-block f32 scaling:
//        Q4_K: acc += xs * (d * float(sum_j sc_j*c_j) - dmin * float(sum_j m_j*S_j))
//        Q6_K: acc += xs * d * float(sum_j sc_j*(c_j - 32*S_j))
//        Q8_0: acc += xs * d * float(c)
//  * K is split across the warps of a CTA (deterministic shared-memory
//    reduction, fixed order), so a 4096x4096 matrix keeps ~14 warps per SM busy.
#include <cuda_fp16.h>

#include "internal.cuh"

namespace ocl {

namespace {

__device__ __forceinline__ uint4 ld_stream(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ void mma_k32(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

__device__ __forceinline__ void mma_k16(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, "
        "{%7,%7,%7,%7};"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a0), "r"(a1), "r"(b0), "r"(0));
}

// ---------------------------------------------------------------------------
// x split: one warp per (row m, 256-k block b).
// ---------------------------------------------------------------------------
__global__ void xsplit_kernel(const float* __restrict__ x, int rows, int64_t k, XPlanes p) {
    const int b = blockIdx.x, m = blockIdx.y, lane = threadIdx.x;
    const int64_t k0 = (int64_t)b * 256 + lane * 8;
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = (m < rows && k0 + i < k) ? x[(int64_t)m * k + k0 + i] : 0.0f;
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
    bool finite = true;
#pragma unroll
    for (int i = 0; i < 8; ++i) finite = finite && (fabsf(v[i]) <= 3.402823466e38f);
#pragma unroll
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    finite = __all_sync(0xffffffffu, finite);

    // amax < 2^E with E the biased exponent - 126; scale so that |v| < 2^7.
    int e = 0;
    if (finite && amax > 0.0f) {
        const int E = (int)((__float_as_uint(amax) >> 23) & 0xff) - 126;
        e = max(E - 7, -100);
    }
    const float scale = __uint_as_float((uint32_t)(127 - e) << 23);  // 2^-e, exact
    int8_t q[3][8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float s = finite ? v[i] * scale : 0.0f;
        const float x0 = truncf(s);
        const float r1 = (s - x0) * 128.0f;
        const float x1 = truncf(r1);
        const float r2 = (r1 - x1) * 128.0f;
        const float x2 = fminf(fmaxf(rintf(r2), -127.0f), 127.0f);
        q[0][i] = (int8_t)x0;
        q[1][i] = (int8_t)x1;
        q[2][i] = (int8_t)x2;
    }
#pragma unroll
    for (int sp = 0; sp < 3; ++sp) {
        const int col = 3 * m + sp;
        uint2 packed;
        packed.x = (uint32_t)(uint8_t)q[sp][0] | ((uint32_t)(uint8_t)q[sp][1] << 8) |
                   ((uint32_t)(uint8_t)q[sp][2] << 16) | ((uint32_t)(uint8_t)q[sp][3] << 24);
        packed.y = (uint32_t)(uint8_t)q[sp][4] | ((uint32_t)(uint8_t)q[sp][5] << 8) |
                   ((uint32_t)(uint8_t)q[sp][6] << 16) | ((uint32_t)(uint8_t)q[sp][7] << 24);
        *reinterpret_cast<uint2*>(p.xq + (int64_t)col * p.kx + k0) = packed;
        int s = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) s += q[sp][i];
        s += __shfl_xor_sync(0xffffffffu, s, 1);
        if ((lane & 1) == 0) p.s16[(int64_t)col * (p.kx / 16) + b * 16 + (lane >> 1)] = s;
        s += __shfl_xor_sync(0xffffffffu, s, 2);
        if ((lane & 3) == 0) p.s32[(int64_t)col * (p.kx / 32) + b * 8 + (lane >> 2)] = s;
    }
    if (lane == 0)
        p.xs[(int64_t)m * (p.kx / 256) + b] =
            finite ? __uint_as_float((uint32_t)(127 + e) << 23) : __uint_as_float(0x7fc00000u);
}

// ---------------------------------------------------------------------------
// Shared epilogue: reduce the per-warp partials in a fixed order and fold the
// three int8 planes of each activation row.
// ---------------------------------------------------------------------------
template <int NT>
__device__ __forceinline__ void epilogue(float (&acc)[NT][4], float* red, int ks, int rows, int64_t n,
                                         int64_t rt, const float* __restrict__ bias, float* __restrict__ y) {
    constexpr int C = NT * 8;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        float* r0 = red + (warp * 16 + g) * C + nt * 8 + 2 * t;
        float* r1 = red + (warp * 16 + g + 8) * C + nt * 8 + 2 * t;
        r0[0] = acc[nt][0];
        r0[1] = acc[nt][1];
        r1[0] = acc[nt][2];
        r1[1] = acc[nt][3];
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < 16 * rows; idx += blockDim.x) {
        const int row = idx & 15, m = idx >> 4;
        float p0 = 0.f, p1 = 0.f, p2 = 0.f;
        for (int w = 0; w < ks; ++w) {
            const float* r = red + (w * 16 + row) * C + 3 * m;
            p0 += r[0];
            p1 += r[1];
            p2 += r[2];
        }
        const int64_t o = rt * 16 + row;
        if (o < n) {
            float v = (p2 * (1.0f / 16384.0f) + p1 * (1.0f / 128.0f)) + p0;
            if (bias) v += bias[o];
            y[(int64_t)m * n + o] = v;
        }
    }
}

// ---------------------------------------------------------------------------
// Q4_K
// ---------------------------------------------------------------------------
template <int NT>
__global__ void __launch_bounds__(256) gemv_q4k_kernel(const uint8_t* __restrict__ W, int64_t n, int nkb, int ks,
                                                       XPlanes p, int rows, const float* __restrict__ bias,
                                                       float* __restrict__ y) {
    extern __shared__ float red[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int64_t rt = blockIdx.x;
    const int kb0 = (int)((int64_t)nkb * warp / ks), kb1 = (int)((int64_t)nkb * (warp + 1) / ks);
    const uint8_t* recs = W + (size_t)rt * nkb * 2304;
    const int kx32 = p.kx / 32;

    float acc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int v = 0; v < 4; ++v) acc[nt][v] = 0.f;

    uint4 h0, h1, q[4];
    if (kb0 < kb1) {
        const uint8_t* rec = recs + (size_t)kb0 * 2304;
        h0 = __ldg(reinterpret_cast<const uint4*>(rec + 16 * g));
        h1 = __ldg(reinterpret_cast<const uint4*>(rec + 16 * (g + 8)));
#pragma unroll
        for (int c = 0; c < 4; ++c) q[c] = ld_stream(rec + 256 + 512 * c + 16 * lane);
    }
    for (int kb = kb0; kb < kb1; ++kb) {
        uint4 nh0 = h0, nh1 = h1, nq[4] = {q[0], q[1], q[2], q[3]};
        if (kb + 1 < kb1) {
            const uint8_t* rec = recs + (size_t)(kb + 1) * 2304;
            nh0 = __ldg(reinterpret_cast<const uint4*>(rec + 16 * g));
            nh1 = __ldg(reinterpret_cast<const uint4*>(rec + 16 * (g + 8)));
#pragma unroll
            for (int c = 0; c < 4; ++c) nq[c] = ld_stream(rec + 256 + 512 * c + 16 * lane);
        }
        // scales / mins of rows g (h0) and g+8 (h1)
        int sc0[8], mn0[8], sc1[8], mn1[8];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            sc0[j] = (h0.y >> (8 * j)) & 63;
            mn0[j] = (h0.z >> (8 * j)) & 63;
            sc0[j + 4] = ((h0.w >> (8 * j)) & 0xF) | (((h0.y >> (8 * j + 6)) & 3) << 4);
            mn0[j + 4] = ((h0.w >> (8 * j + 4)) & 0xF) | (((h0.z >> (8 * j + 6)) & 3) << 4);
            sc1[j] = (h1.y >> (8 * j)) & 63;
            mn1[j] = (h1.z >> (8 * j)) & 63;
            sc1[j + 4] = ((h1.w >> (8 * j)) & 0xF) | (((h1.y >> (8 * j + 6)) & 3) << 4);
            mn1[j + 4] = ((h1.w >> (8 * j + 4)) & 0xF) | (((h1.z >> (8 * j + 6)) & 3) << 4);
        }
        const float d0 = f16_bits_to_f32(h0.x & 0xffffu), dm0 = f16_bits_to_f32(h0.x >> 16);
        const float d1 = f16_bits_to_f32(h1.x & 0xffffu), dm1 = f16_bits_to_f32(h1.x >> 16);

#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const int colb = nt * 8 + g;  // B column this lane supplies
            const int8_t* xb = p.xq + (int64_t)colb * p.kx + (int64_t)kb * 256 + 8 * t;
            int C[4] = {0, 0, 0, 0};
#pragma unroll
            for (int c = 0; c < 4; ++c) {
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    const int j = 2 * c + half, sh = 4 * half;
                    const uint2 bb = __ldg(reinterpret_cast<const uint2*>(xb + 32 * j));
                    int r[4];
                    mma_k32(r, (q[c].x >> sh) & 0x0F0F0F0Fu, (q[c].z >> sh) & 0x0F0F0F0Fu,
                            (q[c].y >> sh) & 0x0F0F0F0Fu, (q[c].w >> sh) & 0x0F0F0F0Fu, bb.x, bb.y);
                    C[0] += sc0[j] * r[0];
                    C[1] += sc0[j] * r[1];
                    C[2] += sc1[j] * r[2];
                    C[3] += sc1[j] * r[3];
                }
            }
            // min term with the exact per-32 sums of the two columns this lane owns
            const int ca = nt * 8 + 2 * t, cb = ca + 1;
            const int4* sa = reinterpret_cast<const int4*>(p.s32 + (int64_t)ca * kx32 + (int64_t)kb * 8);
            const int4* sb = reinterpret_cast<const int4*>(p.s32 + (int64_t)cb * kx32 + (int64_t)kb * 8);
            const int4 sa0 = __ldg(sa), sa1 = __ldg(sa + 1), sb0 = __ldg(sb), sb1 = __ldg(sb + 1);
            const int Sa[8] = {sa0.x, sa0.y, sa0.z, sa0.w, sa1.x, sa1.y, sa1.z, sa1.w};
            const int Sb[8] = {sb0.x, sb0.y, sb0.z, sb0.w, sb1.x, sb1.y, sb1.z, sb1.w};
            int M0 = 0, M1 = 0, M2 = 0, M3 = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                M0 += mn0[j] * Sa[j];
                M1 += mn0[j] * Sb[j];
                M2 += mn1[j] * Sa[j];
                M3 += mn1[j] * Sb[j];
            }
            const float xa = __ldg(p.xs + (int64_t)(ca / 3) * (p.kx / 256) + kb);
            const float xb2 = __ldg(p.xs + (int64_t)(cb / 3) * (p.kx / 256) + kb);
            acc[nt][0] += xa * (d0 * (float)C[0] - dm0 * (float)M0);
            acc[nt][1] += xb2 * (d0 * (float)C[1] - dm0 * (float)M1);
            acc[nt][2] += xa * (d1 * (float)C[2] - dm1 * (float)M2);
            acc[nt][3] += xb2 * (d1 * (float)C[3] - dm1 * (float)M3);
        }
        h0 = nh0;
        h1 = nh1;
#pragma unroll
        for (int c = 0; c < 4; ++c) q[c] = nq[c];
    }
    epilogue<NT>(acc, red, ks, rows, n, rt, bias, y);
}

// ---------------------------------------------------------------------------
// Q6_K
// ---------------------------------------------------------------------------
template <int NT>
__global__ void __launch_bounds__(256) gemv_q6k_kernel(const uint8_t* __restrict__ W, int64_t n, int nkb, int ks,
                                                       XPlanes p, int rows, const float* __restrict__ bias,
                                                       float* __restrict__ y) {
    extern __shared__ float red[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int64_t rt = blockIdx.x;
    const int kb0 = (int)((int64_t)nkb * warp / ks), kb1 = (int)((int64_t)nkb * (warp + 1) / ks);
    const uint8_t* recs = W + (size_t)rt * nkb * 3360;
    const int kx16 = p.kx / 16;

    float acc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int v = 0; v < 4; ++v) acc[nt][v] = 0.f;

    uint4 s0, s1, lo[4], hi[2];
    uint32_t dd0 = 0, dd1 = 0;
    auto load = [&](int kb, uint4& a0, uint4& a1, uint32_t& e0, uint32_t& e1, uint4 (&l)[4], uint4 (&h)[2]) {
        const uint8_t* rec = recs + (size_t)kb * 3360;
        a0 = __ldg(reinterpret_cast<const uint4*>(rec + 16 * g));
        a1 = __ldg(reinterpret_cast<const uint4*>(rec + 16 * (g + 8)));
        e0 = __ldg(reinterpret_cast<const unsigned short*>(rec + 256 + 2 * g));
        e1 = __ldg(reinterpret_cast<const unsigned short*>(rec + 256 + 2 * (g + 8)));
#pragma unroll
        for (int u = 0; u < 4; ++u) l[u] = ld_stream(rec + 288 + 512 * u + 16 * lane);
#pragma unroll
        for (int v = 0; v < 2; ++v) h[v] = ld_stream(rec + 2336 + 512 * v + 16 * lane);
    };
    if (kb0 < kb1) load(kb0, s0, s1, dd0, dd1, lo, hi);
    for (int kb = kb0; kb < kb1; ++kb) {
        uint4 ns0 = s0, ns1 = s1, nlo[4] = {lo[0], lo[1], lo[2], lo[3]}, nhi[2] = {hi[0], hi[1]};
        uint32_t nd0 = dd0, nd1 = dd1;
        if (kb + 1 < kb1) load(kb + 1, ns0, ns1, nd0, nd1, nlo, nhi);

        const uint32_t sw0[4] = {s0.x, s0.y, s0.z, s0.w};
        const uint32_t sw1[4] = {s1.x, s1.y, s1.z, s1.w};
        const uint32_t lw[16] = {lo[0].x, lo[0].y, lo[0].z, lo[0].w, lo[1].x, lo[1].y, lo[1].z, lo[1].w,
                                 lo[2].x, lo[2].y, lo[2].z, lo[2].w, lo[3].x, lo[3].y, lo[3].z, lo[3].w};
        const uint32_t hw[8] = {hi[0].x, hi[0].y, hi[0].z, hi[0].w, hi[1].x, hi[1].y, hi[1].z, hi[1].w};
        const float d0 = f16_bits_to_f32(dd0), d1 = f16_bits_to_f32(dd1);

#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const int colb = nt * 8 + g;
            const int8_t* xb = p.xq + (int64_t)colb * p.kx + (int64_t)kb * 256 + 4 * t;
            const int ca = nt * 8 + 2 * t, cb = ca + 1;
            const int4* sa = reinterpret_cast<const int4*>(p.s16 + (int64_t)ca * kx16 + (int64_t)kb * 16);
            const int4* sb = reinterpret_cast<const int4*>(p.s16 + (int64_t)cb * kx16 + (int64_t)kb * 16);
            int C[4] = {0, 0, 0, 0}, Mn[4] = {0, 0, 0, 0};
#pragma unroll
            for (int j4 = 0; j4 < 4; ++j4) {
                const int4 A = __ldg(sa + j4), B = __ldg(sb + j4);
                const int SA[4] = {A.x, A.y, A.z, A.w}, SB[4] = {B.x, B.y, B.z, B.w};
#pragma unroll
                for (int jj = 0; jj < 4; ++jj) {
                    const int j = 4 * j4 + jj;
                    const uint32_t w = lw[j], h = hw[j >> 1];
                    uint32_t a0, a1;
                    if ((j & 1) == 0) {
                        a0 = (w & 0x0F0F0F0Fu) | ((h << 4) & 0x30303030u);
                        a1 = ((w >> 4) & 0x0F0F0F0Fu) | ((h << 2) & 0x30303030u);
                    } else {
                        a0 = (w & 0x0F0F0F0Fu) | (h & 0x30303030u);
                        a1 = ((w >> 4) & 0x0F0F0F0Fu) | ((h >> 2) & 0x30303030u);
                    }
                    const uint32_t b0 = __ldg(reinterpret_cast<const uint32_t*>(xb + 16 * j));
                    int r[4];
                    mma_k16(r, a0, a1, b0);
                    const int scg = (int)(int8_t)(sw0[j >> 2] >> (8 * (j & 3)));
                    const int sch = (int)(int8_t)(sw1[j >> 2] >> (8 * (j & 3)));
                    C[0] += scg * r[0];
                    C[1] += scg * r[1];
                    C[2] += sch * r[2];
                    C[3] += sch * r[3];
                    Mn[0] += scg * SA[jj];
                    Mn[1] += scg * SB[jj];
                    Mn[2] += sch * SA[jj];
                    Mn[3] += sch * SB[jj];
                }
            }
            const float xa = __ldg(p.xs + (int64_t)(ca / 3) * (p.kx / 256) + kb);
            const float xb2 = __ldg(p.xs + (int64_t)(cb / 3) * (p.kx / 256) + kb);
            acc[nt][0] += xa * (d0 * (float)(C[0] - 32 * Mn[0]));
            acc[nt][1] += xb2 * (d0 * (float)(C[1] - 32 * Mn[1]));
            acc[nt][2] += xa * (d1 * (float)(C[2] - 32 * Mn[2]));
            acc[nt][3] += xb2 * (d1 * (float)(C[3] - 32 * Mn[3]));
        }
        s0 = ns0;
        s1 = ns1;
        dd0 = nd0;
        dd1 = nd1;
#pragma unroll
        for (int u = 0; u < 4; ++u) lo[u] = nlo[u];
        hi[0] = nhi[0];
        hi[1] = nhi[1];
    }
    epilogue<NT>(acc, red, ks, rows, n, rt, bias, y);
}

// ---------------------------------------------------------------------------
// Q8_0 (records of 16 rows x 32 k; a warp step covers 8 records = 256 k)
// ---------------------------------------------------------------------------
template <int NT>
__global__ void __launch_bounds__(256) gemv_q80_kernel(const uint8_t* __restrict__ W, int64_t n, int nkb, int ks,
                                                       XPlanes p, int rows, const float* __restrict__ bias,
                                                       float* __restrict__ y) {
    extern __shared__ float red[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int64_t rt = blockIdx.x;
    const int ngrp = (nkb + 7) / 8;
    const int gr0 = (int)((int64_t)ngrp * warp / ks), gr1 = (int)((int64_t)ngrp * (warp + 1) / ks);
    const uint8_t* recs = W + (size_t)rt * nkb * 544;

    float acc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int v = 0; v < 4; ++v) acc[nt][v] = 0.f;

    for (int gr = gr0; gr < gr1; ++gr) {
        const int b0 = gr * 8, nb = min(8, nkb - b0);
        uint4 q[8];
        uint32_t e0[8], e1[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            if (i < nb) {
                const uint8_t* rec = recs + (size_t)(b0 + i) * 544;
                q[i] = ld_stream(rec + 32 + 16 * lane);
                e0[i] = __ldg(reinterpret_cast<const unsigned short*>(rec + 2 * g));
                e1[i] = __ldg(reinterpret_cast<const unsigned short*>(rec + 2 * (g + 8)));
            } else {
                q[i] = make_uint4(0, 0, 0, 0);
                e0[i] = e1[i] = 0;
            }
        }
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const int colb = nt * 8 + g;
            const int ca = nt * 8 + 2 * t, cb = ca + 1;
            const float xa = __ldg(p.xs + (int64_t)(ca / 3) * (p.kx / 256) + gr);
            const float xb2 = __ldg(p.xs + (int64_t)(cb / 3) * (p.kx / 256) + gr);
            float blk[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                if (i < nb) {
                    const int8_t* xb = p.xq + (int64_t)colb * p.kx + (int64_t)(b0 + i) * 32 + 4 * t;
                    const uint32_t bx = __ldg(reinterpret_cast<const uint32_t*>(xb));
                    const uint32_t by = __ldg(reinterpret_cast<const uint32_t*>(xb + 16));
                    int r[4];
                    mma_k32(r, q[i].x, q[i].y, q[i].z, q[i].w, bx, by);
                    const float dg = f16_bits_to_f32(e0[i]), dh = f16_bits_to_f32(e1[i]);
                    blk[0] += dg * (float)r[0];
                    blk[1] += dg * (float)r[1];
                    blk[2] += dh * (float)r[2];
                    blk[3] += dh * (float)r[3];
                }
            }
            acc[nt][0] += xa * blk[0];
            acc[nt][1] += xb2 * blk[1];
            acc[nt][2] += xa * blk[2];
            acc[nt][3] += xb2 * blk[3];
        }
    }
    epilogue<NT>(acc, red, ks, rows, n, rt, bias, y);
}

template <int NT>
cudaError_t launch_nt(int type, const void* tiles, int64_t n, int64_t k, const XPlanes& p, int rows,
                      const float* bias, float* y, int sms, cudaStream_t s) {
    const int64_t n_rt = (n + 15) / 16;
    const int units = type == kQ8_0 ? (int)((k / 32 + 7) / 8) : (int)(k / 256);
    // enough warps to keep ~16 per SM streaming, at most 8 per CTA
    int64_t ks = (int64_t)sms * 16 / n_rt;
    if (ks < 1) ks = 1;
    if (ks > 8) ks = 8;
    if (ks > units) ks = units;
    const size_t smem = (size_t)ks * 16 * NT * 8 * sizeof(float);
    const dim3 grid((unsigned)n_rt), block((unsigned)(32 * ks));
    const uint8_t* w = (const uint8_t*)tiles;
    if (type == kQ4_K)
        gemv_q4k_kernel<NT><<<grid, block, smem, s>>>(w, n, (int)(k / 256), (int)ks, p, rows, bias, y);
    else if (type == kQ6_K)
        gemv_q6k_kernel<NT><<<grid, block, smem, s>>>(w, n, (int)(k / 256), (int)ks, p, rows, bias, y);
    else
        gemv_q80_kernel<NT><<<grid, block, smem, s>>>(w, n, (int)(k / 32), (int)ks, p, rows, bias, y);
    return cudaGetLastError();
}

}  // namespace

XPlanes xplanes_carve(void* base, int64_t k) {
    XPlanes p;
    p.kx = (int)((k + 255) / 256 * 256);
    uintptr_t a = ((uintptr_t)base + 255) & ~(uintptr_t)255;
    auto take = [&](size_t bytes) {
        void* r = (void*)a;
        a = (a + bytes + 255) & ~(uintptr_t)255;
        return r;
    };
    p.xq = (int8_t*)take((size_t)kColsMax * p.kx);
    p.s16 = (int32_t*)take((size_t)kColsMax * (p.kx / 16) * 4);
    p.s32 = (int32_t*)take((size_t)kColsMax * (p.kx / 32) * 4);
    p.xs = (float*)take((size_t)kRowsMax * (p.kx / 256) * 4);
    return p;
}

cudaError_t launch_xsplit(const float* x, int rows, int64_t k, const XPlanes& p, cudaStream_t s) {
    const int nt = (3 * rows + 7) / 8;
    const int mpad = (nt * 8 + 2) / 3;  // activation rows whose planes the GEMV reads
    xsplit_kernel<<<dim3((unsigned)(p.kx / 256), (unsigned)mpad), 32, 0, s>>>(x, rows, k, p);
    return cudaGetLastError();
}

cudaError_t launch_gemv(int type, const void* tiles, int64_t n, int64_t k, const XPlanes& p, int rows,
                        const float* bias, float* y, int sms, cudaStream_t s) {
    switch ((3 * rows + 7) / 8) {
        case 1: return launch_nt<1>(type, tiles, n, k, p, rows, bias, y, sms, s);
        case 2: return launch_nt<2>(type, tiles, n, k, p, rows, bias, y, sms, s);
        case 3: return launch_nt<3>(type, tiles, n, k, p, rows, bias, y, sms, s);
        case 4: return launch_nt<4>(type, tiles, n, k, p, rows, bias, y, sms, s);
        case 5: return launch_nt<5>(type, tiles, n, k, p, rows, bias, y, sms, s);
        case 6: return launch_nt<6>(type, tiles, n, k, p, rows, bias, y, sms, s);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace ocl
