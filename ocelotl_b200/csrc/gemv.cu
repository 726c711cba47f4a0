// gemv.cu -- decode-time (M = 1..16) fused dequantize-and-multiply.
//
// y[m, n] = bias[n] + sum_k x[m, k] * W[n, k] with W in TILED16 records.
//
// Design (B200, HBM-bound):
//  * A tiny split kernel turns x into three int8 planes per row with one
//    power-of-two scale per 256-k block (x = xs * (p0 + p1/2^7 + p2/2^14),
//    |error| < 2^-21 of the block max) plus exact per-16 / per-32 plane sums,
//    once per call, into scratch memory.
//  * GEMV CTAs of 8 warps = RT row tiles x KW warps per row tile.  Every warp
//    streams its (row tile, K slice) records through a private two-stage
//    shared-memory ring filled by bulk asynchronous copies (cp.async.bulk, the
//    non-tensor TMA path) completing on mbarriers; records are contiguous per
//    row tile, so one copy moves one 256-k unit (2304 / 3360 / 4352 bytes).
//    The CTA's slice of the activation planes is bulk-copied into shared memory
//    once and shared by its warps; the KW partial sums of a row tile are added
//    in shared memory.
//  * The GGUF quants are small integers, so the inner products are exact
//    int8 x int8 -> int32 tensor-core MMAs (mma.sync m16n8k32 / m16n8k16): each
//    lane's 16-byte chunk of a record IS its A fragment after one mask (the
//    high Q4_K nibbles run as u8 x s8 at 16x scale).  The only rounding is the
//    per-super-block f32 scaling:
//        Q4_K: acc += xs * (d/16 * float(sum_j sc'_j*c_j) - dmin * float(sum_j m_j*S_j))
//        Q6_K: acc += xs * d * float(sum_j sc_j*(c_j - 32*S_j))
//        Q8_0: acc += xs * sum_b d_b * float(c_b)
//  * For one activation row the three planes sit in MMA columns 0, 2, 4 so each
//    lane keeps only its two useful accumulators.
//  * Narrow matrices also split K across CTAs; those partial sums go through
//    scratch memory and the last CTA of each row group adds them in split order
//    (one counter per group).  Every reduction has a fixed order: deterministic.
//  * Both kernels launch with programmatic dependent launch and the split
//    kernel releases its dependent at once, so a GEMV starts while its
//    predecessors run and fills its rings before griddepcontrol.wait; planes,
//    partials and counters are touched only after the wait.  (Prefetching the
//    whole weight slice into L2 there measured slower and is not done.)
//  * Every mbarrier wait is bounded; a wait that gives up bumps an error counter
//    the host reads (ocl_take_device_errors), drains its own copies and returns.
#include <cuda_fp16.h>

#include <cstdlib>

#include "internal.cuh"

namespace ocl {

namespace {

constexpr int kWarps = 8;   // warps per CTA
// Ring depth per warp, by weight type and layout.  Measured on B200 (Llama-shaped
// matrices, same-box A/B): for a single row, 4 stages beat 2 for Q4_K (2.3 KB
// records) by 0.3-0.6 us per call; for Q6_K (3.3 KB records, 43 KB of planes
// at K = 14336) more than 2 stages cost CTAs per SM and ran slower; Q8_0 units
// are 4.3 KB; with two or more rows (bigger planes) 4 stages lost ~20%.  A
// single-row Q4_K CTA whose K range exceeds 32 units (K = 14336: 43 KB of
// planes) also runs 2 stages, which keeps two CTAs per SM: Q4_K 4096 x 14336
// 11.7 -> 10.1 us (the same change cost 0.2-0.9 us at K = 4096).
constexpr int kLongKUnits = 32;
__host__ __device__ constexpr int stages(int t, int nt, int umax) {
    return (t == kQ4_K && nt == 0 && umax <= kLongKUnits) ? 4 : 2;
}

__host__ __device__ constexpr int unit_bytes(int t) { return t == kQ4_K ? 2304 : t == kQ6_K ? 3360 : 4352; }
__host__ __device__ constexpr int sum_per(int t) { return t == kQ4_K ? 8 : t == kQ6_K ? 16 : 0; }

// ---- PTX helpers ------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Wait with a time limit (~1 s of SM clocks).  Returns false if it gave up.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity))
        if (clock64() - t0 > 2000000000LL) return false;
    return true;
}
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ void mma_s8_k32(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                           uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}
__device__ __forceinline__ void mma_u8_k32(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                           uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}
__device__ __forceinline__ void mma_s8_k16(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, "
        "{%7,%7,%7,%7};"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a0), "r"(a1), "r"(b0), "r"(0));
}
__device__ __forceinline__ float h2f(uint32_t bits) { return __half2float(__ushort_as_half((unsigned short)bits)); }
__device__ __forceinline__ int prmt(uint32_t w, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, 0, %2;" : "=r"(r) : "r"(w), "r"(sel));
    return (int)r;
}
// byte i of w, sign-extended (selector msb = replicate the sign bit)
__device__ __forceinline__ int sext_byte(uint32_t w, int i) {
    return prmt(w, (uint32_t)(i | ((8 + i) << 4) | ((8 + i) << 8) | ((8 + i) << 12)));
}
// byte i of w, zero-extended (selector 4 picks a byte of the zero operand)
__device__ __forceinline__ int zext_byte(uint32_t w, int i) {
    return prmt(w, (uint32_t)(i | (4 << 4) | (4 << 8) | (4 << 12)));
}

// ---------------------------------------------------------------------------
// Activation split: x [rows, k] f32 -> three int8 planes per row (global), one
// warp per (row m, 256-k block b).  Rows past `rows` up to mpad are written as
// zeros (they feed idle MMA columns).  |x / xs| < 2^7 with xs = 2^e per block.
// ---------------------------------------------------------------------------
// `sums` selects which plane sums the GEMV that follows reads (bit 0 per-16
// ints, 1 per-32 ints, 2 per-16 byte pieces, 3 per-32 byte pieces); the others
// are not written.
__global__ void xsplit_kernel(const float* __restrict__ x, int rows, int64_t k, XPlanes p, int sums) {
    // Let the GEMV that follows launch now: it only streams weights until it
    // waits for this kernel.  This kernel itself must wait for its predecessor:
    // x is that kernel's output and the planes may still be read by it.
    pdl_trigger();
    pdl_wait();
    const int b = blockIdx.x, m = blockIdx.y, lane = threadIdx.x;
    const int64_t k0 = (int64_t)b * 256 + lane * 8;
    float v[8];
    // vector loads only where the row start is 16-byte aligned (any f32 pointer is accepted)
    if (m < rows && (k & 3) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 && k0 + 8 <= k) {
        const float4 a = *reinterpret_cast<const float4*>(x + (int64_t)m * k + k0);
        const float4 c = *reinterpret_cast<const float4*>(x + (int64_t)m * k + k0 + 4);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = c.x; v[5] = c.y; v[6] = c.z; v[7] = c.w;
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = (m < rows && k0 + i < k) ? x[(int64_t)m * k + k0 + i] : 0.0f;
    }
    float amax = 0.0f;
    bool finite = true;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        amax = fmaxf(amax, fabsf(v[i]));
        finite = finite && (fabsf(v[i]) <= 3.402823466e38f);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    finite = __all_sync(0xffffffffu, finite);
    // amax < 2^E with E = biased exponent - 126; scale so that |v| < 2^7
    int e = 0;
    if (finite && amax > 0.0f) e = max((int)((__float_as_uint(amax) >> 23) & 0xff) - 126 - 7, -100);
    const float scale = __uint_as_float((uint32_t)(127 - e) << 23);  // 2^-e, exact
    uint32_t pk[3][2] = {{0, 0}, {0, 0}, {0, 0}};
    int sum[3] = {0, 0, 0};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float sv = finite ? v[i] * scale : 0.0f;
        const float x0 = truncf(sv);
        const float r1 = (sv - x0) * 128.0f;
        const float x1 = truncf(r1);
        const float x2 = fminf(fmaxf(rintf((r1 - x1) * 128.0f), -127.0f), 127.0f);
        const int q0 = (int)x0, q1 = (int)x1, q2 = (int)x2;
        pk[0][i >> 2] |= (uint32_t)(q0 & 0xFF) << (8 * (i & 3));
        pk[1][i >> 2] |= (uint32_t)(q1 & 0xFF) << (8 * (i & 3));
        pk[2][i >> 2] |= (uint32_t)(q2 & 0xFF) << (8 * (i & 3));
        sum[0] += q0;
        sum[1] += q1;
        sum[2] += q2;
    }
#pragma unroll
    for (int sp = 0; sp < 3; ++sp) {
        const int c = 3 * m + sp;
        *reinterpret_cast<uint2*>(p.xq + (int64_t)c * p.kx + k0) = make_uint2(pk[sp][0], pk[sp][1]);
        int s = sum[sp] + __shfl_xor_sync(0xffffffffu, sum[sp], 1);
        if ((lane & 1) == 0) {
            const int j = lane >> 1;
            if (sums & 1) p.s16[(int64_t)c * (p.kx / 16) + b * 16 + j] = s;
            if (sums & 4) {
                int8_t* pc = p.p16 + ((int64_t)c * (p.kx / 256) + b) * 32;
                pc[j] = (int8_t)(s & 63);        // s = lo + 64 * hi, lo in 0..63
                pc[16 + j] = (int8_t)(s >> 6);   // |s| <= 2032 -> hi in -32..31
            }
        }
        s += __shfl_xor_sync(0xffffffffu, s, 2);
        if ((lane & 3) == 0) {
            const int j = lane >> 2;
            if (sums & 2) p.s32[(int64_t)c * (p.kx / 32) + b * 8 + j] = s;
            if (sums & 8) {
                int8_t* pc = p.p32 + ((int64_t)c * (p.kx / 256) + b) * 16;
                pc[j] = (int8_t)(s & 63);
                pc[8 + j] = (int8_t)(s >> 6);    // |s| <= 4064 -> hi in -64..63
            }
        }
    }
    if (lane == 0)
        p.xs[(int64_t)m * (p.kx / 256) + b] =
            finite ? __uint_as_float((uint32_t)(127 + e) << 23) : __uint_as_float(0x7fc00000u);
}

// Shared-memory view of the activation planes of one CTA's K range.
struct XSmem {
    int8_t* q;   // [ncp][qstride]  plane c = 3m + s, natural k order
    int32_t* s;  // [ncp][sstride]  per-32 (Q4_K) / per-16 (Q6_K) sums of each plane as lo (0..63) and hi
                 //                 byte pieces, per unit lo[0..n) then hi[0..n) (sstride in ints)
    float* xs;   // [mpad][umax]    block scales 2^e
    int qstride, sstride, umax;
};

// ---- per-unit consumers, general layout (rows >= 2) ---------------------------
// Columns 3m+s of the n8 tiles hold plane s of activation row m; lane (g, t)
// owns rows g, g+8 x columns 2t, 2t+1 of each tile.
template <int NT>
__device__ __forceinline__ void consume_q4k(const uint8_t* rec, int l, const XSmem& X, float (&acc)[NT][4], int g,
                                            int t, int lane) {
    const uint4 h0 = *reinterpret_cast<const uint4*>(rec + 16 * g);
    const uint4 h1 = *reinterpret_cast<const uint4*>(rec + 16 * (g + 8));
    uint4 q[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) q[c] = *reinterpret_cast<const uint4*>(rec + 256 + 512 * c + 16 * lane);
    // 6-bit scales / mins, byte j of each word (rows g: *0, g+8: *1)
    const uint32_t sc0[2] = {h0.y & 0x3F3F3F3Fu, (h0.w & 0x0F0F0F0Fu) | ((h0.y >> 2) & 0x30303030u)};
    const uint32_t mn0[2] = {h0.z & 0x3F3F3F3Fu, ((h0.w >> 4) & 0x0F0F0F0Fu) | ((h0.z >> 2) & 0x30303030u)};
    const uint32_t sc1[2] = {h1.y & 0x3F3F3F3Fu, (h1.w & 0x0F0F0F0Fu) | ((h1.y >> 2) & 0x30303030u)};
    const uint32_t mn1[2] = {h1.z & 0x3F3F3F3Fu, ((h1.w >> 4) & 0x0F0F0F0Fu) | ((h1.z >> 2) & 0x30303030u)};
    const float d0 = h2f(h0.x & 0xffffu) * 0.0625f, dm0 = h2f(h0.x >> 16);
    const float d1 = h2f(h1.x & 0xffffu) * 0.0625f, dm1 = h2f(h1.x >> 16);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        const int8_t* xb = X.q + (nt * 8 + g) * X.qstride + l * 256 + 8 * t;
        int L0 = 0, L1 = 0, L2 = 0, L3 = 0, H0 = 0, H1 = 0, H2 = 0, H3 = 0;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const uint2 bl = *reinterpret_cast<const uint2*>(xb + 64 * c);
            const uint2 bh = *reinterpret_cast<const uint2*>(xb + 64 * c + 32);
            int r[4], u[4];
            mma_s8_k32(r, q[c].x & 0x0F0F0F0Fu, q[c].z & 0x0F0F0F0Fu, q[c].y & 0x0F0F0F0Fu, q[c].w & 0x0F0F0F0Fu,
                       bl.x, bl.y);
            // high nibbles in place: u8 values 16*q
            mma_u8_k32(u, q[c].x & 0xF0F0F0F0u, q[c].z & 0xF0F0F0F0u, q[c].y & 0xF0F0F0F0u, q[c].w & 0xF0F0F0F0u,
                       bh.x, bh.y);
            const int j0 = 2 * c, j1 = 2 * c + 1;
            const int s0l = zext_byte(sc0[j0 >> 2], j0 & 3), s0h = zext_byte(sc0[j1 >> 2], j1 & 3);
            const int s1l = zext_byte(sc1[j0 >> 2], j0 & 3), s1h = zext_byte(sc1[j1 >> 2], j1 & 3);
            L0 += s0l * r[0];
            L1 += s0l * r[1];
            L2 += s1l * r[2];
            L3 += s1l * r[3];
            H0 += s0h * u[0];
            H1 += s0h * u[1];
            H2 += s1h * u[2];
            H3 += s1h * u[3];
        }
        const int ca = nt * 8 + 2 * t, cb = ca + 1;
        // min term sum_j m_j * S_j on the tensor core: A = the mins (k = j, 8 of
        // 16 used), B column g = plane column nt*8+g's per-32 sums as lo (0..63)
        // and hi bytes, one MMA each: M = lo + 64 * hi, exact.
        int ml[4], mh[4];
        {
            const int8_t* pr = reinterpret_cast<const int8_t*>(X.s + (nt * 8 + g) * X.sstride) + l * 16 + 4 * t;
            const uint32_t blo = t < 2 ? *reinterpret_cast<const uint32_t*>(pr) : 0u;
            const uint32_t bhi = t < 2 ? *reinterpret_cast<const uint32_t*>(pr + 8) : 0u;
            const uint32_t a0 = t < 2 ? mn0[t & 1] : 0u, a1 = t < 2 ? mn1[t & 1] : 0u;
            mma_s8_k16(ml, a0, a1, blo);
            mma_s8_k16(mh, a0, a1, bhi);
        }
        const int M0 = ml[0] + 64 * mh[0], M1 = ml[1] + 64 * mh[1], M2 = ml[2] + 64 * mh[2], M3 = ml[3] + 64 * mh[3];
        const float xa = X.xs[(ca / 3) * X.umax + l], xb2 = X.xs[(cb / 3) * X.umax + l];
        acc[nt][0] += xa * (d0 * (float)(16 * L0 + H0) - dm0 * (float)M0);
        acc[nt][1] += xb2 * (d0 * (float)(16 * L1 + H1) - dm0 * (float)M1);
        acc[nt][2] += xa * (d1 * (float)(16 * L2 + H2) - dm1 * (float)M2);
        acc[nt][3] += xb2 * (d1 * (float)(16 * L3 + H3) - dm1 * (float)M3);
    }
}

// A operands of Q6_K sub-block j from the low-nibble word w and crumb word h.
__device__ __forceinline__ void q6_frag(int j, uint32_t w, uint32_t h, uint32_t& a0, uint32_t& a1) {
    if ((j & 1) == 0) {
        a0 = (w & 0x0F0F0F0Fu) | ((h << 4) & 0x30303030u);
        a1 = ((w >> 4) & 0x0F0F0F0Fu) | ((h << 2) & 0x30303030u);
    } else {
        a0 = (w & 0x0F0F0F0Fu) | (h & 0x30303030u);
        a1 = ((w >> 4) & 0x0F0F0F0Fu) | ((h >> 2) & 0x30303030u);
    }
}

template <int NT>
__device__ __forceinline__ void consume_q6k(const uint8_t* rec, int l, const XSmem& X, float (&acc)[NT][4], int g,
                                            int t, int lane) {
    const uint4 s0 = *reinterpret_cast<const uint4*>(rec + 16 * g);
    const uint4 s1 = *reinterpret_cast<const uint4*>(rec + 16 * (g + 8));
    const float d0 = h2f(*reinterpret_cast<const unsigned short*>(rec + 256 + 2 * g));
    const float d1 = h2f(*reinterpret_cast<const unsigned short*>(rec + 256 + 2 * (g + 8)));
    uint4 lo[4], hi[2];
#pragma unroll
    for (int u = 0; u < 4; ++u) lo[u] = *reinterpret_cast<const uint4*>(rec + 288 + 512 * u + 16 * lane);
#pragma unroll
    for (int v = 0; v < 2; ++v) hi[v] = *reinterpret_cast<const uint4*>(rec + 2336 + 512 * v + 16 * lane);
    const uint32_t sw0[4] = {s0.x, s0.y, s0.z, s0.w};
    const uint32_t sw1[4] = {s1.x, s1.y, s1.z, s1.w};
    const uint32_t lw[16] = {lo[0].x, lo[0].y, lo[0].z, lo[0].w, lo[1].x, lo[1].y, lo[1].z, lo[1].w,
                             lo[2].x, lo[2].y, lo[2].z, lo[2].w, lo[3].x, lo[3].y, lo[3].z, lo[3].w};
    const uint32_t hw[8] = {hi[0].x, hi[0].y, hi[0].z, hi[0].w, hi[1].x, hi[1].y, hi[1].z, hi[1].w};
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        const int8_t* xb = X.q + (nt * 8 + g) * X.qstride + l * 256 + 4 * t;
        const int ca = nt * 8 + 2 * t, cb = ca + 1;
        int C[4] = {0, 0, 0, 0};
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            uint32_t a0, a1;
            q6_frag(j, lw[j], hw[j >> 1], a0, a1);
            const uint32_t b0 = *reinterpret_cast<const uint32_t*>(xb + 16 * j);
            int r[4];
            mma_s8_k16(r, a0, a1, b0);
            const int scg = sext_byte(sw0[j >> 2], j & 3), sch = sext_byte(sw1[j >> 2], j & 3);
            C[0] += scg * r[0];
            C[1] += scg * r[1];
            C[2] += sch * r[2];
            C[3] += sch * r[3];
        }
        // offset term sum_j sc_j * S_j on the tensor core: A = the 16 int8
        // scales, B column g = plane column nt*8+g's per-16 sums as lo / hi
        // bytes; C -= 32 * (lo + 64 * hi), exact.
        {
            const int8_t* pr = reinterpret_cast<const int8_t*>(X.s + (nt * 8 + g) * X.sstride) + l * 32 + 4 * t;
            int ol[4], oh[4];
            mma_s8_k16(ol, sw0[t], sw1[t], *reinterpret_cast<const uint32_t*>(pr));
            mma_s8_k16(oh, sw0[t], sw1[t], *reinterpret_cast<const uint32_t*>(pr + 16));
#pragma unroll
            for (int i = 0; i < 4; ++i) C[i] -= 32 * (ol[i] + 64 * oh[i]);
        }
        const float xa = X.xs[(ca / 3) * X.umax + l], xb2 = X.xs[(cb / 3) * X.umax + l];
        acc[nt][0] += xa * (d0 * (float)C[0]);
        acc[nt][1] += xb2 * (d0 * (float)C[1]);
        acc[nt][2] += xa * (d1 * (float)C[2]);
        acc[nt][3] += xb2 * (d1 * (float)C[3]);
    }
}

// Q8_0 unit = up to 8 consecutive 544-byte records (16 rows x 32 k each).
template <int NT>
__device__ __forceinline__ void consume_q80(const uint8_t* rec, int l, int nb, const XSmem& X, float (&acc)[NT][4],
                                            int g, int t, int lane) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        const int8_t* xb = X.q + (nt * 8 + g) * X.qstride + l * 256 + 4 * t;
        float blk[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            if (i < nb) {
                const uint8_t* r8 = rec + 544 * i;
                const uint4 q = *reinterpret_cast<const uint4*>(r8 + 32 + 16 * lane);
                const float dg = h2f(*reinterpret_cast<const unsigned short*>(r8 + 2 * g));
                const float dh = h2f(*reinterpret_cast<const unsigned short*>(r8 + 2 * (g + 8)));
                const uint32_t bx = *reinterpret_cast<const uint32_t*>(xb + 32 * i);
                const uint32_t by = *reinterpret_cast<const uint32_t*>(xb + 32 * i + 16);
                int r[4];
                mma_s8_k32(r, q.x, q.y, q.z, q.w, bx, by);
                blk[0] += dg * (float)r[0];
                blk[1] += dg * (float)r[1];
                blk[2] += dh * (float)r[2];
                blk[3] += dh * (float)r[3];
            }
        }
        const int ca = nt * 8 + 2 * t, cb = ca + 1;
        const float xa = X.xs[(ca / 3) * X.umax + l], xb2 = X.xs[(cb / 3) * X.umax + l];
        acc[nt][0] += xa * blk[0];
        acc[nt][1] += xb2 * blk[1];
        acc[nt][2] += xa * blk[2];
        acc[nt][3] += xb2 * blk[3];
    }
}

// ---- single activation row (M = 1) -----------------------------------------
// The three planes sit in MMA columns 0, 2 and 4 (lane t's even column 2t holds
// plane t for t < 3); the other columns' B fragments are zero registers.  Each lane then
// keeps only its two useful accumulators (rows g and g+8, plane t).
__device__ __forceinline__ int m1_bplane(int g) { return ((g & 1) == 0 && g < 6) ? (g >> 1) : 0; }
__device__ __forceinline__ bool m1_bidle(int g) { return (g & 1) || g >= 6; }  // MMA column reads zeros
__device__ __forceinline__ uint32_t ld_b32(const int8_t* p, bool idle) {
    return idle ? 0u : *reinterpret_cast<const uint32_t*>(p);
}
__device__ __forceinline__ uint2 ld_b64(const int8_t* p, bool idle) {
    return idle ? make_uint2(0u, 0u) : *reinterpret_cast<const uint2*>(p);
}

__device__ __forceinline__ void consume_q4k_m1(const uint8_t* rec, int l, const XSmem& X, float& acc0,
                                               float& acc2, int g, int t, int lane) {
    const int8_t* xb = X.q + m1_bplane(g) * X.qstride + l * 256 + 8 * t;
    const bool bidle = m1_bidle(g);
    const uint4 h0 = *reinterpret_cast<const uint4*>(rec + 16 * g);
    const uint4 h1 = *reinterpret_cast<const uint4*>(rec + 16 * (g + 8));
    uint4 q[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) q[c] = *reinterpret_cast<const uint4*>(rec + 256 + 512 * c + 16 * lane);
    const uint32_t sc0[2] = {h0.y & 0x3F3F3F3Fu, (h0.w & 0x0F0F0F0Fu) | ((h0.y >> 2) & 0x30303030u)};
    const uint32_t mn0[2] = {h0.z & 0x3F3F3F3Fu, ((h0.w >> 4) & 0x0F0F0F0Fu) | ((h0.z >> 2) & 0x30303030u)};
    const uint32_t sc1[2] = {h1.y & 0x3F3F3F3Fu, (h1.w & 0x0F0F0F0Fu) | ((h1.y >> 2) & 0x30303030u)};
    const uint32_t mn1[2] = {h1.z & 0x3F3F3F3Fu, ((h1.w >> 4) & 0x0F0F0F0Fu) | ((h1.z >> 2) & 0x30303030u)};
    int lo0 = 0, hi0 = 0, lo2 = 0, hi2 = 0;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const uint2 bl = ld_b64(xb + 64 * c, bidle);
        const uint2 bh = ld_b64(xb + 64 * c + 32, bidle);
        int r[4], u[4];
        mma_s8_k32(r, q[c].x & 0x0F0F0F0Fu, q[c].z & 0x0F0F0F0Fu, q[c].y & 0x0F0F0F0Fu, q[c].w & 0x0F0F0F0Fu, bl.x,
                   bl.y);
        mma_u8_k32(u, q[c].x & 0xF0F0F0F0u, q[c].z & 0xF0F0F0F0u, q[c].y & 0xF0F0F0F0u, q[c].w & 0xF0F0F0F0u, bh.x,
                   bh.y);
        const int j0 = 2 * c, j1 = 2 * c + 1;
        lo0 += zext_byte(sc0[j0 >> 2], j0 & 3) * r[0];
        hi0 += zext_byte(sc0[j1 >> 2], j1 & 3) * u[0];
        lo2 += zext_byte(sc1[j0 >> 2], j0 & 3) * r[2];
        hi2 += zext_byte(sc1[j1 >> 2], j1 & 3) * u[2];
    }
    // min term sum_j m_j * S_j on the tensor core: A = mins (k = j, 8 of 16 used),
    // B column 2p + h = piece h (lo / hi byte) of plane p's sums, so lane t gets
    // plane t's lo and hi results side by side: M = lo + 64 * hi, exact.
    int mm[4];
    {
        const int8_t* pr = reinterpret_cast<const int8_t*>(X.s + (g < 6 ? (g >> 1) : 0) * X.sstride);
        const uint32_t bm = ld_b32(pr + l * 16 + (g & 1) * 8 + 4 * t, t >= 2 || g >= 6);
        mma_s8_k16(mm, t < 2 ? mn0[t & 1] : 0u, t < 2 ? mn1[t & 1] : 0u, bm);
    }
    const int M0 = mm[0] + 64 * mm[1], M2 = mm[2] + 64 * mm[3];
    const float xs = X.xs[l];
    const float d0 = h2f(h0.x & 0xffffu) * 0.0625f, dm0 = h2f(h0.x >> 16);
    const float d1 = h2f(h1.x & 0xffffu) * 0.0625f, dm1 = h2f(h1.x >> 16);
    acc0 += xs * (d0 * (float)(16 * lo0 + hi0) - dm0 * (float)M0);
    acc2 += xs * (d1 * (float)(16 * lo2 + hi2) - dm1 * (float)M2);
}

__device__ __forceinline__ void consume_q6k_m1(const uint8_t* rec, int l, const XSmem& X, float& acc0,
                                               float& acc2, int g, int t, int lane) {
    const int8_t* xb = X.q + m1_bplane(g) * X.qstride + l * 256 + 4 * t;
    const bool bidle = m1_bidle(g);
    const uint4 s0 = *reinterpret_cast<const uint4*>(rec + 16 * g);
    const uint4 s1 = *reinterpret_cast<const uint4*>(rec + 16 * (g + 8));
    uint4 lo[4], hi[2];
#pragma unroll
    for (int u = 0; u < 4; ++u) lo[u] = *reinterpret_cast<const uint4*>(rec + 288 + 512 * u + 16 * lane);
#pragma unroll
    for (int v = 0; v < 2; ++v) hi[v] = *reinterpret_cast<const uint4*>(rec + 2336 + 512 * v + 16 * lane);
    const uint32_t sw0[4] = {s0.x, s0.y, s0.z, s0.w};
    const uint32_t sw1[4] = {s1.x, s1.y, s1.z, s1.w};
    const uint32_t lw[16] = {lo[0].x, lo[0].y, lo[0].z, lo[0].w, lo[1].x, lo[1].y, lo[1].z, lo[1].w,
                             lo[2].x, lo[2].y, lo[2].z, lo[2].w, lo[3].x, lo[3].y, lo[3].z, lo[3].w};
    const uint32_t hw[8] = {hi[0].x, hi[0].y, hi[0].z, hi[0].w, hi[1].x, hi[1].y, hi[1].z, hi[1].w};
    int C0 = 0, C2 = 0;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        uint32_t a0, a1;
        q6_frag(j, lw[j], hw[j >> 1], a0, a1);
        const uint32_t b0 = ld_b32(xb + 16 * j, bidle);
        int r[4];
        mma_s8_k16(r, a0, a1, b0);
        C0 += sext_byte(sw0[j >> 2], j & 3) * r[0];
        C2 += sext_byte(sw1[j >> 2], j & 3) * r[2];
    }
    // offset term sum_j sc_j * S_j on the tensor core (A = the 16 int8 scales,
    // B column 2p + h = piece h of plane p's per-16 sums): lo + 64 * hi
    {
        const int8_t* pr = reinterpret_cast<const int8_t*>(X.s + (g < 6 ? (g >> 1) : 0) * X.sstride);
        const uint32_t bm = ld_b32(pr + l * 32 + (g & 1) * 16 + 4 * t, g >= 6);
        int mm[4];
        mma_s8_k16(mm, sw0[t], sw1[t], bm);
        C0 -= 32 * (mm[0] + 64 * mm[1]);
        C2 -= 32 * (mm[2] + 64 * mm[3]);
    }
    const float xs = X.xs[l];
    const float d0 = h2f(*reinterpret_cast<const unsigned short*>(rec + 256 + 2 * g));
    const float d1 = h2f(*reinterpret_cast<const unsigned short*>(rec + 256 + 2 * (g + 8)));
    acc0 += xs * (d0 * (float)C0);
    acc2 += xs * (d1 * (float)C2);
}

__device__ __forceinline__ void consume_q80_m1(const uint8_t* rec, int l, int nb, const XSmem& X, float& acc0,
                                               float& acc2, int g, int t, int lane) {
    const int8_t* xb = X.q + m1_bplane(g) * X.qstride + l * 256 + 4 * t;
    const bool bidle = m1_bidle(g);
    float b0 = 0.f, b2 = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        if (i < nb) {
            const uint8_t* r8 = rec + 544 * i;
            const uint4 q = *reinterpret_cast<const uint4*>(r8 + 32 + 16 * lane);
            const uint32_t bx = ld_b32(xb + 32 * i, bidle);
            const uint32_t by = ld_b32(xb + 32 * i + 16, bidle);
            int r[4];
            mma_s8_k32(r, q.x, q.y, q.z, q.w, bx, by);
            b0 += h2f(*reinterpret_cast<const unsigned short*>(r8 + 2 * g)) * (float)r[0];
            b2 += h2f(*reinterpret_cast<const unsigned short*>(r8 + 2 * (g + 8))) * (float)r[2];
        }
    }
    const float xs = X.xs[l];
    acc0 += xs * b0;
    acc2 += xs * b2;
}

// Shared-memory carve-up of one CTA (host and device agree on it).  nt == 0 is
// the single-row layout: planes 0..2 and the byte pieces of their sums.
struct SmemMap {
    int ring, bars, red, xq, xsum, xs, total;
};
__host__ __device__ inline SmemMap smem_map(int type, int nt, int umax, int rows) {
    const int nc = nt * 8, mpad = nt ? (nc + 2) / 3 : 1, ncp = 3 * mpad;
    const int qstride = umax * 256 + 32;
    // ints per sum row: 2 bytes per sum (its lo / hi byte pieces), + 16 bytes of slack
    const int sstride = sum_per(type) ? umax * sum_per(type) / 2 + 4 : 0;
    SmemMap m;
    m.ring = 0;
    m.bars = kWarps * stages(type, nt, umax) * unit_bytes(type);
    m.red = m.bars + (kWarps * stages(type, nt, umax) + 2) * 8;              // +1 barrier for the planes, padded
    m.xq = (m.red + kWarps * 16 * rows * 4 + 127) & ~127;      // per-warp folded outputs
    m.xsum = m.xq + ncp * qstride;
    m.xs = m.xsum + ncp * sstride * 4;
    m.total = m.xs + mpad * umax * 4;
    return m;
}

// ---------------------------------------------------------------------------
// The streaming kernel.  CTA = RT row tiles x KW warps per row tile (RT*KW = 8);
// blockIdx.y = cross-CTA K split.  Warp w owns row tile (w % RT) and K slice
// (w / RT) of the CTA's range.
// ---------------------------------------------------------------------------
// Fused tensor-parallel all-reduce of this CTA's rows (called instead of the
// plain epilogue when a.tp.world > 1, ks == 1), as packets: every output value
// goes to every rank (self included) as ONE 8-byte store (value bits | launch
// tag << 32) into slot [epoch parity][rank][elem] of that rank's buffer (P2P
// stores over NVLink); each rank polls its own slots of this parity until every
// rank's tag has arrived (bounded, ~1 s) and sums them in rank order, so every
// rank gets the same bits.  An aligned 8-byte store is observed whole, so a
// value and its tag travel together: no flag, no system-scope fence and no CTA
// barrier sits on the path.  (A first version pushed the rows, then stored one
// release flag per (rank, row group) and spun on acquire loads; at TP = 8 it cost
// 39 / 74 us per o / down call against 11.5 / 16.8 us for the packets.)
// The epoch lives in device memory, so CUDA-graph replays advance it; the last
// CTA of a launch bumps it.  Tags only grow and slots are double-buffered by
// parity, so the wait tests "reached" (tp_flag_reached), never equality, and a
// peer cannot overwrite a slot before it is read: its next same-parity store
// is two launches on, and its next launch waits for this rank's tags of that
// launch, which this rank stores only after finishing this one (the next launch
// starts behind griddepcontrol.wait).
__device__ __forceinline__ void st_volatile_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_volatile_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void tp_epilogue(const GemvArgs& a, const float* red, int RT, int KW, int64_t r0) {
    __shared__ unsigned int ep_s;
    __shared__ int failed_s;
    const TpArgs& tp = a.tp;
    if (threadIdx.x == 0) {
        ep_s = *reinterpret_cast<volatile unsigned int*>(tp.ctl);
        failed_s = 0;
    }
    __syncthreads();
    const unsigned int ep = ep_s, tag = ep + 1u, par = ep & 1u;
    const int64_t nrows = RT * 16;
    const unsigned long long* mine = nullptr;
#pragma unroll
    for (int p = 0; p < kTpMax; ++p)
        if (p == tp.rank) mine = tp.pkt[p];
    mine += (int64_t)par * tp.world * tp.max_elems;
    for (int idx = threadIdx.x; idx < nrows * a.rows; idx += blockDim.x) {
        const int m = (int)(idx / nrows), rl = (int)(idx - (int64_t)m * nrows);
        const int tile = rl >> 4, row = rl & 15;
        const int64_t o = r0 + rl;
        if (o >= a.n) continue;
        float v = 0.f;
        for (int q = 0; q < KW; ++q) v += red[((q * RT + tile) * a.rows + m) * 16 + row];
        const unsigned long long pkt = (unsigned long long)__float_as_uint(v) | ((unsigned long long)tag << 32);
        const int64_t e = ((int64_t)(par * tp.world + tp.rank)) * tp.max_elems + (int64_t)m * a.n + o;
#pragma unroll
        for (int p = 0; p < kTpMax; ++p)
            if (p < tp.world) st_volatile_u64(tp.pkt[p] + e, pkt);
    }
    bool ok = true;
    const long long t0 = clock64();
    for (int idx = threadIdx.x; idx < nrows * a.rows; idx += blockDim.x) {
        const int m = (int)(idx / nrows);
        const int64_t o = r0 + (idx - (int64_t)m * nrows);
        if (o >= a.n) continue;
        // all ranks' slots are loaded at once and only the missing ones
        // re-polled: one L2 round trip when everything has arrived, instead of
        // one per rank in sequence
        const unsigned long long* slot = mine + (int64_t)m * a.n + o;
        unsigned long long pkt[kTpMax];
#pragma unroll
        for (int s2 = 0; s2 < kTpMax; ++s2)
            pkt[s2] = s2 < tp.world ? ld_volatile_u64(slot + (int64_t)s2 * tp.max_elems) : ((unsigned long long)tag << 32);
        for (;;) {
            bool all = true;
#pragma unroll
            for (int s2 = 0; s2 < kTpMax; ++s2)
                if (!tp_flag_reached((unsigned int)(pkt[s2] >> 32), tag)) {
                    all = false;
                    pkt[s2] = ld_volatile_u64(slot + (int64_t)s2 * tp.max_elems);
                }
            if (all) break;
            if (clock64() - t0 > 2000000000LL) {
                ok = false;
                break;
            }
        }
        float v = 0.f;
#pragma unroll
        for (int s2 = 0; s2 < kTpMax; ++s2)  // rank order: identical bits on every rank
            if (s2 < tp.world) v += __uint_as_float((unsigned int)pkt[s2]);
        if (!ok) break;
        a.y[(int64_t)m * a.n + o] = a.bias ? v + a.bias[o] : v;
    }
    if (!ok) atomicExch(&failed_s, 1);
    __syncthreads();
    if (failed_s && threadIdx.x == 0) {
        atomicAdd(a.err + 1, 1u);
        if (a.host_err) *reinterpret_cast<volatile unsigned int*>(a.host_err) = 1u;
    }
    // advance the epoch once every CTA of this launch is through
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(tp.ctl + 1, 1u) == gridDim.x * gridDim.y - 1) {
            tp.ctl[1] = 0;
            __threadfence();
            atomicAdd(tp.ctl, 1u);
        }
    }
}

constexpr int kEpiPlain = 0, kEpiTp = 1, kEpiGated = 2;

// silu(z) * u with silu(z) = z * sigmoid(z) = z * (1 / (1 + exp(-z)))
// (crates/kernels/src/mlp.rs:77-86, then the gate_buf *= up_buf loop at :227-230).
__device__ __forceinline__ float silu_mul(float z, float u) { return z * (1.0f / (1.0f + expf(-z))) * u; }

// Gated epilogue: the CTA's RT row tiles are RT/2 (gate, up) pairs.  With one
// K split the CTA writes act = silu(gate) * up; with ks splits it writes gate
// and up partials ([ks][rows][2][npad], npad = 16 * pairs) and the last CTA of
// the group adds them in split order before applying silu * up.
__device__ __forceinline__ void gated_epilogue(const GemvArgs& a, const float* red, int RT, int KW, int split) {
    const int P = RT >> 1;
    const int64_t o0 = (int64_t)blockIdx.x * P * 16, npad = (a.n_rt >> 1) * 16;
    for (int idx = threadIdx.x; idx < P * 16 * a.rows; idx += blockDim.x) {
        const int m = idx / (P * 16), pl = idx - m * P * 16;
        const int pr = pl >> 4, row = pl & 15;
        const int64_t o = o0 + pl;
        if (o >= a.n) continue;
        float gv = 0.f, uv = 0.f;
        for (int q = 0; q < KW; ++q) {
            gv += red[((q * RT + 2 * pr) * a.rows + m) * 16 + row];
            uv += red[((q * RT + 2 * pr + 1) * a.rows + m) * 16 + row];
        }
        if (a.ks == 1) {
            a.y[(int64_t)m * a.n + o] = silu_mul(gv, uv);
        } else {
            float* base = a.part + (((int64_t)split * a.rows + m) * 2) * npad;
            base[o] = gv;
            base[npad + o] = uv;
        }
    }
    if (a.ks == 1) return;
    __threadfence();
    __syncthreads();
    __shared__ unsigned int last_g;
    if (threadIdx.x == 0) last_g = (atomicAdd(a.counters + blockIdx.x, 1u) == (unsigned)(a.ks - 1));
    __syncthreads();
    if (!last_g) return;
    __threadfence();
    const int64_t nr = min((int64_t)P * 16, a.n - o0);
    for (int64_t idx = threadIdx.x; idx < nr * a.rows; idx += blockDim.x) {
        const int m = (int)(idx / nr);
        const int64_t o = o0 + (idx - (int64_t)m * nr);
        float gv = 0.f, uv = 0.f;
        for (int s2 = 0; s2 < a.ks; ++s2) {
            const float* base = a.part + (((int64_t)s2 * a.rows + m) * 2) * npad;
            gv += __ldcg(base + o);
            uv += __ldcg(base + npad + o);
        }
        a.y[(int64_t)m * a.n + o] = silu_mul(gv, uv);
    }
    if (threadIdx.x == 0) a.counters[blockIdx.x] = 0;  // ready for the next launch
}

template <int TYPE, int NT, int EPI, int S>
__global__ void __launch_bounds__(256) gemv_kernel(GemvArgs a) {
    // NT == 0: single activation row (planes in MMA columns 0, 2, 4)
    // S (ring depth) = stages(TYPE, NT, a.umax), chosen by the host
    constexpr int UB = unit_bytes(TYPE), NC = NT ? NT * 8 : 8, MPAD = NT ? (NC + 2) / 3 : 1;
    constexpr int NCP = NT ? 3 * MPAD : 3;  // plane rows copied from global
    constexpr int NTA = NT ? NT : 1;
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int RT = a.rt_per_cta, KW = kWarps / RT;
    const int split = blockIdx.y;
    const int kw = warp / RT;
    // CTA range [U0, U1); this warp's slice [u0, u1) inside it
    const int U0 = (int)((int64_t)a.n_units * split / a.ks), U1 = (int)((int64_t)a.n_units * (split + 1) / a.ks);
    const int u0 = U0 + (int)((int64_t)(U1 - U0) * kw / KW), u1 = U0 + (int)((int64_t)(U1 - U0) * (kw + 1) / KW);
    const int nu = u1 - u0;
    const int64_t rt = (int64_t)blockIdx.x * RT + (warp % RT);
    const bool active = rt < a.n_rt;
    const SmemMap map = smem_map(TYPE, NT, a.umax, a.rows);

    uint8_t* ring = smem + map.ring + warp * (S * UB);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + map.bars) + warp * S;
    uint64_t* xbar = reinterpret_cast<uint64_t*>(smem + map.bars) + kWarps * S;
    float* red = reinterpret_cast<float*>(smem + map.red);
    const XSmem X{reinterpret_cast<int8_t*>(smem + map.xq), reinterpret_cast<int32_t*>(smem + map.xsum),
                  reinterpret_cast<float*>(smem + map.xs), a.umax * 256 + 32,
                  sum_per(TYPE) ? a.umax * sum_per(TYPE) / 2 + 4 : 0, a.umax};

    auto unit_src = [&](int u, uint32_t& bytes) -> const uint8_t* {
        if (TYPE == kQ8_0) {
            const int b0 = 8 * u, nb = min(8, a.nblk - b0);
            bytes = (uint32_t)(nb * 544);
            return a.W + ((size_t)rt * a.nblk + b0) * 544;
        }
        bytes = UB;
        return a.W + ((size_t)rt * a.n_units + u) * UB;
    };

    // 1. start the weight stream (weights do not depend on the previous kernel)
    int issued = 0;
    if (lane == 0) {
        if (active)
            for (int i = 0; i < S; ++i) mbar_init(&bars[i], 1);
        if (warp == 0) mbar_init(xbar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        if (active) {
            for (; issued < S && issued < nu; ++issued) {
                uint32_t bytes;
                const uint8_t* src = unit_src(u0 + issued, bytes);
                mbar_expect_tx(&bars[issued], bytes);
                bulk_g2s(ring + issued * UB, src, bytes, &bars[issued]);
            }
        }
    }
    issued = __shfl_sync(0xffffffffu, issued, 0);
    __syncthreads();  // barrier inits visible to every warp

    // 2. activation planes of [U0, U1): wait for the split kernel, then copy
    pdl_wait();
    pdl_trigger();
    const int NU = U1 - U0;
    if (warp == 0) {
        const uint32_t qb = (uint32_t)NU * 256, sb = (uint32_t)(NU * sum_per(TYPE) * 2);
        if (lane == 0) mbar_expect_tx(xbar, NCP * (qb + sb));
        __syncwarp();
        for (int c = lane; c < NCP; c += 32) {
            bulk_g2s(X.q + c * X.qstride, a.p.xq + (int64_t)c * a.p.kx + (int64_t)U0 * 256, qb, xbar);
            if (sum_per(TYPE)) {  // byte pieces of the sums
                const int8_t* src = (TYPE == kQ4_K) ? a.p.p32 : a.p.p16;
                const int per = 2 * sum_per(TYPE);
                bulk_g2s(X.s + c * X.sstride, src + ((int64_t)c * (a.p.kx / 256) + U0) * per, sb, xbar);
            }
        }
    }
    for (int i = threadIdx.x; i < MPAD * NU; i += blockDim.x) {
        const int m = i / NU, o = i - m * NU;
        X.xs[m * X.umax + o] = a.p.xs[(int64_t)m * (a.p.kx / 256) + U0 + o];
    }
    bool ok = mbar_wait_bounded(xbar, 0);
    __syncthreads();

    // 3. consume the ring (units are local to the CTA range: l = u - U0)
    float acc[NTA][4];
#pragma unroll
    for (int nt = 0; nt < NTA; ++nt)
#pragma unroll
        for (int v = 0; v < 4; ++v) acc[nt][v] = 0.f;
    int done = 0;
    if (active) {
        for (; done < nu && ok; ++done) {
            const int st = done % S;
            if (!mbar_wait_bounded(&bars[st], (uint32_t)((done / S) & 1))) {
                ok = false;
                break;
            }
            const uint8_t* rec = ring + st * UB;
            const int l = u0 + done - U0;
            if constexpr (NT == 0) {
                if (TYPE == kQ4_K) consume_q4k_m1(rec, l, X, acc[0][0], acc[0][2], g, t, lane);
                else if (TYPE == kQ6_K) consume_q6k_m1(rec, l, X, acc[0][0], acc[0][2], g, t, lane);
                else consume_q80_m1(rec, l, min(8, a.nblk - 8 * (u0 + done)), X, acc[0][0], acc[0][2], g, t, lane);
            } else {
                if (TYPE == kQ4_K) consume_q4k<NT>(rec, l, X, acc, g, t, lane);
                else if (TYPE == kQ6_K) consume_q6k<NT>(rec, l, X, acc, g, t, lane);
                else consume_q80<NT>(rec, l, min(8, a.nblk - 8 * (u0 + done)), X, acc, g, t, lane);
            }
            __syncwarp();
            if (lane == 0 && issued < nu) {
                uint32_t bytes;
                const uint8_t* src = unit_src(u0 + issued, bytes);
                fence_proxy_async();
                mbar_expect_tx(&bars[st], bytes);
                bulk_g2s(ring + st * UB, src, bytes, &bars[st]);
                ++issued;
            }
            issued = __shfl_sync(0xffffffffu, issued, 0);
        }
        if (!ok) {
            // drain this warp's copies still in flight before its shared memory goes away
            for (int i = done; i < issued; ++i) mbar_wait_bounded(&bars[i % S], (uint32_t)((i / S) & 1));
            if (lane == 0) {
                atomicAdd(a.err + 1, 1u);
                if (a.host_err) *reinterpret_cast<volatile unsigned int*>(a.host_err) = 1u;
            }
        }
    }

    // 4. fold the three planes of each activation row -> red[warp][m][row]
    if constexpr (NT == 0) {
        // lanes 4g+0,1,2 hold planes 0,1,2 of rows g and g+8
        const float p1a = __shfl_sync(0xffffffffu, acc[0][0], 4 * g + 1);
        const float p2a = __shfl_sync(0xffffffffu, acc[0][0], 4 * g + 2);
        const float p1b = __shfl_sync(0xffffffffu, acc[0][2], 4 * g + 1);
        const float p2b = __shfl_sync(0xffffffffu, acc[0][2], 4 * g + 2);
        if (t == 0) {
            red[warp * 16 + g] = (p2a * (1.0f / 16384.0f) + p1a * (1.0f / 128.0f)) + acc[0][0];
            red[warp * 16 + g + 8] = (p2b * (1.0f / 16384.0f) + p1b * (1.0f / 128.0f)) + acc[0][2];
        }
    } else {
        float* tmp = reinterpret_cast<float*>(ring);  // this warp's ring is drained
        __syncwarp();
#pragma unroll
        for (int nt = 0; nt < NTA; ++nt) {
            tmp[g * NC + nt * 8 + 2 * t] = acc[nt][0];
            tmp[g * NC + nt * 8 + 2 * t + 1] = acc[nt][1];
            tmp[(g + 8) * NC + nt * 8 + 2 * t] = acc[nt][2];
            tmp[(g + 8) * NC + nt * 8 + 2 * t + 1] = acc[nt][3];
        }
        __syncwarp();
        for (int idx = lane; idx < 16 * a.rows; idx += 32) {
            const int row = idx & 15, m = idx >> 4;
            const float* r = tmp + row * NC + 3 * m;
            red[(warp * a.rows + m) * 16 + row] = (r[2] * (1.0f / 16384.0f) + r[1] * (1.0f / 128.0f)) + r[0];
        }
    }
    __syncthreads();

    // 5. add the KW slices of each row tile in slice order; write y or a partial
    const int64_t r0 = (int64_t)blockIdx.x * RT * 16;
    if constexpr (EPI == kEpiTp) {  // row-split layer: sum over ranks through peer memory
        tp_epilogue(a, red, RT, KW, r0);
        return;
    } else if constexpr (EPI == kEpiGated) {
        gated_epilogue(a, red, RT, KW, split);
        return;
    } else {
        for (int idx = threadIdx.x; idx < RT * 16 * a.rows; idx += blockDim.x) {
            const int m = idx / (RT * 16), rl = idx - m * RT * 16;
            const int tile = rl >> 4, row = rl & 15;
            const int64_t o = r0 + rl;
            if (o >= a.n) continue;
            float v = 0.f;
            for (int q = 0; q < KW; ++q) v += red[((q * RT + tile) * a.rows + m) * 16 + row];
            if (a.ks == 1) a.y[(int64_t)m * a.n + o] = a.bias ? v + a.bias[o] : v;
            else a.part[((int64_t)split * a.rows + m) * a.n + o] = v;
        }
        if (a.ks == 1) return;

        // 6. cross-CTA split: the last CTA of this row group adds in split order
        __threadfence();
        __syncthreads();
        __shared__ unsigned int last;
        if (threadIdx.x == 0) last = (atomicAdd(a.counters + blockIdx.x, 1u) == (unsigned)(a.ks - 1));
        __syncthreads();
        if (!last) return;
        __threadfence();
        const int64_t nr = min((int64_t)RT * 16, a.n - r0);
        for (int64_t idx = threadIdx.x; idx < nr * a.rows; idx += blockDim.x) {
            const int m = (int)(idx / nr);
            const int64_t o = r0 + (idx - (int64_t)m * nr);
            float v = 0.f;
            for (int s2 = 0; s2 < a.ks; ++s2) v += __ldcg(a.part + ((int64_t)s2 * a.rows + m) * a.n + o);
            a.y[(int64_t)m * a.n + o] = a.bias ? v + a.bias[o] : v;
        }
        if (threadIdx.x == 0) a.counters[blockIdx.x] = 0;  // ready for the next launch
    }
}

template <int TYPE, int NT, int EPI, int S>
cudaError_t launch_typed(const GemvPlan& pl, const GemvArgs& a, bool pdl, cudaStream_t s) {
    // Largest dynamic shared memory enabled so far, per template instance and
    // device (a function attribute is set per device).
    static size_t configured_by_dev[kMaxDevices] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    size_t& configured = configured_by_dev[dev < kMaxDevices ? dev : 0];
    if (pl.smem > 48 * 1024 && (pl.smem > configured || dev >= kMaxDevices)) {
        cudaError_t e = cudaFuncSetAttribute(gemv_kernel<TYPE, NT, EPI, S>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)pl.smem);
        if (e != cudaSuccess) return e;
        configured = pl.smem;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)pl.groups, (unsigned)pl.ks);
    cfg.blockDim = dim3(32 * kWarps);
    cfg.dynamicSmemBytes = pl.smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, gemv_kernel<TYPE, NT, EPI, S>, a);
}

template <int TYPE, int EPI>
cudaError_t launch_nt(const GemvPlan& pl, const GemvArgs& a, bool pdl, cudaStream_t s) {
    switch (pl.nt) {
        case 0:
            if (stages(TYPE, 0, pl.umax) == 4) return launch_typed<TYPE, 0, EPI, (TYPE == kQ4_K ? 4 : 2)>(pl, a, pdl, s);
            return launch_typed<TYPE, 0, EPI, 2>(pl, a, pdl, s);
        case 1: return launch_typed<TYPE, 1, EPI, 2>(pl, a, pdl, s);
        case 2: return launch_typed<TYPE, 2, EPI, 2>(pl, a, pdl, s);
        case 3: return launch_typed<TYPE, 3, EPI, 2>(pl, a, pdl, s);
        case 4: return launch_typed<TYPE, 4, EPI, 2>(pl, a, pdl, s);
        case 5: return launch_typed<TYPE, 5, EPI, 2>(pl, a, pdl, s);
        case 6: return launch_typed<TYPE, 6, EPI, 2>(pl, a, pdl, s);
        default: return cudaErrorInvalidValue;
    }
}

template <int TYPE>
cudaError_t launch_tp(const GemvPlan& pl, const GemvArgs& a, bool pdl, cudaStream_t s) {
    if (a.gated) return launch_nt<TYPE, kEpiGated>(pl, a, pdl, s);
    return a.tp.world > 1 ? launch_nt<TYPE, kEpiTp>(pl, a, pdl, s) : launch_nt<TYPE, kEpiPlain>(pl, a, pdl, s);
}

}  // namespace

GemvPlan plan_gemv(int type, int64_t n, int64_t k, int rows, int sms) {
    GemvPlan pl{};
    pl.nt = rows == 1 ? 0 : (3 * rows + 7) / 8;
    pl.n_rt = (n + 15) / 16;
    pl.n_units = (int)((k + 255) / 256);
    // Measured on B200 (M = 1, Llama-shaped matrices): splitting K across
    // CTAs never paid (its partial-sum round trip and fences cost more than the
    // extra warps bring), and ~1500 streaming warps with K split 2-4 ways inside
    // each CTA did best.  So: ks = 1 unless the staged activation planes do not
    // fit in shared memory, and kw = the power of two nearest 1536 / row tiles
    // (scaled by the SM count), capped at 4 and at half the K units.
    int kw = 1;
    if (rows <= 2) {
        const double target = 1536.0 * sms / 148.0 / (double)pl.n_rt;
        while (kw < 4 && kw * 2 <= pl.n_units / 2 && target >= kw * 1.5) kw *= 2;
        // never leave SMs without a CTA
        while (kw < kWarps && kw * 2 <= pl.n_units / 2 && (pl.n_rt + kWarps / kw - 1) / (kWarps / kw) < sms) kw *= 2;
        // ... but not at the price of a second wave: when the planes of a long
        // K leave room for one CTA per SM (two rows, K = 14336), halve kw while
        // that brings the grid within one wave (measured: down at M = 2,
        // 19.6 -> 16.7 us)
        const size_t per_cta = (size_t)smem_map(type, pl.nt, pl.n_units, rows).total + 1024;
        const int64_t slots = (int64_t)sms * (int64_t)((228 * 1024) / per_cta);
        auto groups_of = [&](int kw_) { return (pl.n_rt + kWarps / kw_ - 1) / (kWarps / kw_); };
        while (kw > 1 && groups_of(kw) > slots && groups_of(kw / 2) <= slots) kw /= 2;
    }
    int ks = 1;
    if (rows > 2) {
        // Batched decode (measured on B200, Llama-shaped matrices, M = 4..16): the
        // staged activation planes grow with M, so wide matrices keep 8 row
        // tiles per CTA, deep ones (K >= 8192) split K across 4-8 CTAs to keep
        // the planes small, and narrow ones split K 2-4 ways inside the CTA.
        if (pl.n_rt >= 768) {
            kw = 1;
        } else if (pl.n_units >= 32) {
            kw = 1;
            ks = rows <= 8 ? 4 : 8;
        } else if (rows <= 8) {
            kw = pl.n_rt <= 256 ? 4 : 2;
        } else {
            kw = pl.n_rt <= 256 ? 2 : 1;
        }
        while (kw > 1 && kw > pl.n_units / 2) kw /= 2;
        if (ks > pl.n_units) ks = pl.n_units;
    }
    auto fits = [&](int ks_) {
        const int umax = (pl.n_units + ks_ - 1) / ks_;
        return smem_map(type, pl.nt, umax, rows).total <= 220 * 1024;
    };
    while (!fits(ks) && ks < pl.n_units) ++ks;
    if (const char* f = getenv("OCL_GEMV_KW")) {  // tuning overrides for experiments
        const int v = atoi(f);
        if (v == 1 || v == 2 || v == 4 || v == 8) kw = v;
    }
    if (const char* f = getenv("OCL_GEMV_KS")) {
        const int v = atoi(f);
        if (v >= 1 && v <= pl.n_units && fits(v)) ks = v;
    }
    pl.kw = kw;
    pl.ks = ks;
    pl.groups = (pl.n_rt + (kWarps / kw) - 1) / (kWarps / kw);
    pl.umax = (pl.n_units + ks - 1) / ks;
    pl.smem = (size_t)smem_map(type, pl.nt, pl.umax, rows).total;
    pl.part_floats = pl.ks > 1 ? (size_t)pl.ks * rows * n : 0;
    return pl;
}

GemvPlan plan_gemv_gated(int type, int64_t n_gate, int64_t k, int rows, int sms) {
    const int64_t n_pairs = (n_gate + 15) / 16;
    GemvPlan pl = plan_gemv(type, 2 * n_pairs * 16, k, rows, sms);
    if (pl.kw > kWarps / 2) {  // at least one whole (gate, up) pair of row tiles per CTA
        pl.kw = kWarps / 2;
        pl.groups = (pl.n_rt + (kWarps / pl.kw) - 1) / (kWarps / pl.kw);
    }
    return pl;
}

bool plan_single_split(GemvPlan& pl, int type, int rows) {
    pl.ks = 1;
    pl.umax = pl.n_units;
    pl.smem = (size_t)smem_map(type, pl.nt, pl.umax, rows).total;
    pl.part_floats = 0;
    return pl.smem <= 220 * 1024;
}

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
    p.p32 = (int8_t*)take((size_t)kColsMax * (p.kx / 256) * 16);
    p.p16 = (int8_t*)take((size_t)kColsMax * (p.kx / 256) * 32);
    return p;
}

cudaError_t launch_xsplit(const float* x, int rows, int64_t k, const XPlanes& p, bool pdl, cudaStream_t s,
                          int type) {
    // the sums the GEMV of `type` reads: byte pieces for a single row, ints otherwise
    int sums = 15;
    if (type == kQ4_K) sums = 8;       // per-32 byte pieces
    else if (type == kQ6_K) sums = 4;  // per-16 byte pieces
    else if (type == kQ8_0) sums = 0;
    const int nt = rows == 1 ? 0 : (3 * rows + 7) / 8;
    const int mpad = nt ? (nt * 8 + 2) / 3 : 1;  // activation rows whose planes the GEMV reads
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(p.kx / 256), (unsigned)mpad);
    cfg.blockDim = dim3(32);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, xsplit_kernel, x, rows, k, p, sums);
}

cudaError_t launch_gemv(int type, const void* tiles, int64_t n, int64_t k, const XPlanes& p, int rows,
                        const float* bias, float* y, const GemvPlan& pl, float* part, unsigned int* counters,
                        unsigned int* err, bool pdl, cudaStream_t s, const TpArgs* tp, unsigned int* host_err) {
    GemvArgs a{};
    a.host_err = host_err;
    if (tp) {
        if (pl.ks != 1) return cudaErrorInvalidValue;
        a.tp = *tp;
    }
    a.W = (const uint8_t*)tiles;
    a.n = n;
    a.k = k;
    a.n_rt = pl.n_rt;
    a.n_units = pl.n_units;
    a.nblk = (int)(k / 32);
    a.ks = pl.ks;
    a.rt_per_cta = kWarps / pl.kw;
    a.umax = pl.umax;
    a.p = p;
    a.rows = rows;
    a.bias = bias;
    a.y = y;
    a.part = part;
    a.counters = counters;
    a.err = err;
    if (type == kQ4_K) return launch_tp<kQ4_K>(pl, a, pdl, s);
    if (type == kQ6_K) return launch_tp<kQ6_K>(pl, a, pdl, s);
    return launch_tp<kQ8_0>(pl, a, pdl, s);
}

cudaError_t launch_gemv_gated(int type, const void* tiles, int64_t n_gate, int64_t k, const XPlanes& p, int rows,
                              float* act, const GemvPlan& pl, float* part, unsigned int* counters, unsigned int* err,
                              bool pdl, cudaStream_t s) {
    if ((kWarps / pl.kw) % 2 != 0 || pl.n_rt % 2 != 0) return cudaErrorInvalidValue;
    GemvArgs a{};
    a.W = (const uint8_t*)tiles;
    a.n = n_gate;
    a.k = k;
    a.n_rt = pl.n_rt;
    a.n_units = pl.n_units;
    a.nblk = (int)(k / 32);
    a.ks = pl.ks;
    a.rt_per_cta = kWarps / pl.kw;
    a.umax = pl.umax;
    a.p = p;
    a.rows = rows;
    a.y = act;
    a.part = part;
    a.counters = counters;
    a.err = err;
    a.gated = 1;
    if (type == kQ4_K) return launch_tp<kQ4_K>(pl, a, pdl, s);
    if (type == kQ6_K) return launch_tp<kQ6_K>(pl, a, pdl, s);
    return launch_tp<kQ8_0>(pl, a, pdl, s);
}

}  // namespace ocl
