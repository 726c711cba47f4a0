// gemm.cu -- prefill (M >= 64) quantized GEMM on the 5th-generation tensor cores.
//
// y[m, n] (bf16) = sum_k x[m, k] (bf16) * W[n, k], W GGUF-quantized in TILED16
// records, f32 accumulation in tensor memory.
//
// One CTA computes a 256 (tokens) x 128 (output features) tile as two 128 x 128
// accumulators in tensor memory that share each dequantized weight tile:
//   * warp 8 (one lane) streams x tiles [256 x 64] bf16 with TMA (tiled,
//     128-byte swizzle, no multicast) into a 4- or 2-stage shared-memory ring;
//   * warps 0-7 dequantize the matching weight tile [128 features x 64 k] from
//     the TILED16 records (prefetched one 256-k unit ahead in registers) into
//     bf16, written directly in the 128-byte-swizzled K-major layout the UMMA
//     descriptors describe; each value is d*sc*q - dmin*m (Q4_K),
//     d*sc*(q-32) (Q6_K) or d*q (Q8_0) in f32, rounded to bf16;
//   * warp 9 allocates 256 TMEM columns and one lane issues
//     tcgen05.mma.cta_group::1.kind::f16 (M=128, N=128, K=16, A and B K-major),
//     releasing each stage with tcgen05.commit to an mbarrier;
//   * warps 0-3 read the accumulator with tcgen05.ld (32 lanes x 32 columns per
//     instruction), convert to bf16 and store y.
// Every mbarrier wait is bounded (~1 s); a wait that gives up bumps the
// context's error counter, the CTA drains what it issued and returns.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdlib>

#include "internal.cuh"

namespace ocl {

namespace {

constexpr int BN = 128, BK = 64;
// A CTA's token tile is ACC x 128 rows (ACC = 2 or 4 TMEM accumulators of 128 x
// 128 f32 sharing every dequantized weight tile).  ACC = 4 uses all 512 TMEM
// columns and halves the dequantization per FLOP; x then arrives in two
// 256-row TMA boxes per stage (a box dimension is at most 256).
// Two shapes of the same kernel: 4 pipeline stages and one CTA per SM, or 2
// stages and two CTAs per SM (<= 96 registers a thread, 2 x 256 TMEM columns),
// which overlaps one CTA's epilogue and pipeline fill with the other's main
// loop.  Measured on B200: the two-CTA form is 3-22% faster once the tile
// grid exceeds one wave of SMs and 7-21% slower below that.
constexpr int MMA_M = 128, BOX_M = 256;        // rows per MMA, rows per x TMA box
constexpr int B_BYTES = BN * BK * 2;           // 16 KB per stage
template <int ACC> struct ATile {
    static constexpr int BM = ACC * MMA_M, BYTES = BM * BK * 2;  // 32 or 64 KB per stage
};
constexpr int PRODUCER_WARPS = 8, TMA_WARP = 8, MMA_WARP = 9, THREADS = 320;
constexpr long long kWaitCycles = 2000000000LL;

// silu(z) * u, silu(z) = z * (1 / (1 + exp(-z))) (crates/kernels/src/mlp.rs:77-86)
__device__ __forceinline__ float silu_mul(float z, float u) { return z * (1.0f / (1.0f + expf(-z))) * u; }
__device__ __forceinline__ uint32_t sa(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mb_init(uint64_t* b, uint32_t n) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(sa(b)), "r"(n));
}
__device__ __forceinline__ void mb_arrive(uint64_t* b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(sa(b)) : "memory");
}
__device__ __forceinline__ void mb_expect_tx(uint64_t* b, uint32_t n) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(sa(b)), "r"(n) : "memory");
}
__device__ __forceinline__ bool mb_try(uint64_t* b, uint32_t ph) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(sa(b)), "r"(ph)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool mb_wait(uint64_t* b, uint32_t ph) {
    if (mb_try(b, ph)) return true;
    const long long t0 = clock64();
    while (!mb_try(b, ph))
        if (clock64() - t0 > kWaitCycles) return false;
    return true;
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(sa(dst)),
        "l"(map), "r"(x), "r"(y), "r"(sa(bar))
        : "memory");
}
// UMMA shared-memory descriptor: K-major, 128-byte swizzle, 8-row groups 1024 B apart.
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// Instruction descriptor: f32 accumulator, bf16 A and B, both K-major, M = 128, N = 128.
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(MMA_M >> 4) << 24);

__device__ __forceinline__ void umma(uint32_t dtmem, uint64_t ad, uint64_t bd, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(dtmem),
        "l"(ad), "l"(bd), "r"(kIdesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(sa(bar))
                 : "memory");
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&v);
}
// Q4_K 6-bit scale / min of sub-block j from the header words y, z, w (scale bytes 0-3, 4-7, 8-11)
__device__ __forceinline__ void q4k_sm(const uint4& h, int j, int& sc, int& m) {
    const int b = j & 3;
    const uint32_t yb = (h.y >> (8 * b)) & 0xFF, zb = (h.z >> (8 * b)) & 0xFF, wb = (h.w >> (8 * b)) & 0xFF;
    if (j < 4) {
        sc = (int)(yb & 63);
        m = (int)(zb & 63);
    } else {
        sc = (int)((wb & 0xF) | ((yb >> 6) << 4));
        m = (int)((wb >> 4) | ((zb >> 6) << 4));
    }
}
__device__ __forceinline__ float h2f(uint32_t bits) { return __half2float(__ushort_as_half((unsigned short)bits)); }
// byte offset of element (row, k) inside a [rows x 64] bf16 tile, 128-byte swizzle
__device__ __forceinline__ int sw128(int row, int k) {
    return row * 128 + ((((k >> 3) ^ (row & 7))) << 4) + ((k & 7) << 1);
}

// ---- per-type register staging of one 256-k unit for one lane of a row tile ----
struct UnitRegs {
    uint4 h0, h1;    // Q4_K headers of rows g, g+8 | Q6_K scales of rows g, g+8
    uint4 c[4];      // Q4_K: chunks c = 0..3 | Q6_K: low-nibble chunks u = 0..3 | Q8_0: records 0..3 of the unit
    uint4 e[4];      // Q6_K: crumb chunks v = 0..1 in e[0..1] | Q8_0: records 4..7
    uint32_t d0, d1; // Q6_K d of rows g, g+8
    uint32_t q8d[8]; // Q8_0: d of rows g | g+8 << 16, per record
};

template <int TYPE>
__device__ __forceinline__ void load_unit(const uint8_t* __restrict__ W, int64_t rt, int64_t n_rt, int n_units,
                                          int nblk, int u, int g, int lane, UnitRegs& R) {
    if (rt >= n_rt) {
        R.h0 = R.h1 = make_uint4(0, 0, 0, 0);
        for (int i = 0; i < 4; ++i) R.c[i] = R.e[i] = make_uint4(0, 0, 0, 0);
        R.d0 = R.d1 = 0;
        for (int i = 0; i < 8; ++i) R.q8d[i] = 0;
        return;
    }
    if (TYPE == kQ4_K) {
        const uint8_t* rec = W + ((size_t)rt * n_units + u) * 2304;
        R.h0 = __ldg(reinterpret_cast<const uint4*>(rec + 16 * g));
        R.h1 = __ldg(reinterpret_cast<const uint4*>(rec + 16 * (g + 8)));
#pragma unroll
        for (int c = 0; c < 4; ++c) R.c[c] = __ldg(reinterpret_cast<const uint4*>(rec + 256 + 512 * c + 16 * lane));
    } else if (TYPE == kQ6_K) {
        const uint8_t* rec = W + ((size_t)rt * n_units + u) * 3360;
        R.h0 = __ldg(reinterpret_cast<const uint4*>(rec + 16 * g));
        R.h1 = __ldg(reinterpret_cast<const uint4*>(rec + 16 * (g + 8)));
        R.d0 = __ldg(reinterpret_cast<const unsigned short*>(rec + 256 + 2 * g));
        R.d1 = __ldg(reinterpret_cast<const unsigned short*>(rec + 256 + 2 * (g + 8)));
#pragma unroll
        for (int c = 0; c < 4; ++c) R.c[c] = __ldg(reinterpret_cast<const uint4*>(rec + 288 + 512 * c + 16 * lane));
#pragma unroll
        for (int v = 0; v < 2; ++v) R.e[v] = __ldg(reinterpret_cast<const uint4*>(rec + 2336 + 512 * v + 16 * lane));
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int b = 8 * u + i;
            uint4 q = make_uint4(0, 0, 0, 0);
            uint32_t d = 0;
            if (b < nblk) {
                const uint8_t* rec = W + ((size_t)rt * nblk + b) * 544;
                q = __ldg(reinterpret_cast<const uint4*>(rec + 32 + 16 * lane));
                d = (uint32_t)__ldg(reinterpret_cast<const unsigned short*>(rec + 2 * g)) |
                    ((uint32_t)__ldg(reinterpret_cast<const unsigned short*>(rec + 2 * (g + 8))) << 16);
            }
            if (i < 4) R.c[i] = q;
            else R.e[i - 4] = q;
            R.q8d[i] = d;
        }
    }
}

// Dequantize quarter qt (k 64*qt .. 64*qt+63 of the unit) of rows g, g+8 of row
// tile rtl into the swizzled bf16 B tile.
template <int TYPE>
__device__ __forceinline__ void dequant_quarter(const UnitRegs& R, int qt, int rtl, int g, int t, uint8_t* btile) {
    const int ra = rtl * 16 + g, rb = ra + 8;
    if (TYPE == kQ4_K) {
        // chunk qt: bytes 0..7 row g, 8..15 row g+8, qs[32*qt + 8t + i]; low nibble ->
        // sub-block 2qt (k = 8t+i), high nibble -> 2qt+1 (k = 32 + 8t + i)
        const uint4 h[2] = {R.h0, R.h1};
        const uint32_t w[2][2] = {{R.c[qt].x, R.c[qt].y}, {R.c[qt].z, R.c[qt].w}};
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const uint4 hd = h[r];
            const float d = h2f(hd.x & 0xffffu), dmin = h2f(hd.x >> 16);
            int sc_lo, m_lo, sc_hi, m_hi;
            q4k_sm(hd, 2 * qt, sc_lo, m_lo);
            q4k_sm(hd, 2 * qt + 1, sc_hi, m_hi);
            const float d1 = d * (float)sc_lo, m1 = dmin * (float)m_lo;
            const float d2 = d * (float)sc_hi, m2 = dmin * (float)m_hi;
            uint32_t lo[4], hi[4];
#pragma unroll
            for (int i = 0; i < 8; i += 2) {
                const uint32_t b0 = (w[r][i >> 2] >> (8 * (i & 3))) & 0xFF;
                const uint32_t b1 = (w[r][(i + 1) >> 2] >> (8 * ((i + 1) & 3))) & 0xFF;
                lo[i >> 1] = pack_bf16(d1 * (float)(b0 & 15) - m1, d1 * (float)(b1 & 15) - m1);
                hi[i >> 1] = pack_bf16(d2 * (float)(b0 >> 4) - m2, d2 * (float)(b1 >> 4) - m2);
            }
            const int row = r ? rb : ra;
            *reinterpret_cast<uint4*>(btile + sw128(row, 8 * t)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
            *reinterpret_cast<uint4*>(btile + sw128(row, 32 + 8 * t)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        }
    } else if (TYPE == kQ6_K) {
        // low chunk qt: word jj -> sub-block j = 4qt+jj, nibble 2i = row g, 2i+1 = row g+8,
        // element k = 16j + 4t + i (quarter-local 16jj + 4t + i); crumbs from chunk qt/2,
        // words 2(qt%2), 2(qt%2)+1 (sub-block pairs)
        const uint32_t lw[4] = {R.c[qt].x, R.c[qt].y, R.c[qt].z, R.c[qt].w};
        const uint4 hc = R.e[qt >> 1];
        const uint32_t hw[4] = {hc.x, hc.y, hc.z, hc.w};
        const float d0 = h2f(R.d0), d1 = h2f(R.d1);
        const uint32_t sw0[4] = {R.h0.x, R.h0.y, R.h0.z, R.h0.w};
        const uint32_t sw1[4] = {R.h1.x, R.h1.y, R.h1.z, R.h1.w};
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
            const int j = 4 * qt + jj;
            const uint32_t crumb = hw[2 * (qt & 1) + (jj >> 1)];
            const int sh = 2 * (2 * (jj & 1));  // bits of row g (row g+8: +2)
            const float ds0 = d0 * (float)(int8_t)(sw0[j >> 2] >> (8 * (j & 3)));
            const float ds1 = d1 * (float)(int8_t)(sw1[j >> 2] >> (8 * (j & 3)));
            float va[4], vb[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t nib = lw[jj] >> (8 * i);
                const uint32_t cr = crumb >> (8 * i);
                const int qa = (int)((nib & 15) | (((cr >> sh) & 3) << 4)) - 32;
                const int qb = (int)(((nib >> 4) & 15) | (((cr >> (sh + 2)) & 3) << 4)) - 32;
                va[i] = ds0 * (float)qa;
                vb[i] = ds1 * (float)qb;
            }
            const int kq = 16 * jj + 4 * t;
            *reinterpret_cast<uint2*>(btile + sw128(ra, kq)) = make_uint2(pack_bf16(va[0], va[1]), pack_bf16(va[2], va[3]));
            *reinterpret_cast<uint2*>(btile + sw128(rb, kq)) = make_uint2(pack_bf16(vb[0], vb[1]), pack_bf16(vb[2], vb[3]));
        }
    } else {
        // records 2qt, 2qt+1 of the unit (32 k each): chunk bytes 0..3 row g q[4t..],
        // 4..7 row g+8 q[4t..], 8..11 row g q[16+4t..], 12..15 row g+8 q[16+4t..]
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
            const int ri = 2 * qt + rr;
            const uint4 q = ri < 4 ? R.c[ri] : R.e[ri - 4];
            const float da = h2f(R.q8d[ri] & 0xffffu), db = h2f(R.q8d[ri] >> 16);
            const uint32_t wa[2] = {q.x, q.z}, wb[2] = {q.y, q.w};
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                float va[4], vb[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    va[i] = da * (float)(int8_t)(wa[hh] >> (8 * i));
                    vb[i] = db * (float)(int8_t)(wb[hh] >> (8 * i));
                }
                const int kq = 32 * rr + 16 * hh + 4 * t;
                *reinterpret_cast<uint2*>(btile + sw128(ra, kq)) =
                    make_uint2(pack_bf16(va[0], va[1]), pack_bf16(va[2], va[3]));
                *reinterpret_cast<uint2*>(btile + sw128(rb, kq)) =
                    make_uint2(pack_bf16(vb[0], vb[1]), pack_bf16(vb[2], vb[3]));
            }
        }
    }
}

// GATED: W holds interleaved gate/up row tiles (tile 2t = gate tile t, tile
// 2t+1 = up tile t; N = their total padded rows) and y [M, n_out] =
// silu(gate) * up: each 32-column accumulator slice a thread reads is one
// (gate, up) pair of 16-row tiles.
template <int TYPE, bool GATED, int STAGES, int ACCS>
__global__ void __launch_bounds__(THREADS, (STAGES == 2 && ACCS == 2) ? 2 : 1)
    qgemm_kernel(const __grid_constant__ CUtensorMap xmap, const uint8_t* __restrict__ W, int64_t M, int64_t N,
                 int64_t K, uint16_t* __restrict__ y, int64_t n_out, unsigned int* __restrict__ err,
                 float* __restrict__ yf, const float* __restrict__ bias) {
    constexpr int BM = ATile<ACCS>::BM, A_BYTES = ATile<ACCS>::BYTES;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 1024-byte alignment for the swizzled tiles
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t* atiles = smem;
    uint8_t* btiles = smem + STAGES * A_BYTES;
    uint64_t* full_a = reinterpret_cast<uint64_t*>(btiles + STAGES * B_BYTES);
    uint64_t* full_b = full_a + STAGES;
    uint64_t* empty = full_b + STAGES;
    uint64_t* done = empty + STAGES;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    __shared__ int abort_flag_s;
    volatile int& abort_flag = abort_flag_s;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t m0 = (int64_t)blockIdx.x * BM, n0 = (int64_t)blockIdx.y * BN;
    const int n_units = (int)(K / 256), nkb = (int)(K / BK);
    const int64_t n_rt = (N + 15) / 16;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mb_init(&full_a[s], 1);
            mb_init(&full_b[s], PRODUCER_WARPS);
            mb_init(&empty[s], 1);
        }
        mb_init(done, 1);
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == MMA_WARP) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(sa(tmem_slot)),
                     "r"(ACCS * BN));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;

    if (warp < PRODUCER_WARPS) {
        // ---- dequantize weight tiles ------------------------------------------
        const int g = lane >> 2, t = lane & 3, rtl = warp;
        const int64_t rt = n0 / 16 + rtl;
        UnitRegs cur, nxt;
        load_unit<TYPE>(W, rt, n_rt, n_units, (int)(K / 32), 0, g, lane, cur);
        for (int u = 0; u < n_units; ++u) {
            if (u + 1 < n_units) load_unit<TYPE>(W, rt, n_rt, n_units, (int)(K / 32), u + 1, g, lane, nxt);
#pragma unroll
            for (int qt = 0; qt < 4; ++qt) {
                const int kb = 4 * u + qt, s = kb % STAGES;
                if (!mb_wait(&empty[s], ((kb / STAGES) & 1) ^ 1)) {
                    atomicExch(&abort_flag_s, 1);
                    break;
                }
                if (abort_flag) break;
                dequant_quarter<TYPE>(cur, qt, rtl, g, t, btiles + s * B_BYTES);
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                if (lane == 0) mb_arrive(&full_b[s]);
            }
            if (abort_flag) break;
            cur = nxt;
        }
    } else if (warp == TMA_WARP) {
        if (lane == 0) {
            int issued = 0;
            for (int kb = 0; kb < nkb; ++kb) {
                const int s = kb % STAGES;
                if (!mb_wait(&empty[s], ((kb / STAGES) & 1) ^ 1) || abort_flag) {
                    atomicExch(&abort_flag_s, 1);
                    break;
                }
                mb_expect_tx(&full_a[s], A_BYTES);
#pragma unroll
                for (int h = 0; h < BM / BOX_M; ++h)
                    tma_load_2d(atiles + s * A_BYTES + h * (BOX_M * BK * 2), &xmap, kb * BK, (int)m0 + h * BOX_M,
                                &full_a[s]);
                ++issued;
            }
            // make sure no copy is still landing when the CTA leaves
            for (int kb = issued - STAGES > 0 ? issued - STAGES : 0; kb < issued; ++kb)
                mb_wait(&full_a[kb % STAGES], (kb / STAGES) & 1);
        }
    } else {  // MMA_WARP
        if (lane == 0) {
            int kb = 0;
            for (; kb < nkb; ++kb) {
                const int s = kb % STAGES;
                const uint32_t ph = (kb / STAGES) & 1;
                if (!mb_wait(&full_a[s], ph) || !mb_wait(&full_b[s], ph) || abort_flag) {
                    atomicExch(&abort_flag_s, 1);
                    break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t a_base = sa(atiles + s * A_BYTES), b_base = sa(btiles + s * B_BYTES);
#pragma unroll
                for (int kk = 0; kk < BK / 16; ++kk)
#pragma unroll
                    for (int acc = 0; acc < ACCS; ++acc)  // 128-row A halves, 16 KB apart
                        umma(tmem + acc * BN, umma_desc(a_base + acc * (MMA_M * 128) + 32 * kk),
                             umma_desc(b_base + 32 * kk), (kb | kk) != 0);
                umma_commit(&empty[s]);
            }
            umma_commit(done);  // arrives once every MMA issued above has completed
        }
    }

    // ---- epilogue: warps 0-3 own TMEM lanes 32w .. 32w+31 (tokens) -------------
    if (warp < 4) {
        const bool ok = mb_wait(done, 0);
        if (!ok) atomicExch(&abort_flag_s, 1);
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        if (__all_sync(0xffffffffu, ok && !abort_flag)) {
#pragma unroll 1
            for (int acc = 0; acc < ACCS; ++acc) {
            const int64_t m = m0 + acc * MMA_M + 32 * warp + lane;
#pragma unroll
            for (int c0 = 0; c0 < BN; c0 += 32) {
                uint32_t v[32];
                const uint32_t taddr = tmem + ((uint32_t)(32 * warp) << 16) + (uint32_t)(acc * BN + c0);
                asm volatile(
                    "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
                    "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
                    : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                      "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
                      "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]),
                      "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]),
                      "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
                    : "r"(taddr));
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                if (m < M && GATED && yf) {
                    float p[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i) p[i] = silu_mul(__uint_as_float(v[i]), __uint_as_float(v[16 + i]));
                    const int64_t n = (n0 + c0) / 2;
                    float* dst = yf + m * n_out + n;
                    if (n + 16 <= n_out && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
#pragma unroll
                        for (int i = 0; i < 4; ++i)
                            reinterpret_cast<float4*>(dst)[i] = make_float4(p[4 * i], p[4 * i + 1], p[4 * i + 2], p[4 * i + 3]);
                    } else {
                        for (int i = 0; i < 16 && n + i < n_out; ++i) dst[i] = p[i];
                    }
                } else if (m < M && GATED) {
                    uint32_t p[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        p[i] = pack_bf16(silu_mul(__uint_as_float(v[2 * i]), __uint_as_float(v[16 + 2 * i])),
                                         silu_mul(__uint_as_float(v[2 * i + 1]), __uint_as_float(v[17 + 2 * i])));
                    const int64_t n = (n0 + c0) / 2;
                    uint16_t* dst = y + m * n_out + n;
                    if (n + 16 <= n_out && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
                        reinterpret_cast<uint4*>(dst)[0] = make_uint4(p[0], p[1], p[2], p[3]);
                        reinterpret_cast<uint4*>(dst)[1] = make_uint4(p[4], p[5], p[6], p[7]);
                    } else {
                        for (int i = 0; i < 16 && n + i < n_out; ++i)
                            dst[i] = (uint16_t)(i & 1 ? p[i >> 1] >> 16 : p[i >> 1] & 0xffffu);
                    }
                } else if (m < M && yf) {
                    // f32 output (+ bias): the linear_d form of the prefill GEMM
                    float p[32];
                    const int64_t n = n0 + c0;
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        p[i] = __uint_as_float(v[i]) + ((bias && n + i < N) ? __ldg(bias + n + i) : 0.0f);
                    float* dst = yf + m * N + n;
                    if (n + 32 <= N && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
#pragma unroll
                        for (int i = 0; i < 8; ++i)
                            reinterpret_cast<float4*>(dst)[i] = make_float4(p[4 * i], p[4 * i + 1], p[4 * i + 2], p[4 * i + 3]);
                    } else {
                        for (int i = 0; i < 32 && n + i < N; ++i) dst[i] = p[i];
                    }
                } else if (m < M) {
                    uint32_t p[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i) p[i] = pack_bf16(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1]));
                    const int64_t n = n0 + c0;
                    uint16_t* dst = y + m * N + n;
                    if (n + 32 <= N && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
#pragma unroll
                        for (int i = 0; i < 4; ++i)
                            reinterpret_cast<uint4*>(dst)[i] = make_uint4(p[4 * i], p[4 * i + 1], p[4 * i + 2], p[4 * i + 3]);
                    } else {
                        for (int i = 0; i < 32 && n + i < N; ++i)
                            dst[i] = (uint16_t)(i & 1 ? p[i >> 1] >> 16 : p[i >> 1] & 0xffffu);
                    }
                }
            }
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (threadIdx.x == 0 && abort_flag) atomicAdd(err + 1, 1u);
    if (warp == MMA_WARP) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ACCS * BN));
    }
}

// 512-token tiles from 2048 tokens on (measured, 8B layer: +4.6% at M = 2048,
// -17% at M = 512, where the tile grid no longer fills the SMs).  The gain is
// small because one such CTA fills an SM: it halves the dequantization per
// FLOP but also the producer warps per SM, which the two-CTA 256-token form has.
inline bool wide_tokens(int64_t M, int64_t, int) { return M >= 2048; }

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

template <int TYPE, bool GATED, int STAGES, int ACCS>
cudaError_t launch_staged(const CUtensorMap& map, const void* w, int64_t M, int64_t N, int64_t K, uint16_t* y,
                          int64_t n_out, unsigned int* err, cudaStream_t s, float* yf, const float* bias) {
    const size_t smem = 1024 + STAGES * (ATile<ACCS>::BYTES + B_BYTES) + (3 * STAGES + 2) * 8;
    static bool configured_by_dev[kMaxDevices] = {};  // a function attribute is set per device
    int dev = 0;
    cudaGetDevice(&dev);
    bool& configured = configured_by_dev[dev < kMaxDevices ? dev : 0];
    if (!configured || dev >= kMaxDevices) {
        cudaError_t e = cudaFuncSetAttribute(qgemm_kernel<TYPE, GATED, STAGES, ACCS>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        configured = true;
    }
    constexpr int BM = ATile<ACCS>::BM;
    const dim3 grid((unsigned)((M + BM - 1) / BM), (unsigned)((N + BN - 1) / BN));
    qgemm_kernel<TYPE, GATED, STAGES, ACCS><<<grid, THREADS, smem, s>>>(map, (const uint8_t*)w, M, N, K, y, n_out, err, yf, bias);
    return cudaGetLastError();
}

template <int TYPE, bool GATED>
cudaError_t launch_typed(const CUtensorMap& map, const void* w, int64_t M, int64_t N, int64_t K, uint16_t* y,
                         int64_t n_out, unsigned int* err, cudaStream_t s, float* yf, const float* bias) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int64_t tiles = ((M + 255) / 256) * ((N + BN - 1) / BN);
    static const int force_acc = [] { const char* f = getenv("OCL_GEMM_ACC"); return f ? atoi(f) : 0; }();
    const bool wide = force_acc ? force_acc == 4 : wide_tokens(M, N, sms);
    if (wide) return launch_staged<TYPE, GATED, 2, 4>(map, w, M, N, K, y, n_out, err, s, yf, bias);
    if (tiles > sms) return launch_staged<TYPE, GATED, 2, 2>(map, w, M, N, K, y, n_out, err, s, yf, bias);
    return launch_staged<TYPE, GATED, 4, 2>(map, w, M, N, K, y, n_out, err, s, yf, bias);
}

}  // namespace

cudaError_t launch_qgemm(int type, const void* tiles, int64_t M, int64_t N, int64_t K, const uint16_t* x,
                         uint16_t* y, unsigned int* err, cudaStream_t s, int64_t gated_n_out, float* yf,
                         const float* bias) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return cudaErrorNotSupported;
    CUtensorMap map;
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)M};
    const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    const cuuint32_t box[2] = {BK, BOX_M};  // 64 x 256 bf16 per box: two 128-row MMA halves
    const cuuint32_t estr[2] = {1, 1};
    if (enc(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t*>(x), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return cudaErrorInvalidValue;
    if (gated_n_out > 0) {
        // interleaved gate/up: N = padded rows of both; BN = 128 keeps whole pairs per CTA
        if (type == kQ4_K) return launch_typed<kQ4_K, true>(map, tiles, M, N, K, y, gated_n_out, err, s, yf, nullptr);
        if (type == kQ6_K) return launch_typed<kQ6_K, true>(map, tiles, M, N, K, y, gated_n_out, err, s, yf, nullptr);
        return launch_typed<kQ8_0, true>(map, tiles, M, N, K, y, gated_n_out, err, s, yf, nullptr);
    }
    if (type == kQ4_K) return launch_typed<kQ4_K, false>(map, tiles, M, N, K, y, N, err, s, yf, bias);
    if (type == kQ6_K) return launch_typed<kQ6_K, false>(map, tiles, M, N, K, y, N, err, s, yf, bias);
    return launch_typed<kQ8_0, false>(map, tiles, M, N, K, y, N, err, s, yf, bias);
}

// x f32 -> bf16 (round to nearest even), the prefill GEMM's activation operand.
__global__ void cast_bf16_kernel(const float* __restrict__ x, uint16_t* __restrict__ xb, int64_t n) {
    const int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 4;
    if (i + 4 <= n && (reinterpret_cast<uintptr_t>(x) & 15) == 0) {
        const float4 v = *reinterpret_cast<const float4*>(x + i);
        *reinterpret_cast<uint2*>(xb + i) = make_uint2(pack_bf16(v.x, v.y), pack_bf16(v.z, v.w));
    } else {
        for (int64_t j = i; j < i + 4 && j < n; ++j) {
            const __nv_bfloat16 b = __float2bfloat16_rn(x[j]);
            xb[j] = *reinterpret_cast<const uint16_t*>(&b);
        }
    }
}

cudaError_t launch_cast_bf16(const float* x, uint16_t* xb, int64_t n, cudaStream_t s) {
    const int64_t threads = (n + 3) / 4;
    cast_bf16_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(x, xb, n);
    return cudaGetLastError();
}

}  // namespace ocl
