// repack.cu -- GGUF blocks <-> TILED16 records, dequantization, Q8_0 row gather.
//
// None of these is on the per-token hot path except the embedding gather; they
// run at weight-upload time (repack), for DeviceBuffer::to_host (dequant), and for
// the layout round-trip check (unpack).  All are plain integer/byte work: one
// thread per output 32-bit word, grid-stride, coalesced writes.
#include "internal.cuh"

namespace ocl {

namespace {

// Source byte of a GGUF block for the TILED16 record byte `o` of row tile `rt`,
// k-group `kb`.  Rows >= n_rows read as zero.
__device__ inline uint32_t tiled_byte(int type, const uint8_t* __restrict__ src, int64_t n_rows,
                                      int64_t nkb, int64_t rt, int64_t kb, int o) {
    const int bb = block_bytes(type);
    auto blk = [&](int r) -> const uint8_t* {
        const int64_t row = rt * 16 + r;
        return row < n_rows ? src + (row * nkb + kb) * bb : nullptr;
    };
    if (type == kQ4_K) {
        if (o < 256) {
            const uint8_t* b = blk(o >> 4);
            return b ? b[o & 15] : 0u;
        }
        const int p = o - 256, c = p >> 9, lane = (p >> 4) & 31, w = p & 15;
        const int g = lane >> 2, t = lane & 3, half = w >> 3, i = w & 7;
        const uint8_t* b = blk(g + 8 * half);
        return b ? b[16 + 32 * c + 8 * t + i] : 0u;
    }
    if (type == kQ6_K) {
        if (o < 256) {
            const uint8_t* b = blk(o >> 4);
            return b ? b[192 + (o & 15)] : 0u;
        }
        if (o < 288) {
            const uint8_t* b = blk((o - 256) >> 1);
            return b ? b[208 + (o & 1)] : 0u;
        }
        if (o < 2336) {
            const int p = o - 288, u = p >> 9, lane = (p >> 4) & 31, w = (p >> 2) & 3, i = p & 3;
            const int g = lane >> 2, t = lane & 3, j = 4 * u + w, k = 16 * j + 4 * t + i;
            const uint8_t* b0 = blk(g);
            const uint8_t* b1 = blk(g + 8);
            const uint32_t lo0 = b0 ? (q6k_get(b0, k) & 15) : 0u;
            const uint32_t lo1 = b1 ? (q6k_get(b1, k) & 15) : 0u;
            return lo0 | (lo1 << 4);
        }
        const int p = o - 2336, v = p >> 9, lane = (p >> 4) & 31, w = (p >> 2) & 3, i = p & 3;
        const int g = lane >> 2, t = lane & 3, j0 = 8 * v + 2 * w;
        const int k0 = 16 * j0 + 4 * t + i, k1 = k0 + 16;
        const uint8_t* b0 = blk(g);
        const uint8_t* b1 = blk(g + 8);
        uint32_t r = 0;
        if (b0) r |= (uint32_t)(q6k_get(b0, k0) >> 4) | ((uint32_t)(q6k_get(b0, k1) >> 4) << 4);
        if (b1) r |= ((uint32_t)(q6k_get(b1, k0) >> 4) << 2) | ((uint32_t)(q6k_get(b1, k1) >> 4) << 6);
        return r;
    }
    // Q8_0
    if (o < 32) {
        const uint8_t* b = blk(o >> 1);
        return b ? b[o & 1] : 0u;
    }
    const int p = o - 32, lane = p >> 4, w = p & 15;
    const int g = lane >> 2, t = lane & 3, hi16 = w >> 3, half = (w >> 2) & 1, i = w & 3;
    const uint8_t* b = blk(g + 8 * half);
    return b ? b[2 + 16 * hi16 + 4 * t + i] : 0u;
}

__global__ void repack_kernel(int type, const uint8_t* __restrict__ src, int64_t n_rows, int64_t nkb,
                              int64_t n_rt, uint32_t* __restrict__ dst) {
    const int rb = rec_bytes(type);
    const int64_t words = n_rt * nkb * (rb / 4);
    for (int64_t wi = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; wi < words;
         wi += (int64_t)gridDim.x * blockDim.x) {
        const int64_t byte = wi * 4;
        const int64_t rec = byte / rb;
        const int o = (int)(byte - rec * rb);
        const int64_t rt = rec / nkb, kb = rec - rt * nkb;
        uint32_t v = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) v |= tiled_byte(type, src, n_rows, nkb, rt, kb, o + i) << (8 * i);
        dst[wi] = v;
    }
}

// Value of element k (0..rec_k-1) of local row r from one record, dequantized.
__device__ inline float tiled_value(int type, const uint8_t* __restrict__ rec, int r, int k) {
    if (type == kQ4_K) {
        const float d = f16_bits_to_f32(rec[16 * r] | (rec[16 * r + 1] << 8));
        const float dmin = f16_bits_to_f32(rec[16 * r + 2] | (rec[16 * r + 3] << 8));
        const int j = k >> 5, c = j >> 1, l = k & 31;
        int sc, m;
        q4k_scale_min(rec + 16 * r + 4, j, sc, m);
        const int q = (rec[t4_qs_off(r, c, l)] >> (4 * (j & 1))) & 15;
        const float d1 = __fmul_rn(d, (float)sc);
        const float m1 = __fmul_rn(dmin, (float)m);
        return __fsub_rn(__fmul_rn(d1, (float)q), m1);
    }
    if (type == kQ6_K) {
        int lo_off, lo_sh, hi_off, hi_sh;
        t6_pos(r, k, lo_off, lo_sh, hi_off, hi_sh);
        const int q = ((rec[lo_off] >> lo_sh) & 15) | (((rec[hi_off] >> hi_sh) & 3) << 4);
        const float d = f16_bits_to_f32(rec[256 + 2 * r] | (rec[257 + 2 * r] << 8));
        const float ds = __fmul_rn(d, (float)(int8_t)rec[16 * r + (k >> 4)]);
        return __fmul_rn(ds, (float)(q - 32));
    }
    const float d = f16_bits_to_f32(rec[2 * r] | (rec[2 * r + 1] << 8));
    return __fmul_rn(d, (float)(int8_t)rec[t8_q_off(r, k)]);
}

__global__ void dequant_kernel(int type, const uint8_t* __restrict__ tiles, int64_t n_rows, int64_t k,
                               float* __restrict__ out) {
    const int rk = rec_k(type), rb = rec_bytes(type);
    const int64_t nkb = k / rk;
    const int64_t total = n_rows * k;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t row = i / k, col = i - row * k;
        const int64_t kb = col / rk;
        const uint8_t* rec = tiles + ((row >> 4) * nkb + kb) * rb;
        out[i] = tiled_value(type, rec, (int)(row & 15), (int)(col - kb * rk));
    }
}

// TILED16 -> GGUF blocks, one thread per output byte of each GGUF block.
__global__ void unpack_kernel(int type, const uint8_t* __restrict__ tiles, int64_t n_rows, int64_t nkb,
                              uint8_t* __restrict__ dst) {
    const int bb = block_bytes(type), rb = rec_bytes(type);
    const int64_t total = n_rows * nkb * bb;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t blk = i / bb;
        const int b = (int)(i - blk * bb);
        const int64_t row = blk / nkb, kb = blk - row * nkb;
        const uint8_t* rec = tiles + ((row >> 4) * nkb + kb) * rb;
        const int r = (int)(row & 15);
        uint32_t v;
        if (type == kQ4_K) {
            if (b < 16) v = rec[16 * r + b];
            else {
                const int p = b - 16;
                v = rec[t4_qs_off(r, p >> 5, p & 31)];
            }
        } else if (type == kQ6_K) {
            auto q6 = [&](int e) {
                int lo_off, lo_sh, hi_off, hi_sh;
                t6_pos(r, e, lo_off, lo_sh, hi_off, hi_sh);
                return (uint32_t)(((rec[lo_off] >> lo_sh) & 15) | (((rec[hi_off] >> hi_sh) & 3) << 4));
            };
            if (b < 128) {  // ql[64h + l'] = lo4(128h+l') | lo4(128h+l'+64) << 4
                const int h = b >> 6, lp = b & 63;
                v = (q6(128 * h + lp) & 15) | ((q6(128 * h + lp + 64) & 15) << 4);
            } else if (b < 192) {  // qh[32h + l]: bits 2kq.. = hi2 of element 128h + l + 32kq
                const int p = b - 128, h = p >> 5, l = p & 31;
                v = 0;
                for (int kq = 0; kq < 4; ++kq) v |= (q6(128 * h + l + 32 * kq) >> 4) << (2 * kq);
            } else if (b < 208) {
                v = rec[16 * r + (b - 192)];
            } else {
                v = rec[256 + 2 * r + (b - 208)];
            }
        } else {
            if (b < 2) v = rec[2 * r + b];
            else v = rec[t8_q_off(r, b - 2)];
        }
        dst[i] = (uint8_t)v;
    }
}

// Q8_0 gather of whole rows.  Bad ids write zeros and bump *bad.
__global__ void embed_kernel(const uint8_t* __restrict__ tiles, int64_t n_rows, int64_t k,
                             const int32_t* __restrict__ ids, int64_t n_ids, float* __restrict__ out,
                             unsigned int* __restrict__ bad) {
    const int64_t nkb = k / 32;
    const int64_t total = n_ids * k;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t n = i / k, col = i - n * k;
        const int64_t id = ids[n];
        if (id < 0 || id >= n_rows) {
            out[i] = 0.0f;
            if (col == 0) atomicAdd(bad, 1u);
            continue;
        }
        const int64_t kb = col >> 5;
        const uint8_t* rec = tiles + ((id >> 4) * nkb + kb) * 544;
        out[i] = tiled_value(kQ8_0, rec, (int)(id & 15), (int)(col & 31));
    }
}

int grid_for(int64_t work, int threads) {
    int64_t g = (work + threads - 1) / threads;
    if (g > 148 * 64) g = 148 * 64;
    if (g < 1) g = 1;
    return (int)g;
}

}  // namespace

cudaError_t launch_repack(int type, const void* src, int64_t n_rows, int64_t k, void* dst, cudaStream_t s) {
    const int64_t nkb = k / rec_k(type), n_rt = (n_rows + 15) / 16;
    const int64_t words = n_rt * nkb * (rec_bytes(type) / 4);
    repack_kernel<<<grid_for(words, 256), 256, 0, s>>>(type, (const uint8_t*)src, n_rows, nkb, n_rt,
                                                      (uint32_t*)dst);
    return cudaGetLastError();
}

cudaError_t launch_dequant(int type, const void* tiles, int64_t n_rows, int64_t k, float* out, cudaStream_t s) {
    dequant_kernel<<<grid_for(n_rows * k, 256), 256, 0, s>>>(type, (const uint8_t*)tiles, n_rows, k, out);
    return cudaGetLastError();
}

cudaError_t launch_unpack(int type, const void* tiles, int64_t n_rows, int64_t k, void* dst, cudaStream_t s) {
    const int64_t nkb = k / block_elems(type);
    unpack_kernel<<<grid_for(n_rows * nkb * block_bytes(type), 256), 256, 0, s>>>(
        type, (const uint8_t*)tiles, n_rows, nkb, (uint8_t*)dst);
    return cudaGetLastError();
}

cudaError_t launch_embed(const void* tiles, int64_t n_rows, int64_t k, const int32_t* ids, int64_t n_ids,
                         float* out, unsigned int* bad, cudaStream_t s) {
    embed_kernel<<<grid_for(n_ids * k, 256), 256, 0, s>>>((const uint8_t*)tiles, n_rows, k, ids, n_ids, out, bad);
    return cudaGetLastError();
}

}  // namespace ocl
