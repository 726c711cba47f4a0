// layout.cuh -- GGUF block formats and the TILED16 device layout.
//
// GGUF block formats (public ggml format; the reference only names the tags,
// crates/loader/src/gguf_inspect.rs:140,144,146):
//   Q4_K  256 weights / 144 B: d f16 @0, dmin f16 @2, scales[12] @4, qs[128] @16
//   Q6_K  256 weights / 210 B: ql[128] @0, qh[64] @128, int8 scales[16] @192, d f16 @208
//   Q8_0   32 weights /  34 B: d f16 @0, int8 qs[32] @2
//
// TILED16 layout.  Rows are grouped in tiles of 16 (rows past N are zero-filled).
// Tile records are stored [row_tile][k_group] so one row tile's K stream is
// contiguous.  Inside a record, lane L of a warp (g = L/4, t = L%4) owns rows g
// and g+8; every 16-byte chunk a lane loads is exactly the A-operand fragment of
// one or two m16n8kX int8 tensor-core MMAs for those rows.  Record maps:
//
// Q4_K record = 16 rows x 256 k, 2304 B:
//   [0,256)      row r header at 16r: the 16 GGUF header bytes (d, dmin, scales)
//   [256,2304)   quants: chunk (c, L) at 256 + 512c + 16L, c = 0..3:
//                bytes 0..7  = row g   qs[32c+8t .. 32c+8t+7]
//                bytes 8..15 = row g+8 qs[32c+8t .. 32c+8t+7]
//                low nibbles feed sub-block 2c, high nibbles sub-block 2c+1; MMA
//                slot 4t+i <-> k = 8t+i, slot 16+4t+i <-> k = 8t+4+i (i = 0..3).
// Q6_K record = 16 rows x 256 k, 3360 B:
//   [0,256)      row r int8 scales[16] at 16r
//   [256,288)    row r d (f16) at 256+2r
//   [288,2336)   low 4 bits: chunk (u, L) at 288 + 512u + 16L, u = 0..3; 32-bit
//                word w is sub-block j = 4u+w; nibble 2i = row g, nibble 2i+1 =
//                row g+8, value at k = 16j + 4t + i.
//   [2336,3360)  high 2 bits: chunk (v, L) at 2336 + 512v + 16L, v = 0..1; word w
//                is the sub-block pair j0 = 8v+2w, j1 = j0+1; in byte i bits 0-1 =
//                row g (j0), 2-3 = row g+8 (j0), 4-5 = row g (j1), 6-7 = row g+8 (j1),
//                value at k = 16j + 4t + i.
// Q8_0 record = 16 rows x 32 k (one block), 544 B:
//   [0,32)       row r d (f16) at 2r
//   [32,544)     chunk L at 32 + 16L: bytes 0..3 row g q[4t..], 4..7 row g+8 q[4t..],
//                8..11 row g q[16+4t..], 12..15 row g+8 q[16+4t..]
//
// Each record has the same byte count as the 16 GGUF blocks it holds.
#pragma once
#include <cstddef>
#include <cstdint>

namespace ocl {

constexpr int kQ8_0 = 8, kQ4_K = 12, kQ6_K = 14;

__host__ __device__ constexpr int block_bytes(int t) {
    return t == kQ4_K ? 144 : t == kQ6_K ? 210 : t == kQ8_0 ? 34 : 0;
}
__host__ __device__ constexpr int block_elems(int t) {
    return t == kQ4_K ? 256 : t == kQ6_K ? 256 : t == kQ8_0 ? 32 : 0;
}
// Bytes of one TILED16 record and the k it covers.
__host__ __device__ constexpr int rec_bytes(int t) {
    return t == kQ4_K ? 2304 : t == kQ6_K ? 3360 : t == kQ8_0 ? 544 : 0;
}
__host__ __device__ constexpr int rec_k(int t) { return block_elems(t); }

// IEEE binary16 -> binary32, exact for every input (subnormals renormalised,
// inf/NaN payload kept), same result as f16_bits_to_f32 in
// crates/loader/src/safetensors_values.rs:155-183.
__host__ __device__ inline float f16_bits_to_f32(uint32_t h) {
    const uint32_t sign = (h & 0x8000u) << 16;
    const uint32_t exp = (h >> 10) & 0x1fu;
    const uint32_t frac = h & 0x3ffu;
    uint32_t bits;
    if (exp == 0) {
        if (frac == 0) {
            bits = sign;
        } else {
#ifdef __CUDA_ARCH__
            const int shift = __clz(frac) - 21;
#else
            const int shift = __builtin_clz(frac) - 21;
#endif
            bits = sign | ((uint32_t)(127 - 14 - shift) << 23) | (((frac << shift) & 0x3ffu) << 13);
        }
    } else if (exp == 0x1f) {
        bits = sign | 0x7f800000u | (frac << 13);
    } else {
        bits = sign | ((exp + 112u) << 23) | (frac << 13);
    }
    union { uint32_t u; float f; } v;
    v.u = bits;
    return v.f;
}

// Q4_K 6-bit scale / min of sub-block j from the 12 packed bytes.
__host__ __device__ inline void q4k_scale_min(const uint8_t* s, int j, int& sc, int& m) {
    if (j < 4) {
        sc = s[j] & 63;
        m = s[j + 4] & 63;
    } else {
        sc = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4);
        m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

// 6-bit quant (0..63) of element e (0..255) of a GGUF Q6_K block.
__host__ __device__ inline int q6k_get(const uint8_t* blk, int e) {
    const int h = e >> 7, r = e & 127, kq = r >> 5, l = r & 31;
    const uint8_t* L = blk + 64 * h;
    const uint8_t* H = blk + 128 + 32 * h;
    const int lo = (kq & 1) ? L[l + 32] : L[l];
    const int lo4 = (kq & 2) ? (lo >> 4) : (lo & 15);
    const int hi2 = (H[l] >> (2 * kq)) & 3;
    return lo4 | (hi2 << 4);
}

// ---- TILED16 accessors (byte offsets inside one record) -------------------
// Q4_K: byte of qs[32c + l] for local row r (0..15).
__host__ __device__ inline int t4_qs_off(int r, int c, int l) {
    const int g = r & 7, half = r >> 3, t = l >> 3;
    return 256 + 512 * c + 16 * (4 * g + t) + 8 * half + (l & 7);
}
// Q6_K: (nibble byte offset, nibble shift) and (crumb byte offset, shift) of
// element k (0..255) of local row r.
__host__ __device__ inline void t6_pos(int r, int k, int& lo_off, int& lo_sh, int& hi_off, int& hi_sh) {
    const int g = r & 7, half = r >> 3;
    const int j = k >> 4, t = (k >> 2) & 3, i = k & 3;
    const int lane = 4 * g + t;
    // low nibble: word w = j%4 of chunk u = j/4; nibble index 2i+half
    const int nib = 2 * i + half;
    lo_off = 288 + 512 * (j >> 2) + 16 * lane + 4 * (j & 3) + (nib >> 1);
    lo_sh = 4 * (nib & 1);
    // crumb: chunk v = j/8, word w = (j%8)/2, byte i, bits 2*(2*(j&1)+half)
    hi_off = 2336 + 512 * (j >> 3) + 16 * lane + 4 * ((j & 7) >> 1) + i;
    hi_sh = 2 * (2 * (j & 1) + half);
}
// Q8_0: byte of q[k] (k = 0..31) for local row r.
__host__ __device__ inline int t8_q_off(int r, int k) {
    const int g = r & 7, half = r >> 3;
    const int hi16 = k >> 4, t = (k >> 2) & 3, i = k & 3;
    return 32 + 16 * (4 * g + t) + 8 * hi16 + 4 * half + i;
}

}  // namespace ocl
