/*
 * oracle.c -- CPU restatement of the reference's quantized-linear arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY (see oracle.h).  Build with -ffp-contract=off so the
 * scalar paths keep Rust's "no implicit FMA" semantics; the AVX2 body uses
 * explicit FMA intrinsics exactly where the reference does.
 */
#include "oracle.h"

#include <pthread.h>
#include <stdlib.h>
#include <string.h>

#if defined(__x86_64__)
#include <immintrin.h>
#endif

/* ------------------------------------------------------------------------- */
/* f16 -> f32, crates/loader/src/safetensors_values.rs:155-183                */
/* ------------------------------------------------------------------------- */
float orc_f16_to_f32(uint16_t bits) {
    uint32_t sign = ((uint32_t)(bits & 0x8000u)) << 16;
    uint32_t exp = (bits >> 10) & 0x1fu;
    uint32_t frac = bits & 0x03ffu;
    uint32_t out;
    if (exp == 0) {
        if (frac == 0) {
            out = sign;
        } else {
            /* subnormal: renormalise */
            uint32_t f = frac;
            int32_t e = -14;
            while ((f & 0x0400u) == 0) {
                f <<= 1;
                e -= 1;
            }
            f &= 0x03ffu;
            out = sign | ((uint32_t)(e + 127) << 23) | (f << 13);
        }
    } else if (exp == 0x1f) {
        out = sign | 0x7f800000u | (frac << 13);
    } else {
        out = sign | ((exp + (127 - 15)) << 23) | (frac << 13);
    }
    float r;
    memcpy(&r, &out, 4);
    return r;
}

static uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

size_t orc_block_bytes(int t) {
    switch (t) {
        case ORC_Q4_K: return 144;
        case ORC_Q6_K: return 210;
        case ORC_Q8_0: return 34;
        default: return 0;
    }
}

size_t orc_block_elems(int t) {
    switch (t) {
        case ORC_Q4_K: return 256;
        case ORC_Q6_K: return 256;
        case ORC_Q8_0: return 32;
        default: return 0;
    }
}

/* ------------------------------------------------------------------------- */
/* Block dequantization (public GGUF block formats).                          */
/* ------------------------------------------------------------------------- */

/* Q4_K: d f16 @0, dmin f16 @2, 12 B packed 6-bit scales/mins @4, 128 B quants
 * @16.  Sub-block j (32 weights): j<4: sc=s[j]&63, m=s[j+4]&63; j>=4:
 * sc=(s[j+4]&15)|((s[j-4]>>6)<<4), m=(s[j+4]>>4)|((s[j]>>6)<<4).  Weights
 * 64c..64c+31 are the low nibbles of qs[32c..32c+31], 64c+32..64c+63 the high
 * nibbles.  y = (d*sc)*q - (dmin*m). */
static void dq_q4_k(const uint8_t* b, float* y) {
    const float d = orc_f16_to_f32(rd16(b));
    const float dmin = orc_f16_to_f32(rd16(b + 2));
    const uint8_t* s = b + 4;
    const uint8_t* qs = b + 16;
    for (int j = 0; j < 8; ++j) {
        int sc, m;
        if (j < 4) {
            sc = s[j] & 63;
            m = s[j + 4] & 63;
        } else {
            sc = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4);
            m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
        }
        const float d1 = d * (float)sc;
        const float m1 = dmin * (float)m;
        const int c = j >> 1;
        const int shift = (j & 1) ? 4 : 0;
        for (int l = 0; l < 32; ++l) {
            const int q = (qs[32 * c + l] >> shift) & 0xF;
            y[32 * j + l] = d1 * (float)q - m1;
        }
    }
}

/* Q6_K: ql[128] @0, qh[64] @128, int8 scales[16] @192, d f16 @208.  For half
 * h, l in 0..31 the four values at 128h+l+32k come from L=ql+64h, H=qh+32h:
 * q0=(L[l]&15)|((H[l]&3)<<4), q1=(L[l+32]&15)|(((H[l]>>2)&3)<<4),
 * q2=(L[l]>>4)|(((H[l]>>4)&3)<<4), q3=(L[l+32]>>4)|(((H[l]>>6)&3)<<4);
 * scale index 8h+2k+l/16; y = (d*sc)*(q-32). */
static void dq_q6_k(const uint8_t* b, float* y) {
    const uint8_t* ql = b;
    const uint8_t* qh = b + 128;
    const int8_t* sc = (const int8_t*)(b + 192);
    const float d = orc_f16_to_f32(rd16(b + 208));
    for (int h = 0; h < 2; ++h) {
        const uint8_t* L = ql + 64 * h;
        const uint8_t* H = qh + 32 * h;
        for (int l = 0; l < 32; ++l) {
            int q[4];
            q[0] = ((L[l] & 15) | ((H[l] & 3) << 4)) - 32;
            q[1] = ((L[l + 32] & 15) | (((H[l] >> 2) & 3) << 4)) - 32;
            q[2] = ((L[l] >> 4) | (((H[l] >> 4) & 3) << 4)) - 32;
            q[3] = ((L[l + 32] >> 4) | (((H[l] >> 6) & 3) << 4)) - 32;
            for (int k = 0; k < 4; ++k) {
                const float ds = d * (float)sc[8 * h + 2 * k + l / 16];
                y[128 * h + l + 32 * k] = ds * (float)q[k];
            }
        }
    }
}

/* Q8_0: d f16 @0, int8 qs[32] @2; y = d*q. */
static void dq_q8_0(const uint8_t* b, float* y) {
    const float d = orc_f16_to_f32(rd16(b));
    const int8_t* qs = (const int8_t*)(b + 2);
    for (int l = 0; l < 32; ++l) y[l] = d * (float)qs[l];
}

static int dequant_row(int t, const uint8_t* row, size_t k, float* out) {
    const size_t bb = orc_block_bytes(t), be = orc_block_elems(t);
    if (!bb || k % be) return -1;
    for (size_t i = 0; i < k / be; ++i) {
        const uint8_t* b = row + i * bb;
        float* y = out + i * be;
        if (t == ORC_Q4_K) dq_q4_k(b, y);
        else if (t == ORC_Q6_K) dq_q6_k(b, y);
        else dq_q8_0(b, y);
    }
    return 0;
}

int orc_dequant(int t, const uint8_t* blocks, size_t n_rows, size_t k, float* out) {
    const size_t bb = orc_block_bytes(t), be = orc_block_elems(t);
    if (!bb || k % be) return -1;
    const size_t row_bytes = (k / be) * bb;
    for (size_t r = 0; r < n_rows; ++r)
        if (dequant_row(t, blocks + r * row_bytes, k, out + r * k)) return -1;
    return 0;
}

/* ------------------------------------------------------------------------- */
/* Scalar multiply, crates/kernels/src/lib.rs:1974-2123.                      */
/* The reference tiles 4 rows x 4 outputs, but every output keeps its own     */
/* accumulator initialised to bias[o] (or 0) and adds x[r,k]*w[o,k] for       */
/* k = 0..K-1 in order; the per-output result is therefore exactly this loop. */
/* ------------------------------------------------------------------------- */
static float dot_seq(const float* x, const float* w, size_t k, float acc) {
    for (size_t i = 0; i < k; ++i) acc += x[i] * w[i];
    return acc;
}

int orc_linear_out_by_in(const float* x, size_t rows, size_t in_features, const float* w,
                         size_t out_features, const float* bias, float* out) {
    for (size_t r = 0; r < rows; ++r)
        for (size_t o = 0; o < out_features; ++o)
            out[r * out_features + o] =
                dot_seq(x + r * in_features, w + o * in_features, in_features, bias ? bias[o] : 0.0f);
    return 0;
}

/* ------------------------------------------------------------------------- */
/* AVX2 body, crates/kernels/src/cpu_avx2.rs:58-272.  Written against a chunk */
/* of `nout` consecutive output features starting at `o0` (weights w point at */
/* row o0); the chunking is on 4-aligned boundaries so the 4x4 tiling and the */
/* tails fall exactly where the reference puts them.                          */
/* ------------------------------------------------------------------------- */
int orc_has_avx2(void) {
#if defined(__x86_64__)
    __builtin_cpu_init();
    return __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma");
#else
    return 0;
#endif
}

#if defined(__x86_64__)
__attribute__((target("avx2,fma"))) static float hsum_ps_avx(__m256 v) {
    const __m128 hi = _mm256_extractf128_ps(v, 1);
    const __m128 lo = _mm256_castps256_ps128(v);
    const __m128 sum128 = _mm_add_ps(hi, lo);
    const __m128 shuf1 = _mm_movehdup_ps(sum128);
    const __m128 sum64 = _mm_add_ps(sum128, shuf1);
    const __m128 shuf2 = _mm_movehl_ps(shuf1, sum64);
    const __m128 sum32 = _mm_add_ss(sum64, shuf2);
    return _mm_cvtss_f32(sum32);
}

__attribute__((target("avx2,fma"))) static void avx2_chunk(const float* x, size_t rows, size_t K,
                                                         const float* w, size_t o0, size_t nout,
                                                         size_t out_features, const float* bias,
                                                         float* out) {
    const size_t tiled_rows = rows - rows % 4;
    const size_t tiled_out = nout - nout % 4;
    const size_t k_simd = K - K % 8;
    for (size_t row = 0; row < tiled_rows; row += 4) {
        const float* xr[4] = {x + row * K, x + (row + 1) * K, x + (row + 2) * K, x + (row + 3) * K};
        for (size_t od = 0; od < tiled_out; od += 4) {
            const float* wr[4] = {w + od * K, w + (od + 1) * K, w + (od + 2) * K, w + (od + 3) * K};
            __m256 acc[4][4];
            for (int a = 0; a < 4; ++a)
                for (int b = 0; b < 4; ++b) acc[a][b] = _mm256_setzero_ps();
            for (size_t k = 0; k < k_simd; k += 8) {
                __m256 xv[4], wv[4];
                for (int a = 0; a < 4; ++a) xv[a] = _mm256_loadu_ps(xr[a] + k);
                for (int b = 0; b < 4; ++b) wv[b] = _mm256_loadu_ps(wr[b] + k);
                /* acc[row offset][output offset] */
                for (int a = 0; a < 4; ++a)
                    for (int b = 0; b < 4; ++b) acc[a][b] = _mm256_fmadd_ps(xv[a], wv[b], acc[a][b]);
            }
            float s[4][4];
            for (int a = 0; a < 4; ++a)
                for (int b = 0; b < 4; ++b) s[a][b] = hsum_ps_avx(acc[a][b]);
            for (size_t kt = k_simd; kt < K; ++kt)
                for (int a = 0; a < 4; ++a)
                    for (int b = 0; b < 4; ++b) s[a][b] += xr[a][kt] * wr[b][kt];
            for (int a = 0; a < 4; ++a)
                for (int b = 0; b < 4; ++b)
                    out[(row + a) * out_features + o0 + od + b] =
                        s[a][b] + (bias ? bias[o0 + od + b] : 0.0f);
        }
        for (size_t to = tiled_out; to < nout; ++to) {
            const float bv = bias ? bias[o0 + to] : 0.0f;
            for (int a = 0; a < 4; ++a)
                out[(row + a) * out_features + o0 + to] = dot_seq(xr[a], w + to * K, K, bv);
        }
    }
    for (size_t row = tiled_rows; row < rows; ++row)
        for (size_t od = 0; od < nout; ++od)
            out[row * out_features + o0 + od] =
                dot_seq(x + row * K, w + od * K, K, bias ? bias[o0 + od] : 0.0f);
}
#endif

int orc_linear_out_by_in_avx2(const float* x, size_t rows, size_t in_features, const float* w,
                              size_t out_features, const float* bias, float* out) {
#if defined(__x86_64__)
    if (!orc_has_avx2()) return -2;
    avx2_chunk(x, rows, in_features, w, 0, out_features, out_features, bias, out);
    return 0;
#else
    return -2;
#endif
}

/* ------------------------------------------------------------------------- */
/* Quantized linear: dequantize a chunk of weight rows, multiply that chunk.   */
/* ------------------------------------------------------------------------- */
typedef struct {
    int type, avx2;
    const uint8_t* blocks;
    const float* x;
    size_t rows, K, N, o_begin, o_end;
    const float* bias;
    float* out;
    int status;
} qjob;

enum { CHUNK = 4 }; /* keeps chunk starts 4-aligned, matching the AVX2 tiling */

static void* q_worker(void* arg) {
    qjob* j = (qjob*)arg;
    const size_t row_bytes = (j->K / orc_block_elems(j->type)) * orc_block_bytes(j->type);
    float* wbuf = (float*)malloc(sizeof(float) * CHUNK * j->K);
    if (!wbuf) {
        j->status = -3;
        return NULL;
    }
    for (size_t o = j->o_begin; o < j->o_end; o += CHUNK) {
        const size_t n = (j->o_end - o) < CHUNK ? (j->o_end - o) : CHUNK;
        for (size_t i = 0; i < n; ++i) dequant_row(j->type, j->blocks + (o + i) * row_bytes, j->K, wbuf + i * j->K);
#if defined(__x86_64__)
        if (j->avx2) {
            avx2_chunk(j->x, j->rows, j->K, wbuf, o, n, j->N, j->bias, j->out);
            continue;
        }
#endif
        for (size_t r = 0; r < j->rows; ++r)
            for (size_t i = 0; i < n; ++i)
                j->out[r * j->N + o + i] =
                    dot_seq(j->x + r * j->K, wbuf + i * j->K, j->K, j->bias ? j->bias[o + i] : 0.0f);
    }
    free(wbuf);
    j->status = 0;
    return NULL;
}

static int q_linear_impl(int t, const uint8_t* blocks, const float* x, size_t rows, size_t K,
                         size_t N, const float* bias, float* out, int threads, int avx2) {
    if (!orc_block_bytes(t) || K % orc_block_elems(t)) return -1;
    if (avx2 && !orc_has_avx2()) return -2;
    if (threads < 1) threads = 1;
    size_t chunks = (N + CHUNK - 1) / CHUNK;
    if ((size_t)threads > chunks) threads = (int)(chunks ? chunks : 1);
    qjob* jobs = (qjob*)calloc((size_t)threads, sizeof(qjob));
    pthread_t* tids = (pthread_t*)calloc((size_t)threads, sizeof(pthread_t));
    if (!jobs || !tids) {
        free(jobs);
        free(tids);
        return -3;
    }
    size_t per = (chunks + (size_t)threads - 1) / (size_t)threads;
    for (int i = 0; i < threads; ++i) {
        size_t b = (size_t)i * per * CHUNK, e = b + per * CHUNK;
        if (b > N) b = N;
        if (e > N) e = N;
        jobs[i] = (qjob){t, avx2, blocks, x, rows, K, N, b, e, bias, out, 0};
    }
    int rc = 0;
    if (threads == 1) {
        q_worker(&jobs[0]);
    } else {
        for (int i = 0; i < threads; ++i) pthread_create(&tids[i], NULL, q_worker, &jobs[i]);
        for (int i = 0; i < threads; ++i) pthread_join(tids[i], NULL);
    }
    for (int i = 0; i < threads; ++i)
        if (jobs[i].status) rc = jobs[i].status;
    free(jobs);
    free(tids);
    return rc;
}

int orc_q_linear(int t, const uint8_t* blocks, const float* x, size_t rows, size_t K, size_t N,
                 const float* bias, float* out, int threads) {
    return q_linear_impl(t, blocks, x, rows, K, N, bias, out, threads, 0);
}

int orc_q_linear_avx2(int t, const uint8_t* blocks, const float* x, size_t rows, size_t K, size_t N,
                      const float* bias, float* out, int threads) {
    return q_linear_impl(t, blocks, x, rows, K, N, bias, out, threads, 1);
}
