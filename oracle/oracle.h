/*
 * oracle.h -- CPU restatement of the reference's quantized-linear arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (the ocelotl_b200 package,
 * its CUDA library or the C ABI in include/) links, loads or calls this code.
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use it,
 * and only as the checker / the timed CPU reference.
 *
 * What it restates (paths are inside the Dieshen/ocelotl workspace):
 *   - f16 -> f32: crates/loader/src/safetensors_values.rs:155-183
 *   - multiply:   crates/kernels/src/lib.rs:1974-2123 (linear_out_by_in_compute:
 *                 bias-initialised accumulator, sequential k per output, f32,
 *                 no FMA contraction -- rustc never contracts a*b+c)
 *   - AVX2 body:  crates/kernels/src/cpu_avx2.rs:58-272 (8-lane FMA partial
 *                 sums, hsum_ps_avx, scalar k tail, bias added last)
 *   - validation: crates/kernels/src/lib.rs:2443-2494 (length checks)
 *   - row-chunk threading: crates/kernels/src/lib.rs:2294-2391 (disjoint
 *                 output chunks, bit-identical to serial)
 * The dequantize half has no code in the reference: the workspace only names the
 * GGUF type tags (crates/loader/src/gguf_inspect.rs:140,144,146 -> Q8_0=8,
 * Q4K=12, Q6K=14) and rejects quantized weights before compute.  The block
 * arithmetic is the public GGUF/ggml block format (third-party, not vendored in
 * the reference); it is pinned bit-for-bit by tests/golden fixtures produced with
 * the `gguf` 0.19.0 Python package (`gguf.quants.dequantize`).
 */
#ifndef OCELOTL_ORACLE_H
#define OCELOTL_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GGUF tensor-type tags (crates/loader/src/gguf_inspect.rs:178,182,184). */
enum { ORC_Q8_0 = 8, ORC_Q4_K = 12, ORC_Q6_K = 14 };

float orc_f16_to_f32(uint16_t bits);

/* Bytes per block and weights per block for a supported tag; 0 otherwise. */
size_t orc_block_bytes(int ggml_type);
size_t orc_block_elems(int ggml_type);

/* Dequantize n_rows rows of k weights each (row-major GGUF blocks along k). */
int orc_dequant(int ggml_type, const uint8_t* blocks, size_t n_rows, size_t k, float* out);

/* Scalar linear_out_by_in: out[r,o] = bias[o] + sum_k x[r,k]*w[o,k]. */
int orc_linear_out_by_in(const float* x, size_t rows, size_t in_features,
                         const float* w, size_t out_features, const float* bias,
                         float* out);

/* AVX2+FMA linear_out_by_in restatement (x86-64 with avx2+fma only). */
int orc_linear_out_by_in_avx2(const float* x, size_t rows, size_t in_features,
                              const float* w, size_t out_features, const float* bias,
                              float* out);

/* Quantized linear: dequantize each weight row, then the scalar multiply for that
 * output feature.  Bit-identical to orc_dequant + orc_linear_out_by_in (same
 * per-output accumulation order) but needs only one row of f32 scratch per
 * thread.  threads <= 1 runs serially; otherwise output features are split into
 * contiguous chunks, one per thread (bit-identical to serial). */
int orc_q_linear(int ggml_type, const uint8_t* blocks, const float* x, size_t rows,
                 size_t in_features, size_t out_features, const float* bias, float* out,
                 int threads);

/* Same, with the AVX2 multiply body (mode "avx2" of the reference CPU backend). */
int orc_q_linear_avx2(int ggml_type, const uint8_t* blocks, const float* x, size_t rows,
                      size_t in_features, size_t out_features, const float* bias,
                      float* out, int threads);

/* 1 when the host supports avx2 and fma. */
int orc_has_avx2(void);

#ifdef __cplusplus
}
#endif
#endif
