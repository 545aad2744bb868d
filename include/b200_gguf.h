/*
 * b200_gguf.h — dequantisation of GGUF k-quant weights (the GGML block formats Q4_K and
 * Q6_K that a Q4_K_M file holds) to bf16 on the GPU, for the denoising loop's linears.
 *
 * In the reference, a GGUF linear is candle's QMatMul (src/quantized_transformer.rs:14-33):
 * the weight stays in its block format and candle dequantises it for the matmul.  Here a
 * layer's blocks are dequantised into a bf16 scratch right before that layer's GEMMs (at
 * the denoising loop's batch sizes the GEMMs are compute-bound, so the scratch pass costs
 * a fraction of a percent of the step).
 *
 * Formats (GGML, QK_K = 256 weights per super-block, stored row-major along the input
 * dimension; all multi-byte fields little-endian):
 *   Q4_K, 144 bytes: f16 d, f16 dmin, 12 bytes of packed 6-bit (scale, min) for 8
 *         sub-blocks of 32, 128 bytes of 4-bit quants (64-weight chunk c: low nibbles of
 *         bytes 32c..32c+31 are its first 32 weights, high nibbles the next 32).
 *         w = (d * scale_j) * q - (dmin * min_j)
 *   Q6_K, 210 bytes: 128 bytes low 4 bits, 64 bytes high 2 bits, 16 int8 scales (one
 *         per 16 weights), f16 d.  w = (d * scale_j) * (q - 32)
 * Every product and difference is rounded to f32 separately (no fused multiply-add), then
 * rounded to bf16 (nearest even): the result equals the GGML reference dequantisation
 * rounded to bf16, bit for bit.
 *
 * Conventions are those of b200_attn.h.  `blocks` needs 16-byte alignment for Q4_K and
 * 2-byte for Q6_K; `out` 16-byte alignment.
 */
#ifndef B200_GGUF_H
#define B200_GGUF_H

#include <stddef.h>
#include <stdint.h>

#include "b200_attn.h"

#ifdef __cplusplus
extern "C" {
#endif

#define B200_QK_K 256
#define B200_Q4_K_BLOCK_BYTES 144
#define B200_Q6_K_BLOCK_BYTES 210

/* n_blocks consecutive Q4_K super-blocks -> out[n_blocks * 256] bf16. */
int b200_dequant_q4_k(const void* blocks, void* out, int64_t n_blocks, b200_stream_t stream);

/* n_blocks consecutive Q6_K super-blocks -> out[n_blocks * 256] bf16. */
int b200_dequant_q6_k(const void* blocks, void* out, int64_t n_blocks, b200_stream_t stream);

#define B200_KQUANT_Q4_K 0
#define B200_KQUANT_Q6_K 1
#define B200_KQUANT_GEMV_MAX_ROWS 2

/*
 * y[i, j] = sum_k x[i, k] * W[j, k] for i < m <= 2, j < n: the weight W [n, k] is n rows
 * of k / 256 consecutive super-blocks of `qtype` (Q4_K or Q6_K, the GGUF tensor's bytes),
 * expanded in registers to exactly the bf16 values the dequantisation above writes, and
 * never written out; products and sums in f32.  x: f32 rows ldx apart; y: f32 rows ldy apart.  The weight is read once,
 * so at a few rows the product costs about its quantised bytes at HBM speed.  Replaces
 * candle's QMatMul::forward on a batch of a few rows (src/quantized_transformer.rs:20-33:
 * the timestep embedder and the modulation linear run at one row per sequence).
 * k % 256 == 0.  B200_ERR_INVALID for m > 2: from a few rows on, the expansion work
 * repeated per row makes the dequantisation above plus a tensor-core GEMM faster.
 */
int b200_kquant_gemv(const float* x, int64_t ldx, const void* blocks, int32_t qtype, float* y,
                     int64_t ldy, int32_t m, int32_t n, int32_t k, b200_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* B200_GGUF_H */
