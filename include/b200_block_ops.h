/*
 * b200_block_ops.h — C ABI of the elementwise steps of the Qwen-Image-2.1 single-stream
 * block that sit between its GEMMs (src/transformer.rs:396-427), used by the denoising
 * loop built around the attention path (b200attn/mmdit.py).  These are not part of the
 * attention drop-in boundary (b200_attn.h): in the reference they are candle ops of
 * TransformerBlock::forward, GatedMlp::forward and FinalLayer::forward.
 *
 * Conventions are those of b200_attn.h: device pointers owned by the caller, 16-byte
 * aligned; work on the caller's stream; 0 or a negative b200_status; never abort.
 */
#ifndef B200_BLOCK_OPS_H
#define B200_BLOCK_OPS_H

#include <stddef.h>
#include <stdint.h>

#include "b200_attn.h"

#ifdef __cplusplus
extern "C" {
#endif

/*
 * Gated residual add followed by the modulated LayerNorm of the next branch, one pass
 * over the f32 residual stream x [rows, cols]:
 *
 *   if (y)   x[r,:] += tanh(gate[m,:]) * y[r,:]            (x updated in place)
 *   if (out) out[r,:] = LN(x[r,:]) * (1 + scale[m,:])      (bf16)
 *
 * with m = r / rows_per_mod the modulation row of token r (the tokens of one sequence
 * share their timestep's modulation), gate/scale rows mod_stride floats apart, and LN the
 * affine-free LayerNorm of the reference (weight 1, bias 0, eps 1e-6; fixed_layer_norm,
 * src/transformer.rs:364-372).  Replaces, per block, `x.broadcast_add(tanh(gate) *
 * branch)` followed by `norm(x) * (1 + scale)` (src/transformer.rs:411-424), and
 * FinalLayer::forward's `norm(x) * (1 + scale)` (src/transformer.rs:448-454).  y (bf16)
 * may be NULL (no residual add: the first block's norm1); out may be NULL (residual add
 * only).
 * Requires cols % 4 == 0 and cols <= 8192.
 */
int b200_residual_adaln(float* x, const void* y, const float* gate, const float* scale,
                        void* out, int64_t rows, int32_t cols, int64_t rows_per_mod,
                        int64_t mod_stride, float eps, b200_stream_t stream);

/*
 * SwiGLU of GatedMlp::forward (src/transformer.rs:326-331):
 *   h[r, j] = silu(gp[r, j]) * gp[r, F + j]      (bf16 in, f32 math, bf16 out)
 * where gp [rows, 2F] is the output of one GEMM against the stacked weights
 * [gate_layer ; proj] (the activation is on gate_layer).  Requires F % 8 == 0.
 */
int b200_swiglu(const void* gp, void* h, int64_t rows, int32_t ffn, b200_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* B200_BLOCK_OPS_H */
