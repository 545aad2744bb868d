/*
 * b200_gemm.h — C = A · Bᵀ on the sm_100a tensor cores, and the out-projection of
 * head-sharded attention fused with the reduction of its partial sums across GPUs.
 *
 * In the reference, `to_out` (src/transformer.rs:196) is one Linear on one GPU.  Sharding
 * the heads over N GPUs gives each GPU the input columns of its heads, so each computes a
 * full-width partial [T, hidden] and the N partials must be summed on every GPU (an
 * all-reduce).  Here that is two launches per GPU around the caller's barriers:
 *   1. b200_gemm_scatter: the GEMM's epilogue stores each partial tile, in bf16, straight
 *      into the GPU that owns its rows (rows are split into N equal blocks), into that
 *      owner's slot for this GPU — plain stores over NVLink, as soon as the tile is done
 *      (the reduce-scatter traffic overlaps the GEMM);
 *   2. b200_reduce_gather_bf16: each owner sums its N slots in f32 in a fixed order
 *      (deterministic) and writes the bf16 rows into every GPU's output buffer.
 * Per GPU each launch moves (N-1)/N of the output over NVLink, as a ring all-reduce does.
 * The caller orders: every GPU done reading the previous output before (1); every GPU's
 * (1) before any (2); every (2) before the output is read — e.g. a symmetric-memory or
 * NCCL barrier between the launches.
 *
 * Conventions are those of b200_attn.h.
 *   A: [M, K] bf16, row stride lda elements (lda >= K, lda % 8 == 0), 16-byte aligned
 *   B: [N, K] bf16, row stride ldb (a Linear weight [out, in], or a column slice of one)
 *   C: [M, N] with row stride ldc (ldc >= N, ldc % 8 == 0), 16-byte aligned
 *   K % 8 == 0, N % 32 == 0; any M.
 * status: optional device int32, set non-zero if a device-side wait ran out.
 */
#ifndef B200_GEMM_H
#define B200_GEMM_H

#include <stddef.h>
#include <stdint.h>

#include "b200_attn.h"

#ifdef __cplusplus
extern "C" {
#endif

#define B200_GEMM_STORE_BF16 0    /* C bf16 = A·Bᵀ                                       */
#define B200_GEMM_RED_F32 1       /* C f32 += A·Bᵀ (red.global.add; C may be a peer's)    */
#define B200_GEMM_SCATTER_BF16 2  /* internal: the epilogue of b200_gemm_scatter          */
#define B200_GEMM_QKV 3           /* internal: the epilogue of b200_qkv_norm_rope_gemm    */
#define B200_GEMM_MAX_OWNERS 8

int b200_gemm(const void* a, int64_t lda, const void* b, int64_t ldb, void* c, int64_t ldc,
              int32_t m, int32_t n, int32_t k, int32_t mode, int32_t* status,
              b200_stream_t stream);

/*
 * A · Bᵀ with row m stored (bf16) into owner q = m / rows_per_owner, slot src_slot:
 * owner_bufs[q] + (src_slot * rows_per_owner + m - q * rows_per_owner) * ldc.
 * owner_bufs: host array of n_owners (<= 8) device pointers (peer pointers for other
 * GPUs), each a buffer of n_owners * rows_per_owner rows; n_owners * rows_per_owner >= M.
 */
int b200_gemm_scatter(const void* a, int64_t lda, const void* b, int64_t ldb,
                      void* const* owner_bufs, int32_t n_owners, int32_t src_slot,
                      int32_t rows_per_owner, int64_t ldc, int32_t m, int32_t n, int32_t k,
                      int32_t* status, b200_stream_t stream);

/*
 * out[dst_row0 + r, :] = bf16(sum over s < n_src of slots[s * slot_rows + r, :]) for
 * r < rows (<= slot_rows), written into each of the n_dst (<= 8) buffers dst_bufs (host
 * array of device pointers, peer pointers for other GPUs).  slots: bf16
 * [n_src * slot_rows, ld]; cols % 8 == 0.
 */
int b200_reduce_gather_bf16(const void* slots, int32_t n_src, int32_t slot_rows, int32_t rows,
                            int32_t cols, int64_t ld, void* const* dst_bufs, int32_t n_dst,
                            int64_t dst_row0, int64_t dst_ld, b200_stream_t stream);

/*
 * The owner's step of a head-sharded block with the tanh-gated residual and the next
 * modulated LayerNorm fused in: for r < rows (<= slot_rows),
 *   sum       = sum over s < n_src of slots[s * slot_rows + r, :]   (f32, fixed order)
 *   x[r, :]  += tanh(gate[m, :]) * sum                              (f32, in place)
 *   out[dst_row0 + r, :] = bf16(LN(x[r, :]) * (1 + scale[m, :]))   into every dst buffer
 * with m = (dst_row0 + r) / rows_per_mod (gate / scale rows mod_stride floats apart) and LN
 * the reference's affine-free LayerNorm (eps).  x [rows, ldx] f32 holds the owner's rows of
 * the residual stream (the stream is split over the ranks like the reduce-scatter); the
 * bf16 result, all-gathered, is the next GEMM's input.  Replaces, for the head-sharded
 * block, the sum of the to_out partials followed by `x + tanh(gate1) * attn` and
 * `norm2(x) * (1 + scale2)` (src/transformer.rs:196, 411-418).  cols % 8 == 0, cols <= 8192.
 */
/*
 * The owner's step with the reduction done by the NVSwitch.  mc_part / mc_out are CUDA
 * multicast addresses (cuMulticast objects, e.g. torch symmetric memory's multicast_ptr)
 * bound to every rank's bf16 partial [*, part_ld] and output [*, out_ld] buffers.  For
 * r < rows, row g = row0 + r:
 *   sum    = multimem.ld_reduce add over the ranks of part[g, :]  (f32 accumulate, bf16)
 *   x == NULL:  out[g, :] = sum                                    on every rank
 *   else:       x[r, :] += tanh(gate[m, :]) * sum ;  out[g, :] = bf16(LN(x[r]) (1 + scale[m]))
 * with m = g / rows_per_mod, as b200_reduce_residual_adaln_gather.  Every rank's partial
 * must be complete (a barrier) before the call and every owner's call must finish (a
 * barrier) before `out` is read.  Per GPU, NVLink carries (1 + 1/N) partials each way
 * instead of the 2 (N-1)/N of the scatter / gather pair, so it pays from N = 4 up.
 * The result is deterministic up to the switch's reduction order.  cols % 8 == 0,
 * cols <= 8192; 16-byte aligned addresses.
 */
int b200_reduce_nvls(const void* mc_part, int64_t part_ld, void* mc_out, int64_t out_ld,
                     int64_t row0, int32_t rows, int32_t cols, float* x, int64_t ldx,
                     const float* gate, const float* scale, int64_t rows_per_mod,
                     int64_t mod_stride, float eps, b200_stream_t stream);

int b200_reduce_residual_adaln_gather(const void* slots, int32_t n_src, int32_t slot_rows,
                                      int32_t rows, int32_t cols, int64_t ld, float* x,
                                      int64_t ldx, const float* gate, const float* scale,
                                      int64_t rows_per_mod, int64_t mod_stride, float eps,
                                      void* const* dst_bufs, int32_t n_dst, int64_t dst_row0,
                                      int64_t dst_ld, b200_stream_t stream);

/*
 * The Q/K/V projections of one attention layer with the Q/K RMSNorm and RoPE in the
 * GEMM's epilogue: x [B * T, in_features] bf16 (row stride ldx) times w_qkv
 * [3 * H * 128, in_features] bf16 (to_q, to_k, to_v stacked) transposed, then
 *   q_rot, k_rot: head-major [B, H, T, 128] bf16, RMSNorm (norm_q_w / norm_k_w, eps) then
 *                 interleaved RoPE with pe rows pe + b * pe_batch_stride + t * 128 (f32)
 *   v:            token-major [B, T, H * 128] bf16
 * — the inputs of b200_joint_attention.  Replaces src/transformer.rs:173-185 (to_q / to_k
 * / to_v, reshape, norm_q / norm_k, transpose, apply_rope) for a cached step; the
 * unfused equivalent is three GEMMs and b200_qk_norm_rope.  H must be even.
 */
int b200_qkv_norm_rope_gemm(const void* x, int64_t ldx, const void* w_qkv, int32_t batch,
                            int32_t tokens, int32_t heads, int32_t in_features,
                            const float* norm_q_w, const float* norm_k_w, float eps,
                            const float* pe, int64_t pe_batch_stride, void* q_rot,
                            void* k_rot, void* v, int32_t* status, b200_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* B200_GEMM_H */
