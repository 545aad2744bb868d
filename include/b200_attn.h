/*
 * b200_attn.h — C ABI of the B200 (sm_100a) MMDiT joint-attention path.
 *
 * The library replaces, at both attention call sites of the Qwen-Image-2.1 engine,
 * the span from Q/K RMSNorm to the head merge:
 *   - src/transformer.rs:179-193            (Attention::forward, safetensors model)
 *   - src/quantized_transformer.rs:139-151  (Attention::forward, GGUF model)
 * i.e. norm_q/norm_k -> apply_rope -> cat(prefix K/V, step K/V) -> chunked_attention
 * -> transpose/reshape to [B, S, H*D].  The projections (to_q/to_k/to_v/to_out) stay
 * with the caller.
 *
 * Conventions (all entry points):
 *   - Every pointer named "device" is a CUDA device pointer owned by the caller; the
 *     library never frees or retains it.  Host pointers are read during the call only.
 *   - Work is enqueued on the caller's stream; nothing synchronises the device unless
 *     the function says so.
 *   - Functions return 0 (B200_OK) or a negative b200_status; they never abort.
 *   - Tensors are dense row-major, bf16 unless stated.  head_dim must be 128.
 *   - Entry points are reentrant, with one exception: b200_attn_fwd_noalloc, whose
 *     calls share one scratch array per device (see there).  Process state: per-device
 *     host caches (kernel attributes; the no-alloc array's device address), guarded by
 *     mutexes and keyed by the CUDA context, so they are rebuilt after cudaDeviceReset;
 *     and the no-alloc entry point's device array (B200_NOALLOC_SCRATCH_BYTES on every
 *     GPU that loads this library's kernels).
 */
#ifndef B200_ATTN_H
#define B200_ATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B200_ATTN_HEAD_DIM 128
#define B200_ATTN_ABI_VERSION 4

typedef enum {
  B200_OK = 0,
  B200_ERR_INVALID = -1,     /* null pointer, negative size, misaligned pointer      */
  B200_ERR_UNSUPPORTED = -2, /* head_dim != 128, device is not sm_100               */
  B200_ERR_CUDA = -3,        /* a CUDA runtime / driver call failed                  */
  B200_ERR_WORKSPACE = -4,   /* workspace missing or smaller than required          */
  B200_ERR_LAYOUT = -5,      /* layout / mask not representable (see key_valid)     */
  B200_ERR_DEVICE_TIMEOUT = -6 /* a device-side wait ran out (status word)          */
} b200_status;

/* Element types named by entry points that take more than one (b200_flash_attention_ex,
 * the head-sharding communicator of b200_tp.h). */
typedef enum { B200_DTYPE_BF16 = 0, B200_DTYPE_F32 = 1, B200_DTYPE_F16 = 2 } b200_dtype;

/* Opaque CUDA stream (cudaStream_t / CUstream); NULL = legacy default stream. */
typedef void* b200_stream_t;

/*
 * Per-batch-row key-length descriptor.  It replaces the reference's key_valid mask
 * ([B, 1, 1, P+T] bool, src/transformer.rs:642-649 and 736-745): keys
 * [0, prefix_valid) of the prefix cache and [0, target_valid) of this call's keys are
 * attended, the rest are masked.  b200_key_valid_to_desc() converts a key_valid mask.
 */
typedef struct {
  int32_t prefix_valid; /* 0 <= prefix_valid <= prefix_len */
  int32_t target_valid; /* 1 <= target_valid <= target_len */
} b200_kv_desc;

/*
 * Arguments of b200_attn_fwd (one attention layer of one cached denoising step).
 * Shapes: B = batch, T = target_len (this call's tokens), P = prefix_len, H = heads,
 * D = head_dim = 128.
 */
typedef struct {
  int32_t batch;       /* B >= 1                                                   */
  int32_t heads;       /* H >= 1                                                   */
  int32_t head_dim;    /* D, must be 128                                           */
  int32_t target_len;  /* T >= 0 (0 = nothing to do)                               */
  int32_t prefix_len;  /* P >= 0 (0 = no prefix cache, plain self-attention)       */
  const void* q;       /* device [B,T,H,D] bf16: raw to_q output (token-major)     */
  const void* k;       /* device [B,T,H,D] bf16: raw to_k output                   */
  const void* v;       /* device [B,T,H,D] bf16: raw to_v output                   */
  const void* prefix_k;/* device [B,H,P,D] bf16: cached post-RoPE keys (NULL if P=0) */
  const void* prefix_v;/* device [B,H,P,D] bf16: cached values         (NULL if P=0) */
  const float* norm_q_w; /* device [D] f32: RMSNorm weight of norm_q               */
  const float* norm_k_w; /* device [D] f32: RMSNorm weight of norm_k               */
  float norm_eps;      /* RMSNorm epsilon (1e-6 in the reference)                 */
  const float* pe;     /* device [T,D] f32: RoPE rows of this call's tokens,
                          interleaved (cos_i, sin_i) per pair i (EmbedNd::forward) */
  const b200_kv_desc* desc; /* device [B] or NULL (all keys valid)                 */
  float scale;         /* softmax scale, D^-0.5 in the reference                   */
  void* out;           /* device [B,T,H*D] bf16: attention output, ready for to_out */
  void* k_rot_out;     /* device [B,H,T,D] bf16 or NULL: this call's post-RoPE K
                          (the prefix-cache layout); required when NULL workspace
                          is too small to hold it, see b200_attn_workspace_bytes   */
  void* v_out;         /* device [B,H,T,D] bf16 or NULL: this call's V, cache layout */
  void* workspace;     /* device scratch, >= b200_attn_workspace_bytes() bytes     */
  size_t workspace_bytes;
  int32_t* status;     /* device int32 or NULL: set non-zero if a device-side wait
                          ran out (1 = load, 2 = mma, 3 = softmax, 4 = epilogue)   */
  const int32_t* row_limit; /* device [T] or NULL: query row q sees only this call's keys
                          [0, row_limit[q]) (non-decreasing in q).  The prefix-fill pass
                          passes b200_block_causal_limits() of its layout with
                          prefix_len = 0, which replaces build_block_causal_mask
                          (src/attention_mask.rs:18-66, src/transformer.rs:696-702)  */
  int64_t pe_batch_stride; /* floats between the pe rows of consecutive batch rows: 0 =
                          one [T,D] table for every row (the reference: one layout per
                          call, src/transformer.rs:729-734); T*D = a [B,T,D] table, for a
                          batch of prompts with different prefix lengths, whose target
                          tokens differ in the RoPE frame position.  Multiple of 4.    */
} b200_attn_args;

/*
 * Bytes of the region that lets the attention kernel split its last partial wave of
 * work across the idle SMs (partial results of up to 160 pieces + arrival counters).
 */
#define B200_ATTN_SPLIT_WORKSPACE_BYTES 21299968u

/* Scratch bytes b200_attn_fwd wants for these args: post-RoPE Q, K unless k_rot_out is
 * given, and B200_ATTN_SPLIT_WORKSPACE_BYTES for the tail split.  A workspace without
 * the split region (B200_ATTN_SPLIT_WORKSPACE_BYTES less) is accepted and runs without
 * the split.  Replaces nothing in the reference (candle allocates). */
int b200_attn_workspace_bytes(const b200_attn_args* args, size_t* bytes);

/*
 * One joint-attention layer: Q/K RMSNorm + RoPE, attention of the T queries over
 * [prefix K/V (desc.prefix_valid keys) ; this call's K/V (desc.target_valid keys)],
 * output in [B,T,H*D].  Replaces src/transformer.rs:179-193 and
 * src/quantized_transformer.rs:139-151 (norm -> apply_rope -> Tensor::cat ->
 * chunked_attention -> transpose/reshape).  Two kernels on `stream`; no host sync.
 */
int b200_attn_fwd(const b200_attn_args* args, b200_stream_t stream);

/*
 * b200_attn_fwd without a workspace, for callers that cannot allocate device memory
 * when they call (a frozen or foreign allocator, a plugin host that only hands over
 * the input and output tensors).  No counterpart in the reference: it has no such
 * constraint, candle allocates on every call.
 *
 * The scratch (post-RoPE Q, and K when k_rot_out is NULL) lives in a fixed device array
 * of B200_NOALLOC_SCRATCH_BYTES inside the library, held by every GPU that loads it
 * until exit; args->workspace and args->workspace_bytes are ignored.  Problems whose
 * required scratch (b200_attn_workspace_bytes() less B200_ATTN_SPLIT_WORKSPACE_BYTES)
 * exceeds the limit return B200_ERR_WORKSPACE (e.g. with B = 1, H = 32: up to T = 4096
 * tokens with k_rot_out NULL, 8192 with it given); the tail split is used when its
 * region also fits.
 * The first call on a device (and the first after the device's context changed, e.g.
 * after cudaDeviceReset) looks up the array's device address (no allocation); make that
 * first call before any stream capture.  The array's memory itself is committed when
 * the CUDA module holding the library's kernels is loaded on the device: with lazy
 * module loading (the CUDA 12 default) that is the first launch or symbol lookup of any
 * of this library's attention entry points, so a caller that freezes its allocator
 * should make one such call during warm-up, before the freeze.  All calls on a device
 * share the one array: calls that may overlap on the GPU (other streams, other
 * threads) race on it, so serialise them.  Nothing in it needs clearing between calls.
 */
#define B200_NOALLOC_SCRATCH_BYTES (64u << 20)
int b200_attn_fwd_noalloc(const b200_attn_args* args, b200_stream_t stream);

/*
 * The attention part of b200_attn_fwd, for callers that already hold post-norm,
 * post-RoPE Q and K: q_rot device [B,H,T,D], k_rot device [B,H,T,D] (head-major, the
 * cache layout), v device [B,T,H,D] (token-major projection output), prefix_k/prefix_v
 * device [B,H,P,D] (NULL if P = 0), desc device [B] or NULL; out device [B,T,H*D].
 * workspace: device, >= B200_ATTN_SPLIT_WORKSPACE_BYTES to enable the tail split, or
 * NULL.  Replaces Tensor::cat + chunked_attention + transpose/reshape
 * (src/transformer.rs:186-193, src/quantized_transformer.rs:145-151).  One kernel (plus
 * a small memset of arrival counters when the tail is split).
 */
int b200_joint_attention(const void* q_rot, const void* k_rot, const void* v,
                         const void* prefix_k, const void* prefix_v, int32_t batch,
                         int32_t heads, int32_t target_len, int32_t prefix_len,
                         int32_t head_dim, const b200_kv_desc* desc, float scale, void* out,
                         void* workspace, size_t workspace_bytes, int32_t* status,
                         b200_stream_t stream);

/*
 * The FA2 branch's contract on [B,S,H,D] tensors: out = softmax(q k^T * scale [masked]) v
 * with token-major q [B,Sq,H,D], k, v [B,Skv,H,D] and out [B,Sq,H,D], no transposes.
 * Replaces flash_attention / candle_flash_attn::flash_attn(q, k, v, scale, causal = false)
 * (src/transformer.rs:243-254), whose tensors have this layout.  key_len (device int32 [B]
 * or NULL): batch row b attends to keys [0, key_len[b]).  One kernel on `stream`; no
 * workspace, no host sync.
 *
 * b200_flash_attention takes bf16 tensors.  b200_flash_attention_ex takes the element
 * type: B200_DTYPE_BF16, or B200_DTYPE_F16 for IEEE half q/k/v/out, the type the
 * reference's FA2 branch casts its inputs to (src/transformer.rs:244-251).  Any other
 * dtype returns B200_ERR_UNSUPPORTED before launching.  Both compute in f32 (scores,
 * softmax, accumulation) with P rounded to the input type for the P.V product.
 */
int b200_flash_attention(const void* q, const void* k, const void* v, void* out,
                         int32_t batch, int32_t sq, int32_t skv, int32_t heads,
                         int32_t head_dim, float scale, const int32_t* key_len,
                         int32_t* status, b200_stream_t stream);
int b200_flash_attention_ex(const void* q, const void* k, const void* v, void* out,
                            int32_t batch, int32_t sq, int32_t skv, int32_t heads,
                            int32_t head_dim, float scale, const int32_t* key_len,
                            int32_t dtype, int32_t* status, b200_stream_t stream);

/*
 * Plain attention on [B,H,S,D] tensors: out = softmax(q k^T * scale [masked]) v.
 * Replaces chunked_attention(q, k, v, scale, mask) (src/transformer.rs:259-296) and
 * its flash_attention branch (src/transformer.rs:243-254) for a mask of the form
 * key_valid [B,1,1,Skv] expressed as key_len[b] valid leading keys.
 *   q   device [B,H,Sq,D] bf16;  k, v device [B,H,Skv,D] bf16;  out device [B,H,Sq,D] bf16
 *   key_len device int32 [B] (1 <= key_len[b] <= Skv) or NULL (all Skv keys valid).
 */
int b200_chunked_attention(const void* q, const void* k, const void* v, void* out,
                           int32_t batch, int32_t heads, int32_t sq, int32_t skv,
                           int32_t head_dim, float scale, const int32_t* key_len,
                           int32_t* status, b200_stream_t stream);

/*
 * Q/K RMSNorm + RoPE alone (the prologue of b200_attn_fwd).  x device [B,T,H,D] bf16
 * (token-major projection output) -> y device [B,H,T,D] bf16 (head-major).  Replaces
 * `x.reshape(..).apply(&norm).transpose(1,2)` + apply_rope (src/transformer.rs:179-185,
 * src/rope.rs:222-228).  norm_w may be NULL to skip the norm (RoPE only); pe may be
 * NULL to skip RoPE.
 */
int b200_norm_rope(const void* x, void* y, int32_t batch, int32_t tokens, int32_t heads,
                   int32_t head_dim, const float* norm_w, float eps, const float* pe,
                   b200_stream_t stream);

/*
 * The prologue b200_attn_fwd launches: RMSNorm + RoPE of Q and K in one kernel.
 * q, k device [B,T,H,D] bf16 -> q_rot, k_rot device [B,H,T,D] bf16; norm weights device
 * [D] f32; pe device [T,D] f32.  With b200_joint_attention it splits b200_attn_fwd into
 * its two launches (src/transformer.rs:179-185).
 */
int b200_qk_norm_rope(const void* q, const void* k, void* q_rot, void* k_rot, int32_t batch,
                      int32_t tokens, int32_t heads, int32_t head_dim, const float* norm_q_w,
                      const float* norm_k_w, float eps, const float* pe, b200_stream_t stream);

/* ---- host-side mirrors of the reference's layout / RoPE / mask code (no device) ---- */

/*
 * JointLayout::new (src/joint_layout.rs:52-103).  Host arrays.
 *   text_image_mask [text_len] (0/1) or NULL; cond_shapes [n_cond][2] (h, w);
 *   target_h, target_w: latent grid of the generated image.
 * Outputs (capacity `cap` tokens, caller-allocated): image_ids [len] (-1 text, else
 * image block index), image_pad_mask [len]; img_shapes [(n_cond+1)][3] (frame,h,w);
 * *len_out, *prefix_len_out, *target_len_out.
 * Errors mirror the reference's bail! cases (B200_ERR_LAYOUT).
 */
int b200_joint_layout(int32_t text_len, const uint8_t* text_image_mask,
                      const int32_t* cond_shapes, int32_t n_cond, int32_t target_h,
                      int32_t target_w, int32_t cap, int64_t* image_ids,
                      uint8_t* image_pad_mask, int32_t* img_shapes, int32_t* len_out,
                      int32_t* prefix_len_out, int32_t* target_len_out);

/*
 * EmbedNd::forward position rules (src/rope.rs:118-172): per token (frame, h, w)
 * positions.  img_shapes [n_shapes][3] host, image_pad_mask [seq_len] host;
 * pos_out [seq_len][3] host int64.
 */
int b200_rope_positions(const int32_t* img_shapes, int32_t n_shapes,
                        const uint8_t* image_pad_mask, int32_t seq_len, int64_t* pos_out);

/*
 * EmbedNd::new + forward (src/rope.rs:37-211): RoPE rows pe_out [seq_len][sum(axes)]
 * host f32, interleaved (cos, sin) per pair, axes e.g. {16, 56, 56}, theta 1e4.
 * Positions outside the reference's table range [-1024, 8191] are B200_ERR_LAYOUT.
 */
int b200_rope_pe(const int32_t* img_shapes, int32_t n_shapes,
                 const uint8_t* image_pad_mask, int32_t seq_len, const int32_t axes[3],
                 float theta, float* pe_out);

/*
 * key_valid -> descriptors.  key_valid host [B][prefix_len + target_len] (0/1) as the
 * reference builds it (src/transformer.rs:736-745).  Padding must be a suffix of the
 * prefix and the target must be fully valid; otherwise B200_ERR_LAYOUT.
 * desc_out host [B].
 */
int b200_key_valid_to_desc(const uint8_t* key_valid, int32_t batch, int32_t prefix_len,
                           int32_t target_len, b200_kv_desc* desc_out);

/*
 * Block-causal mask as per-row key limits (src/attention_mask.rs:18-66): a text token
 * (image_ids[i] < 0) sees keys [0, i+1); a token of image block k sees keys [0, e) where
 * e is one past the block's last token (causal OR same image block).  image_ids host
 * [len] (JointLayout.image_ids, text -1, blocks contiguous); limits_out host [len].
 * Combine with b200_kv_desc.target_valid for the padded-key part of the mask.
 */
int b200_block_causal_limits(const int64_t* image_ids, int32_t len, int32_t* limits_out);

/* Human-readable text of a b200_status; b200_attn_strerror is the same function under
 * the name the engine's binding plan uses. */
const char* b200_strerror(int status);
const char* b200_attn_strerror(int status);

/* ABI version (B200_ATTN_ABI_VERSION). */
int b200_abi_version(void);

/*
 * Self-test of the device-side failure path (no counterpart in the reference): one small
 * kernel waits on a barrier that nothing completes, with the same bounded wait and CTA
 * abort flag as the attention kernel.  After the wait gives up (limit_us, at most 2 s),
 * status[0] = 1 (the wait ran out) and status[1] = 1 (a second waiter left on the abort
 * flag); status (device int32[2]) must be zero before the call.  The context stays usable.
 */
int b200_wait_selftest(int32_t* status, uint32_t limit_us, b200_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* B200_ATTN_H */
