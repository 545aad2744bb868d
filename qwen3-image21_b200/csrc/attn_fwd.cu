// attn_fwd.cu — B200 (sm_100a) joint-attention path of the Qwen-Image-2.1 MMDiT blocks.
//
// Two kernels per attention layer:
//   norm_rope_kernel   per-head RMSNorm (eps 1e-6) + interleaved RoPE of Q and K,
//                      token-major [B,T,H,D] -> head-major [B,H,T,D] bf16 (the K output is
//                      the prefix-cache layout).  Reference: src/transformer.rs:179-185,
//                      src/rope.rs:222-228.
//   joint_attn_kernel  online-softmax attention of 256 query rows (two 128-row tiles) of
//                      one (batch, head) over [prefix keys ; step keys].  K/V tiles of 128
//                      keys arrive by TMA (128-byte swizzle, no multicast) into a 2-stage
//                      ring; S = Q K^T and O += P V run on tcgen05.mma (bf16 -> f32) with
//                      S, P and O in tensor memory; two softmax warpgroups ping-pong so the
//                      tensor core works on one Q tile while the other is in softmax.
//                      Masking comes from per-batch key lengths (and, for the prefix
//                      fill, per-row limits); the last partial wave of work items can be
//                      cut by key range (tail split) and merged by the last piece.  Q, K
//                      and V are read through 4-D tensor maps either head-major or
//                      token-major.  The output tile is staged in the Q slot of shared
//                      memory and written by TMA stores.  Reference: chunked_attention,
//                      src/transformer.rs:259-296; flash_attention, 243-254.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <mutex>

#include "../../include/b200_attn.h"
#include "ptx.cuh"

namespace b200 {

constexpr int kD = 128;        // head_dim
constexpr int kBM = 128;       // query rows per tile
constexpr int kBN = 128;       // keys per K/V tile
constexpr int kQTiles = 2;     // query tiles per CTA
constexpr int kStages = 2;     // K and V ring depth
constexpr int kTileBytes = kBM * kD * 2;       // 32 KiB: 128 x 128 bf16
constexpr int kRegionBytes = 128 * 64 * 2;     // 16 KiB: 128 rows x 64 cols (one swizzle span)
constexpr int kThreads = 384;  // warp 0 TMA, warp 1 MMA, warp 2 TMEM alloc, 4-7 / 8-11 softmax
constexpr int kSmemQ = 0;
constexpr int kSmemK = kSmemQ + kQTiles * kTileBytes;
constexpr int kSmemV = kSmemK + kStages * kTileBytes;
constexpr int kSmemBar = kSmemV + kStages * kTileBytes;
constexpr int kSmemBytes = kSmemBar + 256 + 1024;  // barriers + 1 KiB alignment slack
constexpr uint32_t kTmemCols = 512;  // S0 | S1 | O0 | O1, 128 columns each
constexpr float kRescaleThreshold = 8.0f;  // log2 units: O is rescaled when the max grows >2^8

struct AttnParams {
  int32_t T;                 // query rows
  int32_t P;                 // rows of segment 0 (prefix cache), 0 = none
  int32_t L1;                // rows of segment 1 (this call's keys)
  int32_t v1_token_major;    // segment-1 V map is [B,T,H,D] (coords d, h, row, b)
  int32_t k1_token_major;    // segment-1 K map is [B,T,H,D] (coords d, h, row, b)
  int32_t q_token_major;     // Q map is [B,T,H,D] (coords d, h, row, b)
  int32_t o_token_major;     // output map is [B,T,H,D] (coords d, h, row, b)
  const int32_t* seg0_len;   // valid keys of segment 0 per batch row (stride seg0_stride)
  const int32_t* seg1_len;
  int32_t seg0_stride, seg1_stride;
  // Optional per-query-row limit on segment-1 keys (keys [0, row_limit[q]) are visible),
  // shared by all batch rows and non-decreasing in q: the block-causal mask of the
  // prefix-fill pass.  NULL: every valid key is visible.
  const int32_t* row_limit;
  float scale_log2;          // scale * log2(e)
  uint16_t* out;             // 16-bit elements (bf16, or f16 in the kF16 kernel)
  int64_t out_sb, out_sh, out_sr;  // element strides: batch, head, query row
  int32_t* status;
  // Work units.  An item is one (batch, head, 256-row query block); items are numbered
  // with the query block fastest.  Units [0, n_full) are whole items; each of the last
  // (grid - n_full) / split items is cut into `split` contiguous ranges of key tiles,
  // one unit each, so the last partial wave of CTAs is spread over more SMs.
  int32_t H;
  int32_t nqb;        // query blocks per (batch, head)
  int32_t n_full;
  int32_t split;      // 1 = no split units
  float* part_o;      // [split item][piece][256][128] unnormalised O of each piece
  float* part_ml;     // [split item][piece][2][256] running max m and sum l per row
  int32_t* part_cnt;  // [split item] pieces finished; zero before the launch
};

__device__ __forceinline__ void record_error(const AttnParams& p, volatile int* abort_flag,
                                             int code) {
  *abort_flag = 1;
  if (p.status) atomicCAS(p.status, 0, code);
}

// Bounded wait that also gives up as soon as another role of the CTA has aborted.
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity,
                                              volatile int* abort_flag) {
  return mbar_wait(bar, parity, abort_flag);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Two values rounded to the kernel's 16-bit type (kF16: IEEE half, else bf16), packed.
template <bool kF16>
__device__ __forceinline__ uint32_t pack16x2(float lo, float hi) {
  return kF16 ? pack_f16x2(lo, hi) : pack_bf16x2(lo, hi);
}

// Quiet NaN of the kernel's 16-bit type, twice.
template <bool kF16>
constexpr uint32_t kNaN16x2 = kF16 ? 0x7e007e00u : 0x7fc07fc0u;

__device__ __forceinline__ void named_barrier_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// ---- packed f32x2 arithmetic (sm_100 FFMA2 / FADD2: two lanes per instruction)
__device__ __forceinline__ uint64_t f2pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2unpack(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t f2fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 2^x0, 2^x1 on the FMA pipe instead of the MUFU: x = j + f with j = rint(x) (taken from
// the low mantissa bits of x + 1.5*2^23) and f in [-1/2, 1/2]; 2^f by a degree-4
// polynomial with relative error < 3e-6 (coefficients from csrc/exp2_poly_fit.py); 2^j
// applied by adding j to the exponent field.  x is clamped at -126.5 so j >= -126 (the
// result is then at most ~1e-38 instead of 0, far below any row sum, which is >= 1).
constexpr float kExpC1 = 6.931241751e-01f;
constexpr float kExpC2 = 2.402409911e-01f;
constexpr float kExpC3 = 5.590642616e-02f;
constexpr float kExpC4 = 9.582848288e-03f;
__device__ __forceinline__ void exp2_fma2(float x0, float x1, float& y0, float& y1) {
  constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
  const uint64_t x = f2pack(fmaxf(x0, -126.5f), fmaxf(x1, -126.5f));
  const uint64_t t = f2add(x, f2pack(kMagic, kMagic));
  const uint64_t j = f2add(t, f2pack(-kMagic, -kMagic));
  const uint64_t f = f2fma(j, f2pack(-1.f, -1.f), x);
  uint64_t a = f2fma(f2pack(kExpC4, kExpC4), f, f2pack(kExpC3, kExpC3));
  a = f2fma(a, f, f2pack(kExpC2, kExpC2));
  a = f2fma(a, f, f2pack(kExpC1, kExpC1));
  a = f2fma(a, f, f2pack(1.f, 1.f));
  float a0, a1, t0, t1;
  f2unpack(a, a0, a1);
  f2unpack(t, t0, t1);
  y0 = __int_as_float(__float_as_int(a0) + (__float_as_int(t0) << 23));
  y1 = __int_as_float(__float_as_int(a1) + (__float_as_int(t1) << 23));
}

// One in kPolyEvery exp2 pairs of a full (unmasked) tile runs on the FMA pipe, the rest on
// the MUFU: at D = 128 the MUFU alone needs as many cycles per tile as the tensor core.
constexpr int kPolyEvery = 4;

// Softmax of this thread's 128-key S row (TMEM columns [tS, tS + 128), one row per
// thread): keys >= valid are masked (kMasked); the running max m (log2 units) is raised
// only when the row max exceeds it by more than kRescaleThreshold (lazy rescaling, as in
// FlashAttention-4), so P = 2^(S*c - m) <= 2^8.  P goes to TMEM columns [tS, tS + 64) as
// bf16 pairs, over S columns already read; the f32 p values stay in r for the row sum,
// which the caller takes after handing P to the MMA warp (off the S -> P critical path).
// Returns the factor the O accumulator must be scaled by (1 when m did not move).  A row
// without any valid key so far keeps m = -inf and P = 0.
template <bool kMasked, bool kF16>
__device__ __forceinline__ float softmax_row(uint32_t (&r)[4][32], const int valid,
                                             const float c, float& m, const uint32_t tS) {
#pragma unroll
  for (int q = 0; q < 4; ++q) tmem_ld32(tS + q * 32, r[q]);
  tmem_wait_ld();
  auto v = [&](int col) { return __uint_as_float(r[col >> 5][col & 31]); };
  if (kMasked) {
#pragma unroll
    for (int q = 0; q < 4; ++q)
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (q * 32 + i >= valid) r[q][i] = __float_as_uint(-INFINITY);
  }
  float pm[8];
#pragma unroll
  for (int g = 0; g < 8; ++g) pm[g] = fmaxf(v(g * 16), v(g * 16 + 1));
#pragma unroll
  for (int i = 1; i < 8; ++i)
#pragma unroll
    for (int g = 0; g < 8; ++g) pm[g] = fmax3(pm[g], v(g * 16 + 2 * i), v(g * 16 + 2 * i + 1));
  const float mx =
      fmax3(fmax3(pm[0], pm[1], pm[2]), fmax3(pm[3], pm[4], pm[5]), fmaxf(pm[6], pm[7])) * c;
  float alpha = 1.f;
  if (mx > m + kRescaleThreshold) {
    alpha = ex2_approx(m - mx);  // 0 on the first tile (m = -inf)
    m = mx;
  }
  const uint64_t cc = f2pack(c, c);
  // A row that has not seen a valid key keeps m = -inf; its masked S (-inf) must give
  // P = 2^-inf = 0, not 2^(-inf + inf) = NaN (a tail-split piece can hold such rows).
  const float m_ref = m == -INFINITY ? 0.f : m;
  const uint64_t nm = f2pack(-m_ref, -m_ref);
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    uint32_t pk[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int col = half * 64 + 2 * i;
      float x0, x1, p0, p1;
      f2unpack(f2fma(f2pack(v(col), v(col + 1)), cc, nm), x0, x1);
      if (!kMasked && (i % kPolyEvery) == kPolyEvery - 1) {
        exp2_fma2(x0, x1, p0, p1);
      } else {
        p0 = ex2_approx(x0);
        p1 = ex2_approx(x1);
      }
      r[col >> 5][col & 31] = __float_as_uint(p0);
      r[(col + 1) >> 5][(col + 1) & 31] = __float_as_uint(p1);
      pk[i] = pack16x2<kF16>(p0, p1);
    }
    tmem_st32(tS + half * 32, pk);
  }
  return alpha;
}

// Sum of the 128 f32 p values softmax_row left in r (4 independent f32x2 chains).
__device__ __forceinline__ float row_sum(const uint32_t (&r)[4][32]) {
  uint64_t acc[4] = {f2pack(0.f, 0.f), f2pack(0.f, 0.f), f2pack(0.f, 0.f), f2pack(0.f, 0.f)};
#pragma unroll
  for (int i = 0; i < 64; ++i)
    acc[i & 3] = f2add(acc[i & 3], f2pack(__uint_as_float(r[(2 * i) >> 5][(2 * i) & 31]),
                                          __uint_as_float(r[(2 * i + 1) >> 5][(2 * i + 1) & 31])));
  float s[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) f2unpack(acc[i], s[2 * i], s[2 * i + 1]);
  return ((s[0] + s[1]) + (s[2] + s[3])) + ((s[4] + s[5]) + (s[6] + s[7]));
}

// kF16: Q, K, V, P and the output are IEEE half (the reference's FA2 branch casts to
// f16); otherwise bf16.  Accumulation is f32 either way.
template <bool kF16>
__global__ void __launch_bounds__(kThreads, 1)
    joint_attn_kernel(const __grid_constant__ CUtensorMap tm_q,
                      const __grid_constant__ CUtensorMap tm_k0,
                      const __grid_constant__ CUtensorMap tm_v0,
                      const __grid_constant__ CUtensorMap tm_k1,
                      const __grid_constant__ CUtensorMap tm_v1,
                      const __grid_constant__ CUtensorMap tm_o, const AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem + kSmemQ;
  uint8_t* sK = smem + kSmemK;
  uint8_t* sV = smem + kSmemV;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kSmemBar);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;   // [kStages]
  uint64_t* k_empty = bars + 3;  // [kStages]
  uint64_t* v_full = bars + 5;   // [kStages]
  uint64_t* v_empty = bars + 7;  // [kStages]
  uint64_t* s_full = bars + 9;   // [kQTiles]
  uint64_t* p_full = bars + 11;  // [kQTiles]
  uint64_t* o_full = bars + 13;  // [kQTiles]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 17);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int unit = blockIdx.x;
  int item = unit, piece = 0;
  const bool split_unit = unit >= p.n_full;
  if (split_unit) {
    item = p.n_full + (unit - p.n_full) / p.split;
    piece = (unit - p.n_full) % p.split;
  }
  const int h = (item / p.nqb) % p.H;
  const int b = item / (p.nqb * p.H);
  const int q0 = (item % p.nqb) * (kQTiles * kBM);

  // Key tiles: segment 0 (prefix) then segment 1; each segment's last tile may be ragged.
  int pv = 0;
  if (p.P > 0) pv = p.seg0_len ? min(max(p.seg0_len[(int64_t)b * p.seg0_stride], 0), p.P) : p.P;
  const int tv = p.seg1_len ? min(max(p.seg1_len[(int64_t)b * p.seg1_stride], 0), p.L1) : p.L1;
  // With row limits, this block's rows see at most row_limit[last row] keys (the limits
  // are non-decreasing), so later key tiles are skipped.
  const int tv_blk =
      p.row_limit ? min(tv, max(p.row_limit[min(q0 + kQTiles * kBM, p.T) - 1], 0)) : tv;
  const int n0 = (pv + kBN - 1) / kBN;
  const int n1 = (tv_blk + kBN - 1) / kBN;
  // This unit's key tiles [jb, jb + n) of the n0 + n1 tiles of the item.
  int jb = 0, n = n0 + n1;
  if (split_unit) {
    const int all = n;
    jb = static_cast<int>(static_cast<int64_t>(all) * piece / p.split);
    n = static_cast<int>(static_cast<int64_t>(all) * (piece + 1) / p.split) - jb;
  }

  // Producer (thread 0) helpers: Q, and key tile j of this unit into ring stage j % kStages
  // (K, then V), completion counted on q_full / k_full / v_full.
  auto load_q = [&]() {
    mbar_expect_tx(q_full, kQTiles * kTileBytes);
    for (int t = 0; t < kQTiles; ++t)
      for (int c = 0; c < 2; ++c) {
        uint8_t* dst = sQ + t * kTileBytes + c * kRegionBytes;
        if (p.q_token_major)
          tma_load_4d(dst, &tm_q, q_full, c * 64, h, q0 + t * kBM, b);
        else
          tma_load_4d(dst, &tm_q, q_full, c * 64, q0 + t * kBM, h, b);
      }
  };
  auto load_k = [&](int j) {
    const int s = j & 1;
    const int ja = jb + j;  // tile index within the item
    const bool seg0 = ja < n0;
    const int row = (seg0 ? ja : ja - n0) * kBN;
    mbar_expect_tx(k_full + s, kTileBytes);
    for (int c = 0; c < 2; ++c) {
      uint8_t* dst = sK + s * kTileBytes + c * kRegionBytes;
      if (!seg0 && p.k1_token_major)
        tma_load_4d(dst, &tm_k1, k_full + s, c * 64, h, row, b);
      else
        tma_load_4d(dst, seg0 ? &tm_k0 : &tm_k1, k_full + s, c * 64, row, h, b);
    }
  };
  auto load_v = [&](int j) {
    const int s = j & 1;
    const int ja = jb + j;
    const bool seg0 = ja < n0;
    const int row = (seg0 ? ja : ja - n0) * kBN;
    mbar_expect_tx(v_full + s, kTileBytes);
    for (int c = 0; c < 2; ++c) {
      uint8_t* dst = sV + s * kTileBytes + c * kRegionBytes;
      if (seg0)
        tma_load_4d(dst, &tm_v0, v_full + s, c * 64, row, h, b);
      else if (p.v1_token_major)
        tma_load_4d(dst, &tm_v1, v_full + s, c * 64, h, row, b);
      else
        tma_load_4d(dst, &tm_v1, v_full + s, c * 64, row, h, b);
    }
  };
  if (threadIdx.x == 0) {
    if (n > 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k1);
      tma_prefetch_desc(&tm_v1);
      if (n0 > 0) {
        tma_prefetch_desc(&tm_k0);
        tma_prefetch_desc(&tm_v0);
      }
    }
    mbar_init(q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(k_full + s, 1);
      mbar_init(k_empty + s, 1);
      mbar_init(v_full + s, 1);
      mbar_init(v_empty + s, 1);
    }
    for (int t = 0; t < kQTiles; ++t) {
      mbar_init(s_full + t, 1);
      mbar_init(p_full + t, kBM);
      mbar_init(o_full + t, 1);
    }
    *abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async();
    // Q and the first kStages key tiles go out now: their latency overlaps the TMEM
    // allocation and the CTA barrier below.
    if (n > 0) {
      load_q();
      for (int j = 0; j < n && j < kStages; ++j) {
        load_k(j);
        load_v(j);
      }
    }
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp < 4) {
  // Register split: warpgroup 0 (load, MMA, allocator) gives registers to the two softmax
  // warpgroups; 128 x 56 + 256 x 224 = 384 x 168, the launch allocation.  Each
  // setmaxnreg dominates the code of its role.
  asm volatile("setmaxnreg.dec.sync.aligned.u32 56;" ::: "memory");
  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0 && n > 0) {
      // Q and key tiles [0, kStages) were issued before the CTA barrier.
      bool ok = true;
      for (int j = kStages; j < n && ok; ++j) {
        const int s = j & 1;
        const uint32_t u = static_cast<uint32_t>(j >> 1);
        if (!wait_or_abort(k_empty + s, (u - 1) & 1, abort_flag)) {
          ok = false;
          break;
        }
        load_k(j);
        if (!wait_or_abort(v_empty + s, (u - 1) & 1, abort_flag)) {
          ok = false;
          break;
        }
        load_v(j);
      }
      if (!ok) {
        record_error(p, abort_flag, 1);
        // Let copies already issued land before the CTA's shared memory is released.
        for (int s = 0; s < kStages; ++s) {
          mbar_wait(k_full + s, 0);
          mbar_wait(v_full + s, 0);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    // The whole warp runs the loop (every lane waits; the lanes agree through __all_sync),
    // and one elected lane issues each tcgen05.mma / commit (always the same lane, so its
    // commits track its own MMAs).
    if (n > 0) {
      constexpr uint32_t idesc_qk = idesc_16_f32(kF16, kBM, kBN, 0, 0);
      constexpr uint32_t idesc_pv = idesc_16_f32(kF16, kBM, kD, 0, 1);
      // Descriptors as (low, high) words: a k-step only moves the start address (low 14
      // bits, 16-byte units, < 2^14 inside the 256 KiB shared window), so the offset is
      // added to the low word and never carries into the other fields.
      const uint64_t dQ = smem_desc(smem_addr(sQ), 16, 1024);
      const uint64_t dK = smem_desc(smem_addr(sK), 16, 1024);
      const uint64_t dV = smem_desc(smem_addr(sV), kRegionBytes, 1024);
      const uint32_t hi_qk = static_cast<uint32_t>(dQ >> 32);
      const uint32_t hi_v = static_cast<uint32_t>(dV >> 32);
      const uint32_t lo_q = static_cast<uint32_t>(dQ), lo_k = static_cast<uint32_t>(dK);
      const uint32_t lo_v = static_cast<uint32_t>(dV);
      auto wait = [&](uint64_t* bar, uint32_t parity) {
        return __all_sync(0xffffffffu, wait_or_abort(bar, parity, abort_flag));
      };
      auto commit = [&](uint64_t* bar) {
        if (elect_one()) mma_commit(bar);
      };
      auto qk = [&](int t, int s) {
        const uint32_t d = tmem_base + t * kBN;
        const uint32_t a = lo_q + ((t * kTileBytes) >> 4);
        const uint32_t bk = lo_k + ((s * kTileBytes) >> 4);
        // k-step kk: region kk/4 (16 KiB apart), 32 bytes per step inside the swizzle span
        if (elect_one()) {
          mma_ss_off<0, 0>(d, a, hi_qk, bk, hi_qk, idesc_qk, 0u);
          mma_ss_off<2, 2>(d, a, hi_qk, bk, hi_qk, idesc_qk, 1u);
          mma_ss_off<4, 4>(d, a, hi_qk, bk, hi_qk, idesc_qk, 1u);
          mma_ss_off<6, 6>(d, a, hi_qk, bk, hi_qk, idesc_qk, 1u);
          mma_ss_off<1024, 1024>(d, a, hi_qk, bk, hi_qk, idesc_qk, 1u);
          mma_ss_off<1026, 1026>(d, a, hi_qk, bk, hi_qk, idesc_qk, 1u);
          mma_ss_off<1028, 1028>(d, a, hi_qk, bk, hi_qk, idesc_qk, 1u);
          mma_ss_off<1030, 1030>(d, a, hi_qk, bk, hi_qk, idesc_qk, 1u);
        }
        __syncwarp();
      };
      auto pv_mma = [&](int t, int s, bool acc) {
        const uint32_t d = tmem_base + 2 * kBN + t * kD;
        const uint32_t a = tmem_base + t * kBN;  // P (bf16 pairs) over S's first 64 columns
        const uint32_t bv = lo_v + ((s * kTileBytes) >> 4);
        // k-step kk: 16 keys = 2 KiB of V rows; P columns kk*8 .. kk*8+7
        if (elect_one()) {
          mma_ts_off<0>(d, a, bv, hi_v, idesc_pv, acc ? 1u : 0u);
          mma_ts_off<128>(d, a + 8, bv, hi_v, idesc_pv, 1u);
          mma_ts_off<256>(d, a + 16, bv, hi_v, idesc_pv, 1u);
          mma_ts_off<384>(d, a + 24, bv, hi_v, idesc_pv, 1u);
          mma_ts_off<512>(d, a + 32, bv, hi_v, idesc_pv, 1u);
          mma_ts_off<640>(d, a + 40, bv, hi_v, idesc_pv, 1u);
          mma_ts_off<768>(d, a + 48, bv, hi_v, idesc_pv, 1u);
          mma_ts_off<896>(d, a + 56, bv, hi_v, idesc_pv, 1u);
        }
        __syncwarp();
      };
      bool ok = wait(q_full, 0) && wait(k_full, 0);
      if (ok) {
        tc_fence_after();
        qk(0, 0);
        commit(s_full + 0);
        qk(1, 0);
        commit(s_full + 1);
        commit(k_empty + 0);
      }
      for (int j = 0; j < n && ok; ++j) {
        const int s = j & 1;
        const uint32_t u = static_cast<uint32_t>(j >> 1);
        const int s1 = (j + 1) & 1;
        const uint32_t u1 = static_cast<uint32_t>((j + 1) >> 1);
        const bool more = j + 1 < n;
        if (!wait(v_full + s, u & 1) || !wait(p_full + 0, j & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        pv_mma(0, s, j > 0);
        if (!more) commit(o_full + 0);
        if (more) {
          if (!wait(k_full + s1, u1 & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          qk(0, s1);
          commit(s_full + 0);
        }
        if (!wait(p_full + 1, j & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        pv_mma(1, s, j > 0);
        commit(v_empty + s);
        if (!more) commit(o_full + 1);
        if (more) {
          qk(1, s1);
          commit(s_full + 1);
          commit(k_empty + s1);
        }
      }
      if (!ok && lane == 0) record_error(p, abort_flag, 2);
    }
  }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 224;" ::: "memory");
    // ---------------------------------------------------------------- softmax / epilogue
    const int t = (warp - 4) >> 2;
    const int wq = warp & 3;
    const int row = wq * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    const uint32_t tS = tmem_base + lane_off + t * kBN;
    const uint32_t tO = tmem_base + lane_off + 2 * kBN + t * kD;
    const float c = p.scale_log2;
    float m = -INFINITY;  // running max, scaled (log2) units
    float l = 0.f;        // running sum of p
    bool ok = true;
    // This row's visible segment-1 keys (row limit, then the batch row's valid length).
    const int qrow_lim = q0 + t * kBM + row;
    const int tv_row =
        p.row_limit ? min(tv, max(p.row_limit[min(qrow_lim, p.T - 1)], 0)) : tv;
    for (int j = 0; j < n; ++j) {
      if (!wait_or_abort(s_full + t, j & 1, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int ja = jb + j;
      const int valid = ja < n0 ? min(kBN, pv - ja * kBN) : min(kBN, tv_row - (ja - n0) * kBN);
      // Rows of a warp may have different limits: any masked lane sends the whole warp down
      // the masked path (TMEM loads are warp-collective).
      uint32_t r[4][32];
      const float alpha = __any_sync(0xffffffffu, valid < kBN)
                              ? softmax_row<true, kF16>(r, valid, c, m, tS)
                              : softmax_row<false, kF16>(r, valid, c, m, tS);
      // O rescale: PV of the previous tile is complete (s_full is committed after it).
      if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint32_t o[32];
          tmem_ld32(tO + q * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st32(tO + q * 32, o);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(p_full + t);
      l = l * alpha + row_sum(r);
    }
    if (!ok) record_error(p, abort_flag, 3);
    // Epilogue: O / l -> bf16 rows of `out`.
    const int qrow = q0 + t * kBM + row;
    const bool store = qrow < p.T;
    uint16_t* dst = p.out + b * p.out_sb + h * p.out_sh + static_cast<int64_t>(qrow) * p.out_sr;
    if (!split_unit) {
      if (n == 0) {
        // No valid key: the reference's softmax over an all -inf row is NaN.
        if (store) {
          constexpr uint32_t nan2 = kNaN16x2<kF16>;
          const uint4 nan4 = make_uint4(nan2, nan2, nan2, nan2);
          for (int i = 0; i < kD / 8; ++i) reinterpret_cast<uint4*>(dst)[i] = nan4;
        }
      } else {
        // O row -> this tile's Q slot in shared memory (free: every MMA that read Q is
        // complete once o_full is), in the 128-byte-swizzled layout of the output tensor
        // map's 64-column boxes; then one thread writes the tile with two TMA stores (rows
        // past T are clipped by the map).  The named barrier is reached by all 128 threads
        // of the tile on every path.
        bool have = ok;
        if (have && !wait_or_abort(o_full + t, 0, abort_flag)) {
          record_error(p, abort_flag, 4);
          have = false;
        }
        have = __all_sync(0xffffffffu, have);  // TMEM loads are warp-collective
        uint8_t* stg = sQ + t * kTileBytes;
        if (have) {
          tc_fence_after();
          const float inv_l = 1.f / l;
          uint32_t o[4][32];
#pragma unroll
          for (int q = 0; q < 4; ++q) tmem_ld32(tO + q * 32, o[q]);
          tmem_wait_ld();
#pragma unroll
          for (int c16 = 0; c16 < 16; ++c16) {  // 16-byte chunk = 8 output columns
            const int q = c16 >> 2, i0 = (c16 & 3) * 8;
            const uint4 v4 = make_uint4(
                pack16x2<kF16>(__uint_as_float(o[q][i0]) * inv_l, __uint_as_float(o[q][i0 + 1]) * inv_l),
                pack16x2<kF16>(__uint_as_float(o[q][i0 + 2]) * inv_l, __uint_as_float(o[q][i0 + 3]) * inv_l),
                pack16x2<kF16>(__uint_as_float(o[q][i0 + 4]) * inv_l, __uint_as_float(o[q][i0 + 5]) * inv_l),
                pack16x2<kF16>(__uint_as_float(o[q][i0 + 6]) * inv_l, __uint_as_float(o[q][i0 + 7]) * inv_l));
            const int region = c16 >> 3, chunk = c16 & 7;
            *reinterpret_cast<uint4*>(stg + region * kRegionBytes + row * 128 +
                                      ((chunk ^ (row & 7)) << 4)) = v4;
          }
        }
        fence_proxy_async();
        named_barrier_sync(2 + t, kBM);
        if (wq == 0 && lane == 0 && have) {
          const int r0 = q0 + t * kBM;
          for (int c = 0; c < 2; ++c) {
            if (p.o_token_major)
              tma_store_4d(&tm_o, stg + c * kRegionBytes, c * 64, h, r0, b);
            else
              tma_store_4d(&tm_o, stg + c * kRegionBytes, c * 64, r0, h, b);
          }
          bulk_commit();
          bulk_wait_read0();  // the shared-memory source stays valid until read
        }
      }
    } else {
      // Split unit: publish this piece's unnormalised O and (m, l); the last piece of the
      // item to finish merges all pieces (no CTA ever waits for another one).  Both named
      // barriers are reached by all 256 softmax threads on every path.
      const int sitem = item - p.n_full;
      const int slot = sitem * p.split + piece;
      const int prow = t * kBM + row;  // row within the 256-row block
      float* po = p.part_o + (static_cast<size_t>(slot) * (kQTiles * kBM) + prow) * kD;
      bool have = ok && n > 0;
      if (have && !wait_or_abort(o_full + t, 0, abort_flag)) {
        record_error(p, abort_flag, 4);
        have = false;
      }
      have = __all_sync(0xffffffffu, have);
      if (have) {
        tc_fence_after();
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint32_t o[32];
          tmem_ld32(tO + q * 32, o);
          tmem_wait_ld();
          float4* d4 = reinterpret_cast<float4*>(po + q * 32);
#pragma unroll
          for (int i = 0; i < 8; ++i)
            d4[i] = make_float4(__uint_as_float(o[4 * i]), __uint_as_float(o[4 * i + 1]),
                                __uint_as_float(o[4 * i + 2]), __uint_as_float(o[4 * i + 3]));
        }
      } else {
        for (int i = 0; i < kD / 4; ++i) reinterpret_cast<float4*>(po)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
      float* pml = p.part_ml + static_cast<size_t>(slot) * 2 * (kQTiles * kBM);
      pml[prow] = have ? m : -INFINITY;
      pml[kQTiles * kBM + prow] = have ? l : 0.f;
      __threadfence();
      named_barrier_sync(1, kQTiles * kBM);
      volatile int* last_flag = abort_flag + 1;
      if (threadIdx.x == 4 * 32) {
        const int done = atomicAdd(p.part_cnt + sitem, 1);
        const int last = done == p.split - 1;
        if (last) p.part_cnt[sitem] = 0;  // ready for the next launch
        *last_flag = last;
      }
      named_barrier_sync(1, kQTiles * kBM);
      if (*last_flag) {
        __threadfence();
        const float* ml0 = p.part_ml + static_cast<size_t>(sitem) * p.split * 2 * (kQTiles * kBM);
        float mmax = -INFINITY;
        for (int k = 0; k < p.split; ++k)
          mmax = fmaxf(mmax, __ldcg(ml0 + static_cast<size_t>(k) * 2 * (kQTiles * kBM) + prow));
        float lsum = 0.f;
        float wk[4] = {0.f, 0.f, 0.f, 0.f};
        for (int k = 0; k < p.split && k < 4; ++k) {
          const float* ml = ml0 + static_cast<size_t>(k) * 2 * (kQTiles * kBM);
          const float mk = __ldcg(ml + prow);
          wk[k] = mk == -INFINITY ? 0.f : ex2_approx(mk - mmax);
          lsum += wk[k] * __ldcg(ml + kQTiles * kBM + prow);
        }
        const float inv_l = 1.f / lsum;  // 0/0 = NaN when no piece saw a valid key
        const float* pbase = p.part_o + (static_cast<size_t>(sitem) * p.split * (kQTiles * kBM) + prow) * kD;
#pragma unroll 1
        for (int q = 0; q < 4; ++q) {
          float acc[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) acc[i] = 0.f;
          for (int k = 0; k < p.split && k < 4; ++k) {
            const float4* src = reinterpret_cast<const float4*>(
                pbase + static_cast<size_t>(k) * (kQTiles * kBM) * kD + q * 32);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const float4 x = __ldcg(src + i);
              acc[4 * i] += wk[k] * x.x;
              acc[4 * i + 1] += wk[k] * x.y;
              acc[4 * i + 2] += wk[k] * x.z;
              acc[4 * i + 3] += wk[k] * x.w;
            }
          }
          if (store) {
            uint32_t w[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) w[i] = pack16x2<kF16>(acc[2 * i] * inv_l, acc[2 * i + 1] * inv_l);
            uint4* d4 = reinterpret_cast<uint4*>(dst + q * 32);
#pragma unroll
            for (int i = 0; i < 4; ++i)
              d4[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ------------------------------------------------------------------ wait self-test
// The attention kernel's failure path on a wait that can never complete: warp 0 waits on
// an mbarrier nothing arrives on, gives up after limit_ns, raises the CTA abort flag and
// records status[0] = 1; warp 1, waiting on another such barrier with the abort flag (and
// twice the limit as its own bound), must leave because of the flag and records
// status[1] = 1 when it did.  Both waits end by construction.
__global__ void __launch_bounds__(64) wait_selftest_kernel(int32_t* status, uint64_t limit_ns) {
  __shared__ __align__(8) uint64_t bars[2];
  __shared__ int abort_word;
  volatile int* abort_flag = &abort_word;
  if (threadIdx.x == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    if (!mbar_wait(&bars[0], 0, nullptr, limit_ns)) {
      *abort_flag = 1;
      atomicCAS(status, 0, 1);
    }
  } else if (threadIdx.x == 32 && lane == 0) {
    const uint64_t t0 = global_timer_ns();
    const bool done = mbar_wait(&bars[1], 0, abort_flag, 2 * limit_ns);
    if (!done && *abort_flag && global_timer_ns() - t0 < 2 * limit_ns) atomicCAS(status + 1, 0, 1);
  }
  __syncthreads();
}

// ------------------------------------------------------------------ norm + RoPE
// One warp per token (b, t) at a time (grid-stride over the B*T tokens); a group of 4
// lanes owns one head's row of 128 values, 8 heads side by side, four rows in flight per
// lane (all 32 heads of a token: 8 KiB of loads per warp issued back to back).  Lane `sub`
// of a group holds the 8-value chunks j*4 + sub (j = 0..3), so each load or store
// instruction covers 64 contiguous bytes per row.  The token's RoPE table row is staged
// once per warp in shared memory and the norm weights once per CTA, both reused for every
// head.  Per row: y = RoPE(x / sqrt(mean(x^2) + eps) * w) in f32, rounded to bf16 once,
// written head-major; the sum of squares is 2 shuffles over the group.
struct NormRopeJob {
  const __nv_bfloat16* x;
  __nv_bfloat16* y;
  const float* w;  // NULL: no norm
};

constexpr int kNrRows = 4;     // rows (heads) in flight per lane
constexpr int kNrThreads = 256;

__device__ __forceinline__ void bf16x8_to_f32(const uint4& u, float (&f)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

__device__ __forceinline__ void lds_f32x8(const float* p, float (&f)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p);
  const float4 b = *reinterpret_cast<const float4*>(p + 4);
  f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
  f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}

__global__ void __launch_bounds__(kNrThreads, 2) norm_rope_kernel(
    NormRopeJob j0, NormRopeJob j1, NormRopeJob j2, int B, int T, int H, float eps,
    const float* pe, int64_t pe_bs, int rope_mask, int32_t* zero, int n_zero) {
  __shared__ __align__(16) float s_w[kD];
  __shared__ __align__(16) float s_pe[kNrThreads / 32][kD];
  // Also clears the attention kernel's split arrival counters (n_zero <= 256), which saves
  // a separate memset before the attention launch that follows on the same stream.
  if (zero && blockIdx.x == 0 && blockIdx.y == 0 && static_cast<int>(threadIdx.x) < n_zero)
    zero[threadIdx.x] = 0;
  const NormRopeJob job = blockIdx.y == 0 ? j0 : (blockIdx.y == 1 ? j1 : j2);
  const bool rope = pe != nullptr && ((rope_mask >> blockIdx.y) & 1);
  const bool norm = job.w != nullptr;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int sub = lane & 3;   // chunk column within the group
  const int hl = lane >> 2;   // head offset within the warp's 8
  if (norm && threadIdx.x < kD / 4)
    reinterpret_cast<float4*>(s_w)[threadIdx.x] = reinterpret_cast<const float4*>(job.w)[threadIdx.x];
  __syncthreads();
  float* pe_s = s_pe[warp];
  const int64_t tokens = static_cast<int64_t>(B) * T;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (kNrThreads / 32);
  for (int64_t tok = static_cast<int64_t>(blockIdx.x) * (kNrThreads / 32) + warp; tok < tokens;
       tok += warps) {
    const int b = static_cast<int>(tok / T), t = static_cast<int>(tok - static_cast<int64_t>(b) * T);
    const __nv_bfloat16* xt = job.x + tok * H * kD;
    // Every lane runs the same trip count (the shuffles need the whole warp).
    for (int hb = 0; hb < H; hb += 8 * kNrRows) {
      uint4 xv[kNrRows][4];
#pragma unroll
      for (int r = 0; r < kNrRows; ++r) {
        const int h = hb + r * 8 + hl;
#pragma unroll
        for (int j = 0; j < 4; ++j)
          xv[r][j] = h < H ? *reinterpret_cast<const uint4*>(xt + static_cast<int64_t>(h) * kD +
                                                              j * 32 + sub * 8)
                           : make_uint4(0, 0, 0, 0);
      }
      if (rope && hb == 0) {
        const float4 c = reinterpret_cast<const float4*>(
            pe + static_cast<int64_t>(b) * pe_bs + static_cast<int64_t>(t) * kD)[lane];
        __syncwarp();  // the previous token's reads of pe_s are done
        reinterpret_cast<float4*>(pe_s)[lane] = c;
        __syncwarp();
      }
#pragma unroll
      for (int r = 0; r < kNrRows; ++r) {
        const int h = hb + r * 8 + hl;
        // The row stays packed (bf16) in registers: unpacked once for the sum of squares
        // and again, a chunk at a time, for the transform.
        float inv = 1.f;
        if (norm) {
          float ss = 0.f;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float v[8];
            bf16x8_to_f32(xv[r][j], v);
#pragma unroll
            for (int e = 0; e < 8; ++e) ss = fmaf(v[e], v[e], ss);
          }
          ss += __shfl_xor_sync(0xffffffffu, ss, 1);
          ss += __shfl_xor_sync(0xffffffffu, ss, 2);
          inv = 1.f / sqrtf(ss / static_cast<float>(kD) + eps);
        }
        if (h >= H) continue;
        __nv_bfloat16* yr = job.y + ((static_cast<int64_t>(b) * H + h) * T + t) * kD;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float v[8];
          bf16x8_to_f32(xv[r][j], v);
          if (norm) {
            float w[8];
            lds_f32x8(s_w + j * 32 + sub * 8, w);
#pragma unroll
            for (int e = 0; e < 8; ++e) v[e] = v[e] * inv * w[e];
          }
          if (rope) {
            float cs[8];
            lds_f32x8(pe_s + j * 32 + sub * 8, cs);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const float x0 = v[2 * q], x1 = v[2 * q + 1];
              const float co = cs[2 * q], si = cs[2 * q + 1];
              v[2 * q] = x0 * co - x1 * si;
              v[2 * q + 1] = x0 * si + x1 * co;
            }
          }
          *reinterpret_cast<uint4*>(yr + j * 32 + sub * 8) =
              make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]),
                         pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
        }
      }
    }
  }
}

// ------------------------------------------------------------------ host helpers
namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// 4-D map over a bf16 tensor with 128 columns per row and a 64 x 128-row box, 128-byte
// swizzle, zero fill outside the tensor.  head_major: [B,H,rows,128] with coordinates
// (d, row, h, b); otherwise token-major [B,rows,H,128] with coordinates (d, h, row, b).
int make_map(CUtensorMap* map, const void* base, int B, int H, int rows, bool head_major,
             bool f16 = false) {
  auto fn = encode_fn();
  if (!fn) return B200_ERR_CUDA;
  cuuint64_t dims[4];
  cuuint64_t strides[3];
  cuuint32_t box[4];
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const cuuint64_t row_bytes = kD * 2;
  if (head_major) {
    dims[0] = kD; dims[1] = rows; dims[2] = H; dims[3] = B;
    strides[0] = row_bytes;
    strides[1] = row_bytes * rows;
    strides[2] = row_bytes * rows * H;
    box[0] = 64; box[1] = kBN; box[2] = 1; box[3] = 1;
  } else {
    dims[0] = kD; dims[1] = H; dims[2] = rows; dims[3] = B;
    strides[0] = row_bytes;
    strides[1] = row_bytes * H;
    strides[2] = row_bytes * H * rows;
    box[0] = 64; box[1] = 1; box[2] = kBN; box[3] = 1;
  }
  CUresult r = fn(map, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                  4, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? B200_OK : B200_ERR_CUDA;
}

}  // namespace

// Unique id of the calling thread's current CUDA context (cuCtxGetId: unique for the
// life of the process, so a context re-created after cudaDeviceReset gets a new one);
// 0 when there is no current context yet or the driver lacks the call.  Per-device host
// caches of device state are keyed by it, so they are rebuilt after a reset.
static unsigned long long current_context_id() {
  using GetCurrent = CUresult (*)(CUcontext*);
  using GetId = CUresult (*)(CUcontext, unsigned long long*);
  static GetCurrent get_current = nullptr;
  static GetId get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<GetCurrent>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<GetId>(p);
  });
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (!get_current || !get_id || get_current(&ctx) != CUDA_SUCCESS || !ctx) return 0;
  if (get_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return id;
}

namespace {

std::mutex g_attr_mutex;
unsigned long long g_attr_ctx[64] = {};  // context the kernel attributes were set in

int ensure_kernel_attrs() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return B200_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_attr_mutex);
  const unsigned long long ctx = current_context_id();
  if (dev >= 0 && dev < 64 && ctx != 0 && g_attr_ctx[dev] == ctx) return B200_OK;
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  if (major != 10 || minor != 0) return B200_ERR_UNSUPPORTED;
  if (cudaFuncSetAttribute(joint_attn_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           kSmemBytes) != cudaSuccess ||
      cudaFuncSetAttribute(joint_attn_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           kSmemBytes) != cudaSuccess)
    return B200_ERR_CUDA;
  if (dev >= 0 && dev < 64) g_attr_ctx[dev] = current_context_id();
  return B200_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

constexpr size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Tail split.  With `items` work items on `sms` SMs, the last wave holds items % sms
// CTAs; when that is at most half the SMs, those items are cut into `split` pieces of
// key tiles (at most 4, and at least 2 tiles a piece for the longest item) so the wave
// spreads over the idle SMs.  Each piece needs one slot of partial results.
constexpr int kMaxSplitSlots = 160;  // >= the SM count of sm_100 parts
constexpr size_t kSplitSlotBytes = size_t{kQTiles} * kBM * kD * 4 + 2 * size_t{kQTiles} * kBM * 4;
constexpr size_t kSplitRegionBytes =
    round_up(size_t{kMaxSplitSlots} * kSplitSlotBytes + size_t{kMaxSplitSlots} * 4, 256);
static_assert(kSplitRegionBytes == B200_ATTN_SPLIT_WORKSPACE_BYTES,
              "header constant must match the split-region layout");

struct SplitPlan {
  int n_full, split, units;
};

int sm_count() {
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
    return 148;
  return sms;
}

SplitPlan plan_units(int items, int max_tiles, bool have_region) {
  SplitPlan sp{items, 1, items};
  const int sms = sm_count();
  if (!have_region || items <= sms) return sp;
  const int tail = items % sms;
  if (tail == 0 || 2 * tail > sms) return sp;
  int split = std::min(4, sms / tail);
  split = std::min(split, max_tiles / 2);
  split = std::min(split, kMaxSplitSlots / tail);
  if (split < 2) return sp;
  sp.n_full = items - tail;
  sp.split = split;
  sp.units = sp.n_full + tail * split;
  return sp;
}

// Fills the work-unit fields of prm (split region optional) and launches.
int launch_attention(const CUtensorMap& mq, const CUtensorMap& mk0, const CUtensorMap& mv0,
                     const CUtensorMap& mk1, const CUtensorMap& mv1, const CUtensorMap& mo,
                     AttnParams prm, int B,
                     int H, int T, int max_tiles, void* split_region, cudaStream_t stream,
                     bool counters_zeroed = false, bool f16 = false) {
  int rc = ensure_kernel_attrs();
  if (rc != B200_OK) return rc;
  prm.H = H;
  prm.nqb = (T + kQTiles * kBM - 1) / (kQTiles * kBM);
  const int64_t items = static_cast<int64_t>(B) * H * prm.nqb;
  if (items > 0x7fffffff / 4) return B200_ERR_INVALID;
  const SplitPlan sp = plan_units(static_cast<int>(items), max_tiles, split_region != nullptr);
  prm.n_full = sp.n_full;
  prm.split = sp.split;
  if (sp.split > 1) {
    auto* base = static_cast<uint8_t*>(split_region);
    prm.part_o = reinterpret_cast<float*>(base);
    prm.part_ml = reinterpret_cast<float*>(base + size_t{kMaxSplitSlots} * kQTiles * kBM * kD * 4);
    prm.part_cnt = reinterpret_cast<int32_t*>(base + size_t{kMaxSplitSlots} * kSplitSlotBytes);
    const size_t cnt_bytes = sizeof(int32_t) * static_cast<size_t>(sp.units - sp.n_full) / sp.split;
    if (!counters_zeroed && cudaMemsetAsync(prm.part_cnt, 0, cnt_bytes, stream) != cudaSuccess)
      return B200_ERR_CUDA;
  }
  if (f16)
    joint_attn_kernel<true><<<dim3(sp.units), kThreads, kSmemBytes, stream>>>(mq, mk0, mv0, mk1, mv1, mo, prm);
  else
    joint_attn_kernel<false><<<dim3(sp.units), kThreads, kSmemBytes, stream>>>(mq, mk0, mv0, mk1, mv1, mo, prm);
  return cudaGetLastError() == cudaSuccess ? B200_OK : B200_ERR_CUDA;
}

int launch_norm_rope(const NormRopeJob* jobs, int njobs, int B, int T, int H, float eps,
                     const float* pe, int64_t pe_bs, int rope_mask, cudaStream_t stream,
                     int32_t* zero = nullptr, int n_zero = 0) {
  const int64_t rows = static_cast<int64_t>(B) * T * H;
  if (rows == 0 || njobs == 0) return B200_OK;
  if (rows >= (int64_t{1} << 31)) return B200_ERR_INVALID;
  // One warp per token; enough CTAs (8 warps each) for every SM to hold several per job,
  // the grid-stride loop takes the rest.
  static const int64_t slots = [] {  // resident CTAs of this kernel on the whole GPU
    int dev = 0, n = 148, c = 2;
    if (cudaGetDevice(&dev) == cudaSuccess)
      cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&c, norm_rope_kernel, kNrThreads, 0) !=
            cudaSuccess ||
        c < 1)
      c = 1;
    return int64_t{n} * c;
  }();
  const int64_t tokens = static_cast<int64_t>(B) * T;
  const int64_t want = (tokens + 7) / 8;
  const int64_t cap = std::max<int64_t>(1, slots * 2 / njobs);
  const int64_t blocks = std::min(want, cap);
  NormRopeJob j[3] = {jobs[0], njobs > 1 ? jobs[1] : jobs[0], njobs > 2 ? jobs[2] : jobs[0]};
  dim3 grid(static_cast<unsigned>(blocks), njobs);
  norm_rope_kernel<<<grid, kNrThreads, 0, stream>>>(j[0], j[1], j[2], B, T, H, eps, pe, pe_bs, rope_mask,
                                             zero, n_zero);
  return cudaGetLastError() == cudaSuccess ? B200_OK : B200_ERR_CUDA;
}

// Attention of post-RoPE q [B,H,T,D] over [prefix (B,H,P,D) ; step k_rot (B,H,T,D) and
// v (B,T,H,D, token-major)], out [B,T,H*D].  Arguments are already validated.
int joint_attention(const void* q_rot, const void* k_rot, const void* v, const void* prefix_k,
                    const void* prefix_v, int B, int H, int T, int P, const b200_kv_desc* desc,
                    float scale, void* out, int32_t* status, void* split_region,
                    cudaStream_t stream, bool counters_zeroed = false,
                    const int32_t* row_limit = nullptr) {
  CUtensorMap mq{}, mk0{}, mv0{}, mk1{}, mv1{}, mo{};
  int rc;
  if ((rc = make_map(&mq, q_rot, B, H, T, true)) != B200_OK) return rc;
  if ((rc = make_map(&mo, out, B, H, T, false)) != B200_OK) return rc;
  if ((rc = make_map(&mk1, k_rot, B, H, T, true)) != B200_OK) return rc;
  if ((rc = make_map(&mv1, v, B, H, T, false)) != B200_OK) return rc;
  if (P > 0) {
    if ((rc = make_map(&mk0, prefix_k, B, H, P, true)) != B200_OK) return rc;
    if ((rc = make_map(&mv0, prefix_v, B, H, P, true)) != B200_OK) return rc;
  }
  AttnParams prm{};
  prm.T = T;
  prm.P = P;
  prm.L1 = T;
  prm.v1_token_major = 1;
  prm.seg0_len = desc ? &desc[0].prefix_valid : nullptr;
  prm.seg1_len = desc ? &desc[0].target_valid : nullptr;
  prm.row_limit = row_limit;
  prm.seg0_stride = 2;
  prm.seg1_stride = 2;
  prm.scale_log2 = scale * 1.4426950408889634f;
  prm.out = static_cast<uint16_t*>(out);
  prm.out_sb = static_cast<int64_t>(T) * H * kD;
  prm.out_sh = kD;
  prm.out_sr = static_cast<int64_t>(H) * kD;
  prm.status = status;
  const int max_tiles = (P + kBN - 1) / kBN + (T + kBN - 1) / kBN;
  prm.o_token_major = 1;
  return launch_attention(mq, mk0, mv0, mk1, mv1, mo, prm, B, H, T, max_tiles, split_region, stream,
                          counters_zeroed);
}

}  // namespace
}  // namespace b200

using namespace b200;

extern "C" int b200_attn_workspace_bytes(const b200_attn_args* a, size_t* bytes) {
  if (!a || !bytes) return B200_ERR_INVALID;
  if (a->batch < 0 || a->heads < 0 || a->target_len < 0) return B200_ERR_INVALID;
  const size_t tensor = static_cast<size_t>(a->batch) * a->heads * a->target_len * kD * 2;
  size_t need = round_up(tensor, 256);               // post-RoPE Q
  if (!a->k_rot_out) need += round_up(tensor, 256);  // post-RoPE K
  *bytes = need + kSplitRegionBytes;                 // partial results of the tail split
  return B200_OK;
}

extern "C" int b200_attn_fwd(const b200_attn_args* a, b200_stream_t stream_) {
  if (!a) return B200_ERR_INVALID;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  if (a->head_dim != kD) return B200_ERR_UNSUPPORTED;
  if (a->batch <= 0 || a->heads <= 0 || a->target_len < 0 || a->prefix_len < 0)
    return B200_ERR_INVALID;
  if (a->target_len == 0) return B200_OK;
  if (!a->q || !a->k || !a->v || !a->out || !a->norm_q_w || !a->norm_k_w || !a->pe)
    return B200_ERR_INVALID;
  if (a->prefix_len > 0 && (!a->prefix_k || !a->prefix_v)) return B200_ERR_INVALID;
  if (!(a->scale > 0.f) || !std::isfinite(a->scale)) return B200_ERR_INVALID;
  // Per-batch RoPE rows must keep the 16-byte alignment of the float4 loads.
  if (a->pe_batch_stride < 0 || a->pe_batch_stride % 4 != 0) return B200_ERR_INVALID;
  const void* ptrs[] = {a->q, a->k, a->v, a->out, a->norm_q_w, a->norm_k_w, a->pe,
                        a->workspace, a->k_rot_out, a->v_out, a->prefix_k, a->prefix_v};
  for (const void* ptr : ptrs)
    if (ptr && !aligned16(ptr)) return B200_ERR_INVALID;
  size_t need = 0;
  b200_attn_workspace_bytes(a, &need);
  const size_t need_min = need - kSplitRegionBytes;  // without the tail split
  if (!a->workspace || a->workspace_bytes < need_min) return B200_ERR_WORKSPACE;

  const int B = a->batch, H = a->heads, T = a->target_len, P = a->prefix_len;
  const size_t tensor = static_cast<size_t>(B) * H * T * kD * 2;
  auto* ws = static_cast<uint8_t*>(a->workspace);
  auto* q_rot = reinterpret_cast<__nv_bfloat16*>(ws);
  auto* k_rot = a->k_rot_out ? static_cast<__nv_bfloat16*>(a->k_rot_out)
                             : reinterpret_cast<__nv_bfloat16*>(ws + round_up(tensor, 256));

  NormRopeJob jobs[3] = {
      {static_cast<const __nv_bfloat16*>(a->q), q_rot, a->norm_q_w},
      {static_cast<const __nv_bfloat16*>(a->k), k_rot, a->norm_k_w},
      {static_cast<const __nv_bfloat16*>(a->v), static_cast<__nv_bfloat16*>(a->v_out), nullptr}};
  void* split_region = a->workspace_bytes >= need ? ws + need_min : nullptr;
  int32_t* counters = split_region
                          ? reinterpret_cast<int32_t*>(static_cast<uint8_t*>(split_region) +
                                                       size_t{kMaxSplitSlots} * kSplitSlotBytes)
                          : nullptr;
  int rc = launch_norm_rope(jobs, a->v_out ? 3 : 2, B, T, H, a->norm_eps, a->pe,
                            a->pe_batch_stride, 0x3, stream, counters,
                            counters ? kMaxSplitSlots : 0);
  if (rc != B200_OK) return rc;

  return joint_attention(q_rot, k_rot, a->v, a->prefix_k, a->prefix_v, B, H, T, P, a->desc,
                         a->scale, a->out, a->status, split_region, stream, true, a->row_limit);
}

extern "C" int b200_joint_attention(const void* q_rot, const void* k_rot, const void* v,
                                    const void* prefix_k, const void* prefix_v, int32_t batch,
                                    int32_t heads, int32_t target_len, int32_t prefix_len,
                                    int32_t head_dim, const b200_kv_desc* desc, float scale,
                                    void* out, void* workspace, size_t workspace_bytes,
                                    int32_t* status, b200_stream_t stream) {
  if (head_dim != kD) return B200_ERR_UNSUPPORTED;
  if (batch <= 0 || heads <= 0 || target_len < 0 || prefix_len < 0) return B200_ERR_INVALID;
  if (target_len == 0) return B200_OK;
  if (!q_rot || !k_rot || !v || !out) return B200_ERR_INVALID;
  if (prefix_len > 0 && (!prefix_k || !prefix_v)) return B200_ERR_INVALID;
  const void* ptrs[] = {q_rot, k_rot, v, out, prefix_k, prefix_v};
  for (const void* ptr : ptrs)
    if (ptr && !aligned16(ptr)) return B200_ERR_INVALID;
  if (!(scale > 0.f) || !std::isfinite(scale)) return B200_ERR_INVALID;
  if (workspace && !aligned16(workspace)) return B200_ERR_INVALID;
  void* split_region = workspace && workspace_bytes >= kSplitRegionBytes ? workspace : nullptr;
  return joint_attention(q_rot, k_rot, v, prefix_k, prefix_v, batch, heads, target_len,
                         prefix_len, desc, scale, out, status, split_region,
                         static_cast<cudaStream_t>(stream));
}

extern "C" int b200_chunked_attention(const void* q, const void* k, const void* v, void* out,
                                      int32_t batch, int32_t heads, int32_t sq, int32_t skv,
                                      int32_t head_dim, float scale, const int32_t* key_len,
                                      int32_t* status, b200_stream_t stream_) {
  if (head_dim != kD) return B200_ERR_UNSUPPORTED;
  if (batch <= 0 || heads <= 0 || sq < 0 || skv <= 0) return B200_ERR_INVALID;
  if (sq == 0) return B200_OK;
  if (!q || !k || !v || !out) return B200_ERR_INVALID;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out)) return B200_ERR_INVALID;
  if (!(scale > 0.f) || !std::isfinite(scale)) return B200_ERR_INVALID;
  CUtensorMap mq{}, mk0{}, mv0{}, mk1{}, mv1{}, mo{};
  int rc;
  if ((rc = make_map(&mq, q, batch, heads, sq, true)) != B200_OK) return rc;
  if ((rc = make_map(&mo, out, batch, heads, sq, true)) != B200_OK) return rc;
  if ((rc = make_map(&mk1, k, batch, heads, skv, true)) != B200_OK) return rc;
  if ((rc = make_map(&mv1, v, batch, heads, skv, true)) != B200_OK) return rc;
  AttnParams prm{};
  prm.T = sq;
  prm.P = 0;
  prm.L1 = skv;
  prm.v1_token_major = 0;
  prm.seg1_len = key_len;
  prm.seg1_stride = 1;
  prm.scale_log2 = scale * 1.4426950408889634f;
  prm.out = static_cast<uint16_t*>(out);
  prm.out_sb = static_cast<int64_t>(heads) * sq * kD;
  prm.out_sh = static_cast<int64_t>(sq) * kD;
  prm.out_sr = kD;
  prm.status = status;
  prm.o_token_major = 0;
  return launch_attention(mq, mk0, mv0, mk1, mv1, mo, prm, batch, heads, sq, (skv + kBN - 1) / kBN,
                          nullptr, static_cast<cudaStream_t>(stream_));
}

namespace {
// flash_attn(q, k, v, scale, causal = false) on token-major [B,S,H,D] tensors of either
// 16-bit type; arguments validated by the callers.
int flash_attention_impl(const void* q, const void* k, const void* v, void* out, int32_t batch,
                         int32_t sq, int32_t skv, int32_t heads, float scale,
                         const int32_t* key_len, int32_t* status, cudaStream_t stream, bool f16) {
  CUtensorMap mq{}, mk0{}, mv0{}, mk1{}, mv1{}, mo{};
  int rc;
  if ((rc = make_map(&mq, q, batch, heads, sq, false, f16)) != B200_OK) return rc;
  if ((rc = make_map(&mo, out, batch, heads, sq, false, f16)) != B200_OK) return rc;
  if ((rc = make_map(&mk1, k, batch, heads, skv, false, f16)) != B200_OK) return rc;
  if ((rc = make_map(&mv1, v, batch, heads, skv, false, f16)) != B200_OK) return rc;
  AttnParams prm{};
  prm.T = sq;
  prm.P = 0;
  prm.L1 = skv;
  prm.q_token_major = 1;
  prm.k1_token_major = 1;
  prm.v1_token_major = 1;
  prm.seg1_len = key_len;
  prm.seg1_stride = 1;
  prm.scale_log2 = scale * 1.4426950408889634f;
  prm.out = static_cast<uint16_t*>(out);
  prm.out_sb = static_cast<int64_t>(sq) * heads * kD;
  prm.out_sh = kD;
  prm.out_sr = static_cast<int64_t>(heads) * kD;
  prm.status = status;
  prm.o_token_major = 1;
  return launch_attention(mq, mk0, mv0, mk1, mv1, mo, prm, batch, heads, sq, (skv + kBN - 1) / kBN,
                          nullptr, stream, false, f16);
}

int flash_attention_check(const void* q, const void* k, const void* v, void* out,
                          int32_t batch, int32_t sq, int32_t skv, int32_t heads,
                          int32_t head_dim, float scale) {
  if (head_dim != kD) return B200_ERR_UNSUPPORTED;
  if (batch <= 0 || heads <= 0 || sq < 0 || skv <= 0) return B200_ERR_INVALID;
  if (!q || !k || !v || !out) return B200_ERR_INVALID;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out)) return B200_ERR_INVALID;
  if (!(scale > 0.f) || !std::isfinite(scale)) return B200_ERR_INVALID;
  return B200_OK;
}
}  // namespace

extern "C" int b200_flash_attention(const void* q, const void* k, const void* v, void* out,
                                    int32_t batch, int32_t sq, int32_t skv, int32_t heads,
                                    int32_t head_dim, float scale, const int32_t* key_len,
                                    int32_t* status, b200_stream_t stream_) {
  if (head_dim == kD && batch > 0 && heads > 0 && sq == 0 && skv > 0) return B200_OK;
  const int rc = flash_attention_check(q, k, v, out, batch, sq, skv, heads, head_dim, scale);
  if (rc != B200_OK) return rc;
  return flash_attention_impl(q, k, v, out, batch, sq, skv, heads, scale, key_len, status,
                              static_cast<cudaStream_t>(stream_), false);
}

extern "C" int b200_flash_attention_ex(const void* q, const void* k, const void* v, void* out,
                                       int32_t batch, int32_t sq, int32_t skv, int32_t heads,
                                       int32_t head_dim, float scale, const int32_t* key_len,
                                       int32_t dtype, int32_t* status, b200_stream_t stream_) {
  if (dtype != B200_DTYPE_BF16 && dtype != B200_DTYPE_F16) return B200_ERR_UNSUPPORTED;
  if (head_dim == kD && batch > 0 && heads > 0 && sq == 0 && skv > 0) return B200_OK;
  const int rc = flash_attention_check(q, k, v, out, batch, sq, skv, heads, head_dim, scale);
  if (rc != B200_OK) return rc;
  return flash_attention_impl(q, k, v, out, batch, sq, skv, heads, scale, key_len, status,
                              static_cast<cudaStream_t>(stream_), dtype == B200_DTYPE_F16);
}

extern "C" int b200_norm_rope(const void* x, void* y, int32_t batch, int32_t tokens,
                              int32_t heads, int32_t head_dim, const float* norm_w, float eps,
                              const float* pe, b200_stream_t stream) {
  if (head_dim != kD) return B200_ERR_UNSUPPORTED;
  if (batch < 0 || tokens < 0 || heads < 0) return B200_ERR_INVALID;
  if (!x || !y || !aligned16(x) || !aligned16(y)) return B200_ERR_INVALID;
  if ((norm_w && !aligned16(norm_w)) || (pe && !aligned16(pe))) return B200_ERR_INVALID;
  NormRopeJob job{static_cast<const __nv_bfloat16*>(x), static_cast<__nv_bfloat16*>(y), norm_w};
  return launch_norm_rope(&job, 1, batch, tokens, heads, eps, pe, 0, 0x1,
                          static_cast<cudaStream_t>(stream));
}

extern "C" int b200_qk_norm_rope(const void* q, const void* k, void* q_rot, void* k_rot,
                                 int32_t batch, int32_t tokens, int32_t heads,
                                 int32_t head_dim, const float* norm_q_w, const float* norm_k_w,
                                 float eps, const float* pe, b200_stream_t stream) {
  if (head_dim != kD) return B200_ERR_UNSUPPORTED;
  if (batch < 0 || tokens < 0 || heads < 0) return B200_ERR_INVALID;
  const void* ptrs[] = {q, k, q_rot, k_rot, norm_q_w, norm_k_w, pe};
  for (const void* ptr : ptrs)
    if (!ptr || !aligned16(ptr)) return B200_ERR_INVALID;
  NormRopeJob jobs[2] = {
      {static_cast<const __nv_bfloat16*>(q), static_cast<__nv_bfloat16*>(q_rot), norm_q_w},
      {static_cast<const __nv_bfloat16*>(k), static_cast<__nv_bfloat16*>(k_rot), norm_k_w}};
  return launch_norm_rope(jobs, 2, batch, tokens, heads, eps, pe, 0, 0x3,
                          static_cast<cudaStream_t>(stream));
}

// ------------------------------------------------------------------ no-allocation entry
// For callers that cannot allocate device memory at call time — e.g. an engine whose
// allocator is frozen or owned by another runtime, a plugin host that hands out only
// the input and output tensors, or code between a memory-pool snapshot and its
// replay — b200_attn_fwd_noalloc runs the same two kernels with the scratch taken from
// this file-scope device array instead of a caller workspace.  Every GPU that loads
// the library holds the array until the process exits.
static __device__ __align__(256) unsigned char g_noalloc_scratch[B200_NOALLOC_SCRATCH_BYTES];

namespace {
std::mutex g_noalloc_mutex;
void* g_noalloc_scratch_ptr[64] = {};             // device address of g_noalloc_scratch
unsigned long long g_noalloc_scratch_ctx[64] = {};  // the context that address belongs to
}  // namespace

extern "C" int b200_attn_fwd_noalloc(const b200_attn_args* args, b200_stream_t stream) {
  if (!args) return B200_ERR_INVALID;
  size_t need = 0;
  int rc = b200_attn_workspace_bytes(args, &need);
  if (rc != B200_OK) return rc;
  // The limit applies to the required scratch; the optional tail-split region is used
  // only when it also fits (b200_attn_fwd decides from workspace_bytes).
  if (need - B200_ATTN_SPLIT_WORKSPACE_BYTES > B200_NOALLOC_SCRATCH_BYTES)
    return B200_ERR_WORKSPACE;  // over the fixed limit
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return B200_ERR_CUDA;
  if (dev < 0 || dev >= 64) return B200_ERR_UNSUPPORTED;
  void* scratch = nullptr;
  {
    // One-time set-up per device (with that device current): the host-side name of the
    // array is only a stand-in, so the kernels get its device address.
    // The address is looked up again when the device's context changed (after a
    // cudaDeviceReset the array lives at a new address in a new context).
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    const unsigned long long ctx = current_context_id();
    if (!g_noalloc_scratch_ptr[dev] || ctx == 0 || g_noalloc_scratch_ctx[dev] != ctx) {
      void* ptr = nullptr;
      if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || !ptr)
        return B200_ERR_CUDA;
      g_noalloc_scratch_ptr[dev] = ptr;
      g_noalloc_scratch_ctx[dev] = current_context_id();
    }
    scratch = g_noalloc_scratch_ptr[dev];
  }
  // Nothing in the scratch needs clearing: every byte the attention kernel reads from it
  // (post-RoPE Q, and K when k_rot_out is NULL) is written by the prologue of this call.
  b200_attn_args a = *args;
  a.workspace = scratch;
  a.workspace_bytes = B200_NOALLOC_SCRATCH_BYTES;
  return b200_attn_fwd(&a, stream);
}

extern "C" int b200_wait_selftest(int32_t* status, uint32_t limit_us, b200_stream_t stream) {
  if (!status || limit_us == 0 || limit_us > 2000000u) return B200_ERR_INVALID;
  if (reinterpret_cast<uintptr_t>(status) & 3u) return B200_ERR_INVALID;
  wait_selftest_kernel<<<1, 64, 0, static_cast<cudaStream_t>(stream)>>>(
      status, static_cast<uint64_t>(limit_us) * 1000ull);
  return cudaGetLastError() == cudaSuccess ? B200_OK : B200_ERR_CUDA;
}
