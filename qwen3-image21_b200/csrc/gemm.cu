// gemm.cu — C = A · Bᵀ on tcgen05 with an epilogue that can reduce across GPUs.
//
// A [M, K] and B [N, K] are bf16, K-major (B is a Linear's weight [out, in]); the product
// accumulates in f32 in TMEM.  The epilogue stores bf16, or adds f32 into a buffer with
// `red.global.add` (a local buffer or another GPU's, through a peer pointer), or scatters
// bf16 rows to the GPU that owns them (plain stores over NVLink into that GPU's slot for
// this GPU).  The scatter is the out-projection of head-sharded attention fused with the
// reduce-scatter of its partial sums: a GPU's partial tile leaves for its owner as soon as
// it is computed; b200_reduce_gather_bf16 then sums each owner's slots and broadcasts.
//
// Structure: persistent CTAs (one per SM), 128 x 256 output tiles in a grouped raster
// (tile_coords), 64-deep K steps.
//   warp 0      TMA producer: A and B tiles into a 4-stage ring (no multicast)
//   warp 1      MMA issuer: 4 x tcgen05.mma M128 N256 K16 per K step
//   warp 2      TMEM allocator: 2 x 256 columns, the accumulator of the current tile and
//               of the next one, so a tile's epilogue overlaps the next tile's MMAs
//   warps 4-7   epilogue: TMEM -> registers -> a swizzled 128-row x 128-byte staging tile
//               in shared memory (32 f32 or 64 bf16 columns) -> 16-byte vectors along rows
//               (8 lanes cover one row's 128 contiguous bytes), so global / NVLink traffic
//               leaves in full segments.
// Every wait is bounded (ptx.cuh); a wait that runs out records a status code and the CTA
// unwinds.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdint>
#include <cstdlib>
#include <mutex>

#include "../../include/b200_attn.h"
#include "../../include/b200_gemm.h"
#include "ptx.cuh"

namespace b200 {
namespace {

constexpr int kGM = 128;                     // tile rows
constexpr int kGN = 256;                     // tile columns
constexpr int kGK = 64;                      // K per stage (one 128-byte swizzle span)
constexpr int kGStages = 4;
constexpr int kATileBytes = kGM * kGK * 2;   // 16 KiB
constexpr int kBTileBytes = kGN * kGK * 2;   // 32 KiB
constexpr int kStageBytes = kATileBytes + kBTileBytes;
constexpr int kStageSmem = kGStages * kStageBytes;          // 192 KiB
constexpr int kEpiChunk = 32;                                // columns per epilogue pass
constexpr int kEpiSmem = kGM * kEpiChunk * 4;                // 16 KiB staging tile
constexpr int kGBarOff = kStageSmem + kEpiSmem;
constexpr int kGSmemBytes = kGBarOff + 256 + 1024;           // barriers + alignment slack
constexpr int kGThreads = 256;
constexpr uint32_t kGTmemCols = 512;                         // 2 accumulators x 256

constexpr int kMaxOwners = 8;

struct GemmParams {
  int32_t M, N, K;
  int32_t tile_m;      // rows per output tile: 128 (one CTA) or 256 (a CTA pair)
  int32_t group_m;     // row blocks per raster group (see tile_coords)
  int32_t tiles_m, tiles_n, tiles;
  int32_t mode;        // B200_GEMM_STORE_BF16 / _RED_F32 / _SCATTER_BF16
  int64_t ldc;         // elements between rows of C
  void* C;
  int32_t* status;
  // B200_GEMM_SCATTER_BF16: row m goes to owner q = m / rows_per_owner, into slot
  // `src_slot` of owner q's buffer: peers[q] + (src_slot * rows_per_owner + m - q *
  // rows_per_owner) * ldc.
  void* peers[kMaxOwners];
  int32_t rows_per_owner, src_slot;
  // B200_GEMM_QKV: N = 3 * heads * 128 columns [q | k | v]; row m is token t = m % tokens
  // of batch row b = m / tokens.  q and k get RMSNorm (norm_q / norm_k, eps) and RoPE (pe
  // rows: pe + b * pe_bs + t * 128) and go head-major [B, H, T, 128] to q_out / k_out; v
  // goes token-major [B, T, H * 128] to v_out.
  int32_t heads, tokens;
  const float* pe;
  int64_t pe_bs;
  const float* norm_q;
  const float* norm_k;
  float eps;
  void* q_out;
  void* k_out;
  void* v_out;
};

struct ReduceGatherDst {
  void* ptr[kMaxOwners];
  int32_t n;
  int64_t row0, ld8;
};

__device__ __forceinline__ uint32_t gemm_pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ void red_add_v4(float* p, float a, float b, float c, float d) {
  asm volatile("red.relaxed.sys.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a),
               "f"(b), "f"(c), "f"(d)
               : "memory");
}


// Grouped raster: tiles run in groups of group_m row blocks, row-block-fastest inside a
// group.  The group's A rows (sized on the host to about half of L2) stay in L2 while the
// group walks every column block, and the tiles in flight share a narrow band of B: A
// comes from HBM about once and B once per group, also when B is larger than L2.
__device__ __forceinline__ void tile_coords(const GemmParams& p, int t, int& m0, int& n0) {
  const int per_group = p.group_m * p.tiles_n;
  const int g = t / per_group;
  const int first = g * p.group_m;
  const int gm = min(p.group_m, p.tiles_m - first);
  const int local = t - g * per_group;
  m0 = (first + local % gm) * p.tile_m;
  n0 = (local / gm) * kGN;
}

__device__ __forceinline__ void gemm_error(const GemmParams& p, volatile int* abort_flag, int code) {
  *abort_flag = 1;
  if (p.status) atomicCAS(p.status, 0, code);
}

// One tile's epilogue by the 128 epilogue threads of a CTA: accumulator `ab` of TMEM
// (this thread's lane quadrant `q`, row `trow` of the tile), output rows m0 + trow.
__device__ __forceinline__ void epilogue_tile(const GemmParams& p, uint32_t tmem_base,
                                              uint32_t lane_off, int ab, int m0, int n0,
                                              int q, int lane, int trow, float* stage_tile) {
  // staging tile: row r holds 32 f32 = 8 chunks of 16 bytes, chunk j at (j ^ (r & 7))
  float4* st_row = reinterpret_cast<float4*>(stage_tile) + trow * 8;
  const int sub = lane & 7;  // 16-byte chunk this lane moves in a pass
  const int hidden = p.heads * 128;
  const int which = p.mode == B200_GEMM_QKV ? n0 / hidden : -1;
  if (which == 0 || which == 1) {
    // Q or K of two heads: RMSNorm over each head's 128 values (a first pass over TMEM
    // for the sum of squares), then RoPE, bf16, head-major rows, 64 columns per pass.
    const float* wn = which == 0 ? p.norm_q : p.norm_k;
    __nv_bfloat16* dst_base = static_cast<__nv_bfloat16*>(which == 0 ? p.q_out : p.k_out);
    const int m = m0 + trow;
    const int mb = m < p.M ? m / p.tokens : 0;
    const int mt = m < p.M ? m - mb * p.tokens : 0;
    const float* pe_row = p.pe + mb * p.pe_bs + static_cast<int64_t>(mt) * 128;
    for (int hh = 0; hh < 2; ++hh) {
      const int head = (n0 - which * hidden) / 128 + hh;
      const uint32_t tcol = tmem_base + lane_off + ab * kGN + hh * 128;
      float ss = 0.f;
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        tmem_ld32(tcol + c * 32, r);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) ss = fmaf(__uint_as_float(r[i]), __uint_as_float(r[i]), ss);
      }
      const float inv = 1.f / sqrtf(ss / 128.f + p.eps);
      for (int half = 0; half < 2; ++half) {
        uint32_t w[32];
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          const int c = half * 2 + cc;
          uint32_t r[32];
          tmem_ld32(tcol + c * 32, r);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; i += 2) {
            const int d = c * 32 + 2 * i;  // 2 RoPE pairs: d, d+1 and d+2, d+3
            const float4 cs = m < p.M ? *reinterpret_cast<const float4*>(pe_row + d)
                                      : make_float4(0.f, 0.f, 0.f, 0.f);
            const float4 wv = *reinterpret_cast<const float4*>(wn + d);
            const float x0 = __uint_as_float(r[2 * i]) * inv * wv.x;
            const float x1 = __uint_as_float(r[2 * i + 1]) * inv * wv.y;
            const float x2 = __uint_as_float(r[2 * i + 2]) * inv * wv.z;
            const float x3 = __uint_as_float(r[2 * i + 3]) * inv * wv.w;
            w[cc * 16 + i] = gemm_pack_bf16x2(x0 * cs.x - x1 * cs.y, x0 * cs.y + x1 * cs.x);
            w[cc * 16 + i + 1] = gemm_pack_bf16x2(x2 * cs.z - x3 * cs.w, x2 * cs.w + x3 * cs.z);
          }
        }
        uint4* st4 = reinterpret_cast<uint4*>(stage_tile) + trow * 8;
#pragma unroll
        for (int j = 0; j < 8; ++j)
          st4[j ^ (trow & 7)] = make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
        __syncwarp();
#pragma unroll
        for (int pass = 0; pass < 8; ++pass) {
          const int rr = q * 32 + pass * 4 + (lane >> 3);
          const int mm = m0 + rr;
          const uint4 v = reinterpret_cast<const uint4*>(stage_tile)[rr * 8 + (sub ^ (rr & 7))];
          if (mm < p.M) {
            const int bb = mm / p.tokens, tt = mm - bb * p.tokens;
            const int64_t row = (static_cast<int64_t>(bb) * p.heads + head) * p.tokens + tt;
            *reinterpret_cast<uint4*>(dst_base + row * 128 + half * 64 + sub * 8) = v;
          }
        }
        __syncwarp();
      }
    }
  } else if (p.mode == B200_GEMM_RED_F32) {
    // f32 red-add: 32 columns per pass, 4 f32 (16 bytes) per lane.
    for (int c = 0; c < kGN / kEpiChunk; ++c) {
      const int col0 = n0 + c * kEpiChunk;
      if (col0 >= p.N) break;  // same for every thread of the tile
      uint32_t r[32];
      tmem_ld32(tmem_base + lane_off + ab * kGN + c * kEpiChunk, r);
      tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 8; ++j)
        st_row[j ^ (trow & 7)] = make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                             __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
      __syncwarp();
      // This warp's 32 rows, 4 per pass: lane -> row (lane / 8), chunk (lane % 8).
#pragma unroll
      for (int pass = 0; pass < 8; ++pass) {
        const int rr = q * 32 + pass * 4 + (lane >> 3);
        const int m = m0 + rr;
        const float4 v =
            reinterpret_cast<const float4*>(stage_tile)[rr * 8 + (sub ^ (rr & 7))];
        if (m < p.M)
          red_add_v4(static_cast<float*>(p.C) + static_cast<int64_t>(m) * p.ldc + col0 + sub * 4,
                     v.x, v.y, v.z, v.w);
      }
      __syncwarp();
    }
  } else {
    // bf16 store / scatter: 64 columns per pass (two TMEM loads), 8 bf16 (16 bytes) per
    // lane, so each row leaves as one 128-byte segment.
    for (int c = 0; c < kGN / 64; ++c) {
      const int col0 = n0 + c * 64;
      if (col0 >= p.N) break;  // same for every thread of the tile
      const bool two = col0 + 32 < p.N;
      uint32_t r[32], w[32];
      tmem_ld32(tmem_base + lane_off + ab * kGN + c * 64, r);
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 16; ++i) w[i] = gemm_pack_bf16x2(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
      if (two) {
        tmem_ld32(tmem_base + lane_off + ab * kGN + c * 64 + 32, r);
        tmem_wait_ld();
      }
#pragma unroll
      for (int i = 0; i < 16; ++i)
        w[16 + i] = two ? gemm_pack_bf16x2(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1])) : 0u;
      uint4* st4 = reinterpret_cast<uint4*>(stage_tile) + trow * 8;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        st4[j ^ (trow & 7)] = make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
      __syncwarp();
#pragma unroll
      for (int pass = 0; pass < 8; ++pass) {
        const int rr = q * 32 + pass * 4 + (lane >> 3);
        const int m = m0 + rr;
        const uint4 v = reinterpret_cast<const uint4*>(stage_tile)[rr * 8 + (sub ^ (rr & 7))];
        const int col = col0 + sub * 8;
        if (m < p.M && col < p.N) {
          __nv_bfloat16* dst;
          if (p.mode == B200_GEMM_STORE_BF16) {
            dst = static_cast<__nv_bfloat16*>(p.C) + static_cast<int64_t>(m) * p.ldc + col;
          } else if (p.mode == B200_GEMM_QKV) {  // V: token-major [B, T, H * 128]
            dst = static_cast<__nv_bfloat16*>(p.v_out) + static_cast<int64_t>(m) * hidden +
                  (col - 2 * hidden);
          } else {  // scatter: the owner's slot for this rank, over NVLink for others
            const int owner = m / p.rows_per_owner;
            const int64_t row = static_cast<int64_t>(p.src_slot) * p.rows_per_owner + (m - owner * p.rows_per_owner);
            dst = static_cast<__nv_bfloat16*>(p.peers[owner]) + row * p.ldc + col;
          }
          *reinterpret_cast<uint4*>(dst) = v;
        }
      }
      __syncwarp();
    }
  }
}

__global__ void __launch_bounds__(kGThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                const GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  float* stage_tile = reinterpret_cast<float*>(smem + kStageSmem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kGBarOff);
  uint64_t* full = bars;                    // [kGStages]
  uint64_t* empty = bars + kGStages;        // [kGStages]
  uint64_t* acc_full = bars + 2 * kGStages; // [2]
  uint64_t* acc_empty = acc_full + 2;       // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(acc_empty + 3);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nk = (p.K + kGK - 1) / kGK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kGStages; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(acc_full + b, 1);
      mbar_init(acc_empty + b, 4 * 32);
    }
    *abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async();
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, kGTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_a);
      tma_prefetch_desc(&tm_b);
      uint32_t it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.tiles && ok; tile += gridDim.x) {
        int m0, n0;
        tile_coords(p, tile, m0, n0);
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % kGStages;
          const uint32_t ph = (it / kGStages) & 1;
          if (!mbar_wait(empty + s, ph ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + s * kStageBytes;
          mbar_expect_tx(full + s, kStageBytes);
          tma_load_2d(sa, &tm_a, full + s, kb * kGK, m0);
          tma_load_2d(sa + kATileBytes, &tm_b, full + s, kb * kGK, n0);
        }
      }
      if (!ok) {
        gemm_error(p, abort_flag, 1);
        // Let issued copies land before the shared memory is released.
        for (int s = 0; s < kGStages; ++s) mbar_wait(full + s, 0);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(kGM, kGN, 0, 0);
      const uint64_t d0 = smem_desc(smem_addr(smem), 16, 1024);
      const uint32_t hi = static_cast<uint32_t>(d0 >> 32);
      const uint32_t lo0 = static_cast<uint32_t>(d0);
      uint32_t it = 0;
      int lt = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.tiles && ok; tile += gridDim.x, ++lt) {
        const int ab = lt & 1;
        const uint32_t aph = (lt >> 1) & 1;
        if (!mbar_wait(acc_empty + ab, aph ^ 1, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + ab * kGN;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % kGStages;
          const uint32_t ph = (it / kGStages) & 1;
          if (!mbar_wait(full + s, ph, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a = lo0 + ((s * kStageBytes) >> 4);
          const uint32_t b = a + (kATileBytes >> 4);
          // K step kk: 16 columns = 32 bytes further inside the 128-byte swizzle span
          mma_ss_off<0, 0>(d, a, hi, b, hi, idesc, kb > 0 ? 1u : 0u);
          mma_ss_off<2, 2>(d, a, hi, b, hi, idesc, 1u);
          mma_ss_off<4, 4>(d, a, hi, b, hi, idesc, 1u);
          mma_ss_off<6, 6>(d, a, hi, b, hi, idesc, 1u);
          mma_commit(empty + s);
        }
        if (!ok) break;
        mma_commit(acc_full + ab);
      }
      if (!ok) gemm_error(p, abort_flag, 2);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------------ epilogue
    const int q = warp & 3;                 // TMEM lane quadrant of this warp
    const int trow = q * 32 + lane;         // this thread's row of the tile
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    int lt = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < p.tiles; tile += gridDim.x, ++lt) {
      const int ab = lt & 1;
      const uint32_t aph = (lt >> 1) & 1;
      if (!mbar_wait(acc_full + ab, aph, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      int m0, n0;
      tile_coords(p, tile, m0, n0);
      epilogue_tile(p, tmem_base, lane_off, ab, m0, n0, q, lane, trow, stage_tile);
      tc_fence_before();
      mbar_arrive(acc_empty + ab);
    }
    if (!ok) gemm_error(p, abort_flag, 3);
    // Writes into other GPUs' memory are performed at system scope before the CTA exits,
    // so a barrier after the kernel orders every GPU's reads after them.
    if (p.mode != B200_GEMM_STORE_BF16) __threadfence_system();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kGTmemCols);
  }
}

// ------------------------------------------------------------------ CTA-pair variant
// Two CTAs of a cluster compute one 256 x 256 tile with tcgen05.mma.cta_group::2: each CTA
// loads its 128 rows of A and its 128 rows of B (the pair shares B through the tensor
// cores), so a CTA moves 32 KiB per 64-deep K step instead of 48 KiB, and the ring holds 6
// steps.  CTA 0 issues the MMAs; both CTAs' TMA bytes land on CTA 0's `full` barriers;
// commits reach both CTAs' barriers; each CTA's epilogue reads its own 128 rows of the
// accumulator from its TMEM and arrives once on CTA 0's `acc_empty`.
constexpr int kG2Stages = 6;
constexpr int kHalfTileBytes = 128 * kGK * 2;                // 16 KiB: 128 rows x 64
constexpr int kStage2Bytes = 2 * kHalfTileBytes;             // A half + B half
constexpr int kStage2Smem = kG2Stages * kStage2Bytes;        // 192 KiB
constexpr int kG2BarOff = kStage2Smem + kEpiSmem;
constexpr int kG2SmemBytes = kG2BarOff + 256 + 1024;

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Every thread of both CTAs; release / acquire orders shared-memory writes across the pair.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// 2-D tiled load into this CTA's shared memory whose completion bytes count on the
// leader CTA's barrier at the same offset (the peer bit of the address cleared).  No
// multicast.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint64_t* bar,
                                                 int32_t c0, int32_t c1) {
  const uint32_t mbar = smem_addr(bar) & 0xFEFFFFFFu;
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(mbar), "r"(c0), "r"(c1)
      : "memory");
}

template <uint32_t kOffA, uint32_t kOffB>
__device__ __forceinline__ void mma_pair_ss_off(uint32_t d_tmem, uint32_t a_lo, uint32_t a_hi,
                                                uint32_t b_lo, uint32_t b_hi, uint32_t idesc,
                                                uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b32 la, lb;\n\t.reg .b64 da, db;\n\t"
      "add.u32 la, %1, %7;\n\tadd.u32 lb, %3, %8;\n\t"
      "mov.b64 da, {la, %2};\n\tmov.b64 db, {lb, %4};\n\t"
      "setp.ne.b32 p, %6, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], da, db, %5, p;\n\t}" ::"r"(d_tmem),
      "r"(a_lo), "r"(a_hi), "r"(b_lo), "r"(b_hi), "r"(idesc), "r"(accumulate), "n"(kOffA),
      "n"(kOffB)
      : "memory");
}

// Arrive once on the barrier at this offset in both CTAs of the pair when every tcgen05
// operation issued so far is done.
__device__ __forceinline__ void mma_commit_pair(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(smem_addr(bar)),
      "h"(static_cast<uint16_t>(3))
      : "memory");
}

// Arrive on the barrier at this offset in CTA `cta` of the cluster.
__device__ __forceinline__ void mbar_arrive_remote(uint64_t* bar, uint32_t cta) {
  asm volatile(
      "{\n\t.reg .b32 ra;\n\tmapa.shared::cluster.u32 ra, %0, %1;\n\t"
      "mbarrier.arrive.release.cluster.shared::cluster.b64 _, [ra];\n\t}" ::"r"(smem_addr(bar)),
      "r"(cta)
      : "memory");
}

__device__ __forceinline__ void epilogue_barrier() {
  asm volatile("bar.sync 1, 128;" ::: "memory");
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kGThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tm_a,
                     const __grid_constant__ CUtensorMap tm_b, const GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  float* stage_tile = reinterpret_cast<float*>(smem + kStage2Smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kG2BarOff);
  uint64_t* full = bars;                      // [kG2Stages], used in CTA 0
  uint64_t* empty = bars + kG2Stages;         // [kG2Stages]
  uint64_t* acc_full = bars + 2 * kG2Stages;  // [2]
  uint64_t* acc_empty = acc_full + 2;         // [2], used in CTA 0
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(acc_empty + 3);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int pair = blockIdx.x >> 1;
  const int npairs = gridDim.x >> 1;
  const int nk = (p.K + kGK - 1) / kGK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kG2Stages; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(acc_full + b, 1);
      mbar_init(acc_empty + b, 2);  // one arrival per CTA of the pair
    }
    *abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async();
  }
  if (warp == 2) {
    tmem_alloc_pair(tmem_slot, kGTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers and TMEM are ready before any cross-CTA traffic
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_a);
      tma_prefetch_desc(&tm_b);
      uint32_t it = 0;
      bool ok = true;
      for (int tile = pair; tile < p.tiles && ok; tile += npairs) {
        int m0, n0;
        tile_coords(p, tile, m0, n0);
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % kG2Stages;
          const uint32_t ph = (it / kG2Stages) & 1;
          if (!mbar_wait(empty + s, ph ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + s * kStage2Bytes;
          if (rank == 0) mbar_expect_tx(full + s, 2 * kStage2Bytes);
          tma_load_2d_pair(sa, &tm_a, full + s, kb * kGK, m0 + static_cast<int>(rank) * 128);
          tma_load_2d_pair(sa + kHalfTileBytes, &tm_b, full + s, kb * kGK,
                           n0 + static_cast<int>(rank) * 128);
        }
      }
      if (!ok) {
        gemm_error(p, abort_flag, 1);
        if (rank == 0)  // let issued copies land before shared memory is released
          for (int s = 0; s < kG2Stages; ++s) mbar_wait(full + s, 0);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer (CTA 0)
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(2 * kGM, kGN, 0, 0);
      const uint64_t d0 = smem_desc(smem_addr(smem), 16, 1024);
      const uint32_t hi = static_cast<uint32_t>(d0 >> 32);
      const uint32_t lo0 = static_cast<uint32_t>(d0);
      uint32_t it = 0;
      int lt = 0;
      bool ok = true;
      for (int tile = pair; tile < p.tiles && ok; tile += npairs, ++lt) {
        const int ab = lt & 1;
        const uint32_t aph = (lt >> 1) & 1;
        if (!mbar_wait(acc_empty + ab, aph ^ 1, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + ab * kGN;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % kG2Stages;
          const uint32_t ph = (it / kG2Stages) & 1;
          if (!mbar_wait(full + s, ph, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a = lo0 + ((s * kStage2Bytes) >> 4);
          const uint32_t b = a + (kHalfTileBytes >> 4);
          mma_pair_ss_off<0, 0>(d, a, hi, b, hi, idesc, kb > 0 ? 1u : 0u);
          mma_pair_ss_off<2, 2>(d, a, hi, b, hi, idesc, 1u);
          mma_pair_ss_off<4, 4>(d, a, hi, b, hi, idesc, 1u);
          mma_pair_ss_off<6, 6>(d, a, hi, b, hi, idesc, 1u);
          mma_commit_pair(empty + s);
        }
        if (!ok) break;
        mma_commit_pair(acc_full + ab);
      }
      if (!ok) gemm_error(p, abort_flag, 2);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int trow = q * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    int lt = 0;
    bool ok = true;
    for (int tile = pair; tile < p.tiles; tile += npairs, ++lt) {
      const int ab = lt & 1;
      const uint32_t aph = (lt >> 1) & 1;
      if (!mbar_wait(acc_full + ab, aph, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      int m0, n0;
      tile_coords(p, tile, m0, n0);
      epilogue_tile(p, tmem_base, lane_off, ab, m0 + static_cast<int>(rank) * 128, n0, q, lane,
                    trow, stage_tile);
      tc_fence_before();
      epilogue_barrier();  // all 128 rows of this CTA read
      if (threadIdx.x == 4 * 32) {
        if (rank == 0) mbar_arrive(acc_empty + ab);
        else mbar_arrive_remote(acc_empty + ab, 0);
      }
    }
    if (!ok) gemm_error(p, abort_flag, 3);
    if (p.mode != B200_GEMM_STORE_BF16) __threadfence_system();
  }

  tc_fence_before();
  cluster_sync();  // neither CTA leaves while the other may still signal its barriers
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kGTmemCols);
  }
}

// ------------------------------------------------------------------ host side
PFN_cuTensorMapEncodeTiled_v12000 gemm_encode_fn() {
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

// 2-D map over a bf16 row-major matrix [rows, cols] with `ld` elements between rows; box
// 64 columns x box_rows rows, 128-byte swizzle, zero fill outside.
int make_map_2d(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t ld,
                uint32_t box_rows) {
  auto fn = gemm_encode_fn();
  if (!fn) return B200_ERR_CUDA;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kGK), box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? B200_OK : B200_ERR_CUDA;
}

int gemm_sms() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

int ensure_gemm_attrs() {
  static std::mutex mu;
  static int done_dev = -1;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return B200_ERR_CUDA;
  std::lock_guard<std::mutex> lock(mu);
  if (done_dev == dev) return B200_OK;
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  if (major != 10 || minor != 0) return B200_ERR_UNSUPPORTED;
  if (cudaFuncSetAttribute(gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           kGSmemBytes) != cudaSuccess ||
      cudaFuncSetAttribute(gemm_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           kG2SmemBytes) != cudaSuccess)
    return B200_ERR_CUDA;
  done_dev = dev;
  return B200_OK;
}

inline bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// CTA-pair (256-row) tiles from 512 rows up; B200_GEMM_PAIR=0 / 1 forces one-CTA / pair
// tiles (for comparisons).
bool use_pair_tiles(int32_t m) {
  static const int forced = [] {
    const char* e = std::getenv("B200_GEMM_PAIR");
    return e ? (e[0] == '1' ? 1 : 0) : -1;
  }();
  if (forced >= 0) return forced == 1;
  return m >= 512;
}

}  // namespace
}  // namespace b200

using namespace b200;

namespace b200 {
namespace {

struct QkvArgs {
  int32_t heads, tokens;
  const float* pe;
  int64_t pe_bs;
  const float* norm_q;
  const float* norm_k;
  float eps;
  void* q_out;
  void* k_out;
  void* v_out;
};

int launch_gemm(const void* a, int64_t lda, const void* b, int64_t ldb, void* c, int64_t ldc,
                int32_t m, int32_t n, int32_t k, int32_t mode, int32_t* status,
                cudaStream_t stream, void* const* peers, int32_t n_owners,
                int32_t rows_per_owner, int32_t src_slot, const QkvArgs* qkv = nullptr);

}  // namespace
}  // namespace b200

extern "C" int b200_gemm(const void* a, int64_t lda, const void* b, int64_t ldb, void* c,
                         int64_t ldc, int32_t m, int32_t n, int32_t k, int32_t mode,
                         int32_t* status, b200_stream_t stream) {
  if (mode != B200_GEMM_STORE_BF16 && mode != B200_GEMM_RED_F32) return B200_ERR_INVALID;
  return launch_gemm(a, lda, b, ldb, c, ldc, m, n, k, mode, status,
                     static_cast<cudaStream_t>(stream), nullptr, 0, 0, 0);
}

extern "C" int b200_qkv_norm_rope_gemm(const void* x, int64_t ldx, const void* w_qkv,
                                       int32_t batch, int32_t tokens, int32_t heads,
                                       int32_t in_features, const float* norm_q_w,
                                       const float* norm_k_w, float eps, const float* pe,
                                       int64_t pe_batch_stride, void* q_rot, void* k_rot,
                                       void* v, int32_t* status, b200_stream_t stream) {
  if (batch <= 0 || tokens <= 0 || heads <= 0 || heads % 2 != 0) return B200_ERR_INVALID;
  if (!norm_q_w || !norm_k_w || !pe || !q_rot || !k_rot || !v) return B200_ERR_INVALID;
  const void* ptrs[] = {norm_q_w, norm_k_w, pe, q_rot, k_rot, v};
  for (const void* ptr : ptrs)
    if (reinterpret_cast<uintptr_t>(ptr) & 15u) return B200_ERR_INVALID;
  if (pe_batch_stride < 0 || pe_batch_stride % 4 != 0 || !(eps >= 0.f)) return B200_ERR_INVALID;
  const int64_t m = static_cast<int64_t>(batch) * tokens;
  if (m > 0x7fffffff) return B200_ERR_INVALID;
  QkvArgs qa{heads, tokens, pe, pe_batch_stride, norm_q_w, norm_k_w, eps, q_rot, k_rot, v};
  return launch_gemm(x, ldx, w_qkv, in_features, v, 3 * heads * 128, static_cast<int32_t>(m),
                     3 * heads * 128, in_features, B200_GEMM_QKV, status,
                     static_cast<cudaStream_t>(stream), nullptr, 0, 0, 0, &qa);
}

extern "C" int b200_gemm_scatter(const void* a, int64_t lda, const void* b, int64_t ldb,
                                 void* const* owner_bufs, int32_t n_owners, int32_t src_slot,
                                 int32_t rows_per_owner, int64_t ldc, int32_t m, int32_t n,
                                 int32_t k, int32_t* status, b200_stream_t stream) {
  if (!owner_bufs || n_owners < 1 || n_owners > kMaxOwners) return B200_ERR_INVALID;
  if (src_slot < 0 || src_slot >= n_owners || rows_per_owner <= 0) return B200_ERR_INVALID;
  if (static_cast<int64_t>(rows_per_owner) * n_owners < m) return B200_ERR_INVALID;
  for (int i = 0; i < n_owners; ++i)
    if (!owner_bufs[i] || (reinterpret_cast<uintptr_t>(owner_bufs[i]) & 15u)) return B200_ERR_INVALID;
  return launch_gemm(a, lda, b, ldb, owner_bufs[0], ldc, m, n, k, B200_GEMM_SCATTER_BF16, status,
                     static_cast<cudaStream_t>(stream), owner_bufs, n_owners, rows_per_owner,
                     src_slot);
}

namespace b200 {
namespace {

int launch_gemm(const void* a, int64_t lda, const void* b, int64_t ldb, void* c, int64_t ldc,
                int32_t m, int32_t n, int32_t k, int32_t mode, int32_t* status,
                cudaStream_t stream, void* const* peers, int32_t n_owners,
                int32_t rows_per_owner, int32_t src_slot, const QkvArgs* qkv) {
  if (m < 0 || n < 0 || k < 0) return B200_ERR_INVALID;
  if (m == 0 || n == 0) return B200_OK;
  if (!a || !b || !c || !al16(a) || !al16(b) || !al16(c)) return B200_ERR_INVALID;
  // TMA: 16-byte row strides; epilogue: 32-column chunks, 8- (bf16) or 16-byte vectors.
  if (k == 0 || k % 8 != 0 || lda < k || ldb < k || lda % 8 != 0 || ldb % 8 != 0)
    return B200_ERR_INVALID;
  if (n % 32 != 0 || ldc < n || ldc % 8 != 0) return B200_ERR_INVALID;
  int rc = ensure_gemm_attrs();
  if (rc != B200_OK) return rc;
  const bool pair = use_pair_tiles(m);
  CUtensorMap ma{}, mb{};
  if ((rc = make_map_2d(&ma, a, m, k, lda, kGM)) != B200_OK) return rc;
  if ((rc = make_map_2d(&mb, b, n, k, ldb, pair ? kGN / 2 : kGN)) != B200_OK) return rc;
  GemmParams p{};
  p.M = m;
  p.N = n;
  p.K = k;
  p.tile_m = pair ? 2 * kGM : kGM;
  p.tiles_n = (n + kGN - 1) / kGN;
  p.tiles_m = (m + p.tile_m - 1) / p.tile_m;
  {  // A rows of one raster group: about 64 MiB (half of L2)
    const int64_t rows_bytes = static_cast<int64_t>(p.tile_m) * k * 2;
    const int64_t g = (int64_t{64} << 20) / rows_bytes;
    p.group_m = static_cast<int32_t>(g < 1 ? 1 : (g > p.tiles_m ? p.tiles_m : g));
  }
  const int64_t tiles = static_cast<int64_t>(p.tiles_m) * p.tiles_n;
  if (tiles > 0x7fffffff) return B200_ERR_INVALID;
  p.tiles = static_cast<int32_t>(tiles);
  p.mode = mode;
  p.ldc = ldc;
  p.C = c;
  p.status = status;
  for (int i = 0; i < n_owners; ++i) p.peers[i] = peers[i];
  p.rows_per_owner = rows_per_owner;
  p.src_slot = src_slot;
  if (qkv) {
    p.heads = qkv->heads;
    p.tokens = qkv->tokens;
    p.pe = qkv->pe;
    p.pe_bs = qkv->pe_bs;
    p.norm_q = qkv->norm_q;
    p.norm_k = qkv->norm_k;
    p.eps = qkv->eps;
    p.q_out = qkv->q_out;
    p.k_out = qkv->k_out;
    p.v_out = qkv->v_out;
  } else {
    p.heads = 1;  // unused outside B200_GEMM_QKV
    p.tokens = 1;
  }
  if (pair) {
    const int pairs = gemm_sms() / 2;
    const int grid = 2 * static_cast<int>(tiles < pairs ? tiles : pairs);
    gemm_pair_kernel<<<grid, kGThreads, kG2SmemBytes, stream>>>(ma, mb, p);
  } else {
    const int grid = static_cast<int>(tiles < gemm_sms() ? tiles : gemm_sms());
    gemm_kernel<<<grid, kGThreads, kGSmemBytes, stream>>>(ma, mb, p);
  }
  return cudaGetLastError() == cudaSuccess ? B200_OK : B200_ERR_CUDA;
}

// Sum of a row block's slots, broadcast as bf16: thread -> 8 columns of one row.
__global__ void __launch_bounds__(256) reduce_gather_kernel(const uint4* slots, int32_t n_src,
                                                            int32_t rows, int32_t c8,
                                                            int64_t ld8, int64_t slot_stride8,
                                                            ReduceGatherDst dst) {
  const int64_t total = static_cast<int64_t>(rows) * c8;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / c8;
    const int c = static_cast<int>(i - r * c8);
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int s = 0; s < n_src; ++s) {  // fixed order: the sum does not depend on timing
      const uint4 u = slots[s * slot_stride8 + r * ld8 + c];
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        acc[2 * e] += __uint_as_float(w[e] << 16);
        acc[2 * e + 1] += __uint_as_float(w[e] & 0xffff0000u);
      }
    }
    uint4 o;
    uint32_t ow[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      __nv_bfloat162 v = __floats2bfloat162_rn(acc[2 * e], acc[2 * e + 1]);
      ow[e] = *reinterpret_cast<uint32_t*>(&v);
    }
    o = make_uint4(ow[0], ow[1], ow[2], ow[3]);
    const int64_t drow = dst.row0 + r;
    for (int d = 0; d < dst.n; ++d) static_cast<uint4*>(dst.ptr[d])[drow * dst.ld8 + c] = o;
  }
  __threadfence_system();
}

// The owner's step of the head-sharded block with the gated residual and the next
// LayerNorm fused in (one CTA per row, 256 threads, columns in 8-element groups):
//   sum   = sum over s of slots[s][r, :]              (bf16 partials, f32, fixed order)
//   x[r]  = x[r] + tanh(gate[m]) * sum                (f32, in place: the owner's rows)
//   y     = LN(x[r]) * (1 + scale[m])                 (bf16, written to every dst buffer)
// with m = (row0 + r) / rows_per_mod the row's modulation row.  kNG = groups per thread.
constexpr int kRrThreads = 256;

__device__ __forceinline__ float rr_block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();  // red[] is reused by consecutive reductions
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < kRrThreads / 32; ++w) t += red[w];
  return t;
}

template <int kNG>
__global__ void __launch_bounds__(kRrThreads) reduce_residual_adaln_gather_kernel(
    const uint4* slots, int32_t n_src, int32_t rows, int32_t c8, int64_t ld8,
    int64_t slot_stride8, float* x, int64_t ldx, const float* gate, const float* scale,
    int64_t rows_per_mod, int64_t mod_stride, float eps, ReduceGatherDst dst) {
  __shared__ float red[kRrThreads / 32];
  const float inv_n = 1.f / static_cast<float>(c8 * 8);
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const int64_t m = (dst.row0 + r) / rows_per_mod;
    float xv[kNG][8];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < kNG; ++i) {
      const int c = threadIdx.x + i * kRrThreads;
      if (c < c8) {
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int k = 0; k < n_src; ++k) {  // fixed order: the sum does not depend on timing
          const uint4 u = slots[k * slot_stride8 + r * ld8 + c];
          const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            acc[2 * e] += __uint_as_float(w[e] << 16);
            acc[2 * e + 1] += __uint_as_float(w[e] & 0xffff0000u);
          }
        }
        float4* xr = reinterpret_cast<float4*>(x + r * ldx + c * 8);
        const float4* gr = reinterpret_cast<const float4*>(gate + m * mod_stride + c * 8);
        const float4 x0 = xr[0], x1 = xr[1], g0 = gr[0], g1 = gr[1];
        const float xs[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
        const float gs[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          xv[i][e] = fmaf(tanhf(gs[e]), acc[e], xs[e]);
          s += xv[i][e];
        }
        xr[0] = make_float4(xv[i][0], xv[i][1], xv[i][2], xv[i][3]);
        xr[1] = make_float4(xv[i][4], xv[i][5], xv[i][6], xv[i][7]);
      }
    }
    const float mean = rr_block_sum(s, red) * inv_n;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < kNG; ++i) {
      const int c = threadIdx.x + i * kRrThreads;
      if (c < c8) {
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float d = xv[i][e] - mean;
          q += d * d;
        }
      }
    }
    const float rstd = rsqrtf(rr_block_sum(q, red) * inv_n + eps);
#pragma unroll
    for (int i = 0; i < kNG; ++i) {
      const int c = threadIdx.x + i * kRrThreads;
      if (c < c8) {
        const float4* sr = reinterpret_cast<const float4*>(scale + m * mod_stride + c * 8);
        const float4 s0 = sr[0], s1 = sr[1];
        const float ss[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
        uint32_t ow[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float a = (xv[i][2 * e] - mean) * rstd * (1.f + ss[2 * e]);
          const float b = (xv[i][2 * e + 1] - mean) * rstd * (1.f + ss[2 * e + 1]);
          __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
          ow[e] = *reinterpret_cast<uint32_t*>(&v);
        }
        const uint4 o = make_uint4(ow[0], ow[1], ow[2], ow[3]);
        const int64_t drow = dst.row0 + r;
        for (int d = 0; d < dst.n; ++d) static_cast<uint4*>(dst.ptr[d])[drow * dst.ld8 + c] = o;
      }
    }
  }
  __threadfence_system();
}

// The owner's step with the reduction in the NVSwitch (NVLS): every rank's full partial
// sits in its own buffer, bound with the others to one CUDA multicast object; the owner
// reads its rows through the multicast address with multimem.ld_reduce (the switch adds
// the N ranks' bf16 values, accumulating in f32, and returns the sum rounded to bf16
// once), applies the optional residual and norm2 exactly as
// reduce_residual_adaln_gather_kernel does, and writes each result row once with
// multimem.st to the output's multicast address, which lands it in every rank's buffer.
// Per GPU the links carry its partial out once and the other owners' rows in once,
// (1 + 1/N) x the partial each way, against 2 (N-1)/N x for peer stores.
__device__ __forceinline__ uint4 mc_ld_reduce_bf16x8(const void* addr) {
  uint4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(addr)
               : "memory");
  return v;
}

__device__ __forceinline__ void mc_st_16b(void* addr, const uint4& v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr),
               "f"(__uint_as_float(v.x)), "f"(__uint_as_float(v.y)), "f"(__uint_as_float(v.z)),
               "f"(__uint_as_float(v.w))
               : "memory");
}

struct NvlsArgs {
  const uint4* mc_part;  // multicast address of the partial buffers, 8 bf16 per uint4
  uint4* mc_out;         // multicast address of the output buffers
  int64_t row0, part_ld8, out_ld8;
  int32_t rows, c8;
  float* x;              // this owner's f32 rows, or null: no residual / norm
  int64_t ldx;
  const float* gate;
  const float* scale;
  int64_t rows_per_mod, mod_stride;
  float eps;
};

template <int kNG>
__global__ void __launch_bounds__(kRrThreads) reduce_nvls_kernel(const NvlsArgs a) {
  __shared__ float red[kRrThreads / 32];
  const float inv_n = 1.f / static_cast<float>(a.c8 * 8);
  for (int64_t r = blockIdx.x; r < a.rows; r += gridDim.x) {
    const int64_t grow = a.row0 + r;
    uint4 sum[kNG];
#pragma unroll
    for (int i = 0; i < kNG; ++i) {
      const int c = threadIdx.x + i * kRrThreads;
      if (c < a.c8) sum[i] = mc_ld_reduce_bf16x8(a.mc_part + grow * a.part_ld8 + c);
    }
    if (!a.x) {  // the sum alone, broadcast
#pragma unroll
      for (int i = 0; i < kNG; ++i) {
        const int c = threadIdx.x + i * kRrThreads;
        if (c < a.c8) mc_st_16b(a.mc_out + grow * a.out_ld8 + c, sum[i]);
      }
      continue;  // uniform over the CTA
    }
    const int64_t m = grow / a.rows_per_mod;
    float xv[kNG][8];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < kNG; ++i) {
      const int c = threadIdx.x + i * kRrThreads;
      if (c < a.c8) {
        const uint32_t w[4] = {sum[i].x, sum[i].y, sum[i].z, sum[i].w};
        float4* xr = reinterpret_cast<float4*>(a.x + r * a.ldx + c * 8);
        const float4* gr = reinterpret_cast<const float4*>(a.gate + m * a.mod_stride + c * 8);
        const float4 x0 = xr[0], x1 = xr[1], g0 = gr[0], g1 = gr[1];
        const float xs[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
        const float gs[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float y = __uint_as_float((e & 1) ? (w[e >> 1] & 0xffff0000u) : (w[e >> 1] << 16));
          xv[i][e] = fmaf(tanhf(gs[e]), y, xs[e]);
          s += xv[i][e];
        }
        xr[0] = make_float4(xv[i][0], xv[i][1], xv[i][2], xv[i][3]);
        xr[1] = make_float4(xv[i][4], xv[i][5], xv[i][6], xv[i][7]);
      }
    }
    const float mean = rr_block_sum(s, red) * inv_n;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < kNG; ++i) {
      const int c = threadIdx.x + i * kRrThreads;
      if (c < a.c8) {
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float d = xv[i][e] - mean;
          q += d * d;
        }
      }
    }
    const float rstd = rsqrtf(rr_block_sum(q, red) * inv_n + a.eps);
#pragma unroll
    for (int i = 0; i < kNG; ++i) {
      const int c = threadIdx.x + i * kRrThreads;
      if (c < a.c8) {
        const float4* sr = reinterpret_cast<const float4*>(a.scale + m * a.mod_stride + c * 8);
        const float4 s0 = sr[0], s1 = sr[1];
        const float ss[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
        uint32_t ow[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          __nv_bfloat162 v = __floats2bfloat162_rn((xv[i][2 * e] - mean) * rstd * (1.f + ss[2 * e]),
                                                   (xv[i][2 * e + 1] - mean) * rstd * (1.f + ss[2 * e + 1]));
          ow[e] = *reinterpret_cast<uint32_t*>(&v);
        }
        mc_st_16b(a.mc_out + grow * a.out_ld8 + c, make_uint4(ow[0], ow[1], ow[2], ow[3]));
      }
    }
  }
  asm volatile("fence.proxy.alias;" ::: "memory");
  __threadfence_system();
}

}  // namespace
}  // namespace b200

extern "C" int b200_reduce_nvls(const void* mc_part, int64_t part_ld, void* mc_out,
                                int64_t out_ld, int64_t row0, int32_t rows, int32_t cols,
                                float* x, int64_t ldx, const float* gate, const float* scale,
                                int64_t rows_per_mod, int64_t mod_stride, float eps,
                                b200_stream_t stream) {
  if (!mc_part || !mc_out || row0 < 0 || rows < 0 || cols <= 0 || cols % 8 != 0 ||
      cols > 8192 || part_ld < cols || part_ld % 8 != 0 || out_ld < cols || out_ld % 8 != 0)
    return B200_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(mc_part) & 15u) || (reinterpret_cast<uintptr_t>(mc_out) & 15u))
    return B200_ERR_INVALID;
  if (x) {
    if (!gate || !scale || ldx < cols || ldx % 4 != 0 || rows_per_mod < 1 || mod_stride < 0 ||
        mod_stride % 4 != 0 || !(eps >= 0.f))
      return B200_ERR_INVALID;
    const void* ptrs[] = {x, gate, scale};
    for (const void* q : ptrs)
      if (reinterpret_cast<uintptr_t>(q) & 15u) return B200_ERR_INVALID;
  }
  if (rows == 0) return B200_OK;
  NvlsArgs a{};
  a.mc_part = static_cast<const uint4*>(mc_part);
  a.mc_out = static_cast<uint4*>(mc_out);
  a.row0 = row0;
  a.part_ld8 = part_ld / 8;
  a.out_ld8 = out_ld / 8;
  a.rows = rows;
  a.c8 = cols / 8;
  a.x = x;
  a.ldx = ldx;
  a.gate = gate;
  a.scale = scale;
  a.rows_per_mod = rows_per_mod < 1 ? 1 : rows_per_mod;
  a.mod_stride = mod_stride;
  a.eps = eps;
  const int64_t cap = static_cast<int64_t>(gemm_sms()) * 8;
  const unsigned grid = static_cast<unsigned>(rows < cap ? rows : cap);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (a.c8 <= kRrThreads)
    reduce_nvls_kernel<1><<<grid, kRrThreads, 0, st>>>(a);
  else if (a.c8 <= 2 * kRrThreads)
    reduce_nvls_kernel<2><<<grid, kRrThreads, 0, st>>>(a);
  else
    reduce_nvls_kernel<4><<<grid, kRrThreads, 0, st>>>(a);
  return cudaGetLastError() == cudaSuccess ? B200_OK : B200_ERR_CUDA;
}

extern "C" int b200_reduce_residual_adaln_gather(
    const void* slots, int32_t n_src, int32_t slot_rows, int32_t rows, int32_t cols, int64_t ld,
    float* x, int64_t ldx, const float* gate, const float* scale, int64_t rows_per_mod,
    int64_t mod_stride, float eps, void* const* dst_bufs, int32_t n_dst, int64_t dst_row0,
    int64_t dst_ld, b200_stream_t stream) {
  if (!slots || n_src < 1 || rows < 0 || slot_rows < rows || cols <= 0 || cols % 8 != 0 ||
      cols > 8192 || ld < cols || ld % 8 != 0)
    return B200_ERR_INVALID;
  if (!x || !gate || !scale || ldx < cols || ldx % 4 != 0 || rows_per_mod < 1 ||
      mod_stride < 0 || mod_stride % 4 != 0 || !(eps >= 0.f))
    return B200_ERR_INVALID;
  if (!dst_bufs || n_dst < 1 || n_dst > kMaxOwners || dst_row0 < 0 || dst_ld < cols || dst_ld % 8 != 0)
    return B200_ERR_INVALID;
  const void* ptrs[] = {slots, x, gate, scale};
  for (const void* q : ptrs)
    if (reinterpret_cast<uintptr_t>(q) & 15u) return B200_ERR_INVALID;
  ReduceGatherDst dst{};
  for (int i = 0; i < n_dst; ++i) {
    if (!dst_bufs[i] || (reinterpret_cast<uintptr_t>(dst_bufs[i]) & 15u)) return B200_ERR_INVALID;
    dst.ptr[i] = dst_bufs[i];
  }
  dst.n = n_dst;
  dst.row0 = dst_row0;
  dst.ld8 = dst_ld / 8;
  if (rows == 0) return B200_OK;
  const int64_t cap = static_cast<int64_t>(gemm_sms()) * 8;
  const unsigned grid = static_cast<unsigned>(rows < cap ? rows : cap);
  const int c8 = cols / 8;
  const int64_t sstride = static_cast<int64_t>(slot_rows) * (ld / 8);
  auto* sl = static_cast<const uint4*>(slots);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (c8 <= kRrThreads)
    reduce_residual_adaln_gather_kernel<1><<<grid, kRrThreads, 0, st>>>(
        sl, n_src, rows, c8, ld / 8, sstride, x, ldx, gate, scale, rows_per_mod, mod_stride, eps, dst);
  else if (c8 <= 2 * kRrThreads)
    reduce_residual_adaln_gather_kernel<2><<<grid, kRrThreads, 0, st>>>(
        sl, n_src, rows, c8, ld / 8, sstride, x, ldx, gate, scale, rows_per_mod, mod_stride, eps, dst);
  else
    reduce_residual_adaln_gather_kernel<4><<<grid, kRrThreads, 0, st>>>(
        sl, n_src, rows, c8, ld / 8, sstride, x, ldx, gate, scale, rows_per_mod, mod_stride, eps, dst);
  return cudaGetLastError() == cudaSuccess ? B200_OK : B200_ERR_CUDA;
}

extern "C" int b200_reduce_gather_bf16(const void* slots, int32_t n_src, int32_t slot_rows,
                                       int32_t rows, int32_t cols, int64_t ld,
                                       void* const* dst_bufs, int32_t n_dst, int64_t dst_row0,
                                       int64_t dst_ld, b200_stream_t stream) {
  if (!slots || n_src < 1 || rows < 0 || slot_rows < rows || cols <= 0 || cols % 8 != 0 ||
      ld < cols || ld % 8 != 0)
    return B200_ERR_INVALID;
  if (!dst_bufs || n_dst < 1 || n_dst > kMaxOwners || dst_row0 < 0 || dst_ld < cols || dst_ld % 8 != 0)
    return B200_ERR_INVALID;
  if (reinterpret_cast<uintptr_t>(slots) & 15u) return B200_ERR_INVALID;
  ReduceGatherDst dst{};
  for (int i = 0; i < n_dst; ++i) {
    if (!dst_bufs[i] || (reinterpret_cast<uintptr_t>(dst_bufs[i]) & 15u)) return B200_ERR_INVALID;
    dst.ptr[i] = dst_bufs[i];
  }
  dst.n = n_dst;
  dst.row0 = dst_row0;
  dst.ld8 = dst_ld / 8;
  if (rows == 0) return B200_OK;
  const int64_t total = static_cast<int64_t>(rows) * (cols / 8);
  const int64_t want = (total + 255) / 256;
  const int64_t cap = static_cast<int64_t>(gemm_sms()) * 8;
  reduce_gather_kernel<<<static_cast<unsigned>(want < cap ? want : cap), 256, 0,
                         static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(slots), n_src, rows, cols / 8, ld / 8,
      static_cast<int64_t>(slot_rows) * (ld / 8), dst);
  return cudaGetLastError() == cudaSuccess ? B200_OK : B200_ERR_CUDA;
}
