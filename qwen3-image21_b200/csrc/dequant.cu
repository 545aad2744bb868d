// dequant.cu — GGUF k-quant (Q4_K, Q6_K) super-blocks: to bf16, and a fused
// dequantising matrix-vector product for a few rows of activations.
//
// Dequantisation: one warp per 256-weight super-block, one thread per 8 consecutive
// weights: each thread reads its quant bytes, the block's scale bytes and f16
// super-scales (L1 serves the repeats), and writes one 16-byte bf16 vector, so a warp's
// stores are one contiguous 512-byte row segment.  HBM-bound: per weight 144/256 (Q4_K)
// or 210/256 (Q6_K) bytes in and 2 bytes out.
//
// kquant_gemv_kernel: y[m, n] = sum_k x[m, k] W[n, k] for M <= 2 activation rows, the
// weights read once as super-blocks and expanded in registers to the same bf16 values the
// dequantisation writes (candle's QMatMul on a batch of a few rows,
// src/quantized_transformer.rs:20-33: the timestep embedder and the modulation linear
// run at one row per sequence).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/b200_gguf.h"

namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ float half_bits_to_float(uint32_t bits16) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16)));
}

__device__ __forceinline__ uint4 pack8_bf16(const float (&y)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 v = __floats2bfloat162_rn(y[2 * i], y[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t*>(&v);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// Small non-negative integer (< 2^23) to float, exactly, on the FMA/ALU pipes: the bits
// of 2^23 + q minus 2^23 (instead of an integer-to-float conversion per weight).
__device__ __forceinline__ float small_u2f(uint32_t q) {
  return __fsub_rn(__uint_as_float(0x4B000000u | q), 8388608.0f);
}

// Q4_K: bytes 0-1 d, 2-3 dmin, 4-15 scales, 16-143 quants.  Weights 8t .. 8t+7 of the
// super-block at b, as GGML computes them in f32 (each product and difference rounded).
// Sub-block j's 6-bit (scale, min): j < 4: low 6 bits of scale bytes j and j + 4; j >= 4:
// low / high nibble of byte j + 4 with the top 2 bits of bytes j - 4 / j as bits 4-5.
__device__ __forceinline__ void q4k_weights8(const uint8_t* b, const int t, float (&y)[8]) {
  const uint32_t dd = *reinterpret_cast<const uint32_t*>(b);
  const float d = half_bits_to_float(dd & 0xffffu);
  const float dmin = half_bits_to_float(dd >> 16);
  const uint32_t s0 = *reinterpret_cast<const uint32_t*>(b + 4);   // scale bytes 0-3
  const uint32_t s1 = *reinterpret_cast<const uint32_t*>(b + 8);   // 4-7
  const uint32_t s2 = *reinterpret_cast<const uint32_t*>(b + 12);  // 8-11
  const int chunk = t >> 3;          // 64-weight chunk
  const int hi = (t & 7) >= 4;       // high nibbles: the chunk's second 32 weights
  const int l0 = (t & 3) * 8;
  const int is = 2 * chunk + hi;     // sub-block of 32
  const uint32_t sh = 8u * static_cast<uint32_t>(is & 3);
  uint32_t sc, mn;
  if (is < 4) {
    sc = (s0 >> sh) & 63u;
    mn = (s1 >> sh) & 63u;
  } else {
    const uint32_t lohi = (s2 >> sh) & 0xFFu;  // byte is + 4
    sc = (lohi & 0xFu) | (((s0 >> sh) >> 6 & 3u) << 4);
    mn = (lohi >> 4) | (((s1 >> sh) >> 6 & 3u) << 4);
  }
  const float d1 = __fmul_rn(d, small_u2f(sc));
  const float m1 = __fmul_rn(dmin, small_u2f(mn));
  const uint2 q8 = *reinterpret_cast<const uint2*>(b + 16 + 32 * chunk + l0);
  const uint32_t nib = hi ? 4u : 0u;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const uint32_t word = e < 4 ? q8.x : q8.y;
    const uint32_t q = (word >> (8 * (e & 3) + nib)) & 0xFu;
    y[e] = __fsub_rn(__fmul_rn(d1, small_u2f(q)), m1);
  }
}

__global__ void __launch_bounds__(kThreads) dequant_q4k_kernel(const uint8_t* blocks, uint4* out,
                                                               int64_t n_blocks) {
  const int64_t total = n_blocks * 32;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * kThreads) {
    float y[8];
    q4k_weights8(blocks + (i >> 5) * B200_Q4_K_BLOCK_BYTES, static_cast<int>(i & 31), y);
    out[i] = pack8_bf16(y);
  }
}

// Q6_K: bytes 0-127 ql, 128-191 qh, 192-207 int8 scales, 208-209 d.  The block is only
// 2-byte aligned (210 bytes), so bytes are read as 16-bit words.
__device__ __forceinline__ uint32_t load_u16(const uint8_t* p) {
  return *reinterpret_cast<const uint16_t*>(p);
}

// Weights 8t .. 8t+7 of the Q6_K super-block at b, in f32 as GGML computes them.
__device__ __forceinline__ void q6k_weights8(const uint8_t* b, const int t, float (&y)[8]) {
  {
    const int half = t >> 4;           // 128-weight half
    const int w0 = (t & 15) * 8;       // first weight within the half
    const int g = w0 >> 5;             // group of 32 within the half (0..3)
    const int l0 = w0 & 31;
    const uint8_t* ql = b + 64 * half + ((g & 1) ? 32 : 0) + l0;
    const uint8_t* qh = b + 128 + 32 * half + l0;
    const int scale_idx = 8 * half + (l0 >> 4) + 2 * g;
    const float d = half_bits_to_float(load_u16(b + 208));
    const int8_t s8 = static_cast<int8_t>(b[192 + scale_idx]);
    const float ds = __fmul_rn(d, static_cast<float>(s8));
#pragma unroll
    for (int e = 0; e < 8; e += 2) {
      const uint32_t lo2 = load_u16(ql + e);
      const uint32_t hi2 = load_u16(qh + e);
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const uint32_t lbyte = (lo2 >> (8 * k)) & 0xFFu;
        const uint32_t hbyte = (hi2 >> (8 * k)) & 0xFFu;
        const uint32_t lo = (g >= 2) ? (lbyte >> 4) : (lbyte & 0xFu);
        const uint32_t hb = (hbyte >> (2 * g)) & 3u;
        // (lo | hb << 4) - 32 as a float, exactly: (2^23 + q6) - (2^23 + 32)
        y[e + k] = __fmul_rn(ds, __fsub_rn(__uint_as_float(0x4B000000u | lo | (hb << 4)),
                                           8388640.0f));
      }
    }
  }
}

__global__ void __launch_bounds__(kThreads) dequant_q6k_kernel(const uint8_t* blocks, uint4* out,
                                                               int64_t n_blocks) {
  const int64_t total = n_blocks * 32;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * kThreads) {
    float y[8];
    q6k_weights8(blocks + (i >> 5) * B200_Q6_K_BLOCK_BYTES, static_cast<int>(i & 31), y);
    out[i] = pack8_bf16(y);
  }
}

// ---- fused dequantising GEMV
// A CTA of 8 warps owns 32 consecutive output rows n (4 per warp).  K is walked in
// chunks of kGvChunkBlocks super-blocks: all 256 threads copy the chunk's x columns
// (f32) and the 32 rows' super-blocks (one contiguous segment per row) into shared memory
// with coalesced 16-byte loads, so every byte of the weight is fetched from HBM once with
// many loads in flight; then per super-block lane t expands its 8 weights of each of the
// warp's 4 rows from shared memory and applies x[m, 8t .. 8t+7] of every row m.  Weights
// are rounded to bf16 as b200_dequant_* writes them; products and sums in f32 (packed
// f32x2 FMAs over pairs of weights); each (row, m) sum is reduced over the warp with
// shuffles at the end.
constexpr int kGvRowsPerWarp = 4;
constexpr int kGvRowsPerCta = 8 * kGvRowsPerWarp;
constexpr int kGvChunkBlocks = 8;  // super-blocks per K-chunk (2048 columns)

__device__ __forceinline__ uint64_t gv_pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ uint64_t gv_fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ float gv_sum2(uint64_t v) {
  float a, b;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
  return a + b;
}

template <int kQT, int kMT>
__global__ void __launch_bounds__(kThreads) kquant_gemv_kernel(
    const float* __restrict__ x, int64_t ldx, const uint8_t* __restrict__ blocks,
    int64_t row_bytes, float* __restrict__ y, int64_t ldy, int m_rows, int n_rows, int k) {
  constexpr int kBB = kQT == 0 ? B200_Q4_K_BLOCK_BYTES : B200_Q6_K_BLOCK_BYTES;
  constexpr int kSegMax = kGvChunkBlocks * kBB;          // one row's bytes per chunk
  constexpr int kWBytes = (kGvRowsPerCta * kSegMax + 15) / 16 * 16;
  extern __shared__ __align__(16) uint8_t gv_smem[];
  uint8_t* ws = gv_smem;                                   // [32 rows][kSegMax]
  float* xs = reinterpret_cast<float*>(gv_smem + kWBytes); // [m][kGvChunkBlocks * 256]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cta_n0 = blockIdx.x * kGvRowsPerCta;
  const int rows_here = min(kGvRowsPerCta, n_rows - cta_n0);
  uint64_t acc[kGvRowsPerWarp][kMT];
#pragma unroll
  for (int r = 0; r < kGvRowsPerWarp; ++r)
#pragma unroll
    for (int mm = 0; mm < kMT; ++mm) acc[r][mm] = 0ull;
  const int nb_all = k / 256;
  for (int b0 = 0; b0 < nb_all; b0 += kGvChunkBlocks) {
    const int nb = min(kGvChunkBlocks, nb_all - b0);
    const int seg = nb * kBB;                 // bytes of one row in this chunk
    const int kc = nb * 256;
    __syncthreads();  // the previous chunk is consumed
    // weights: rows_here segments of `seg` bytes, 16-byte vectors when the segments allow
    const uint8_t* src0 = blocks + static_cast<int64_t>(cta_n0) * row_bytes + static_cast<int64_t>(b0) * kBB;
    const bool vec16 = ((reinterpret_cast<uintptr_t>(src0) | static_cast<uintptr_t>(row_bytes) |
                         static_cast<uintptr_t>(seg)) & 15u) == 0;
    if (vec16) {
      const int per_row = seg / 16;
      for (int i = threadIdx.x; i < rows_here * per_row; i += kThreads) {
        const int r = i / per_row, c = i - r * per_row;
        reinterpret_cast<uint4*>(ws + r * kSegMax)[c] =
            __ldg(reinterpret_cast<const uint4*>(src0 + r * row_bytes) + c);
      }
    } else {  // 2-byte aligned (Q6_K rows of odd super-block counts)
      const int per_row = seg / 2;
      for (int i = threadIdx.x; i < rows_here * per_row; i += kThreads) {
        const int r = i / per_row, c = i - r * per_row;
        reinterpret_cast<uint16_t*>(ws + r * kSegMax)[c] =
            __ldg(reinterpret_cast<const uint16_t*>(src0 + r * row_bytes) + c);
      }
    }
    for (int i = threadIdx.x; i < m_rows * kc; i += kThreads) {
      const int mm = i / kc, kk = i - mm * kc;
      xs[mm * (kGvChunkBlocks * 256) + kk] = x[static_cast<int64_t>(mm) * ldx + b0 * 256 + kk];
    }
    __syncthreads();
    for (int j = 0; j < nb; ++j) {
      uint64_t xv[kMT][4];
#pragma unroll
      for (int mm = 0; mm < kMT; ++mm) {
        if (mm < m_rows) {
          const float4* s4 = reinterpret_cast<const float4*>(xs + mm * (kGvChunkBlocks * 256) + j * 256 + lane * 8);
          const float4 a = s4[0], c = s4[1];
          xv[mm][0] = gv_pack(a.x, a.y);
          xv[mm][1] = gv_pack(a.z, a.w);
          xv[mm][2] = gv_pack(c.x, c.y);
          xv[mm][3] = gv_pack(c.z, c.w);
        } else {
#pragma unroll
          for (int e = 0; e < 4; ++e) xv[mm][e] = 0ull;
        }
      }
#pragma unroll
      for (int r = 0; r < kGvRowsPerWarp; ++r) {
        const int lr = warp * kGvRowsPerWarp + r;
        if (lr >= rows_here) break;  // uniform over the warp
        float w[8];
        const uint8_t* b = ws + lr * kSegMax + j * kBB;
        if (kQT == 0)
          q4k_weights8(b, lane, w);
        else
          q6k_weights8(b, lane, w);
        uint64_t w2[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {  // round the pair to bf16 (one cvt), widen back exactly
          __nv_bfloat162 h = __floats2bfloat162_rn(w[2 * e], w[2 * e + 1]);
          const uint32_t u = *reinterpret_cast<uint32_t*>(&h);
          w2[e] = gv_pack(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
        }
#pragma unroll
        for (int mm = 0; mm < kMT; ++mm)
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[r][mm] = gv_fma2(w2[e], xv[mm][e], acc[r][mm]);
      }
    }
  }
  float out[kGvRowsPerWarp][kMT];
#pragma unroll
  for (int r = 0; r < kGvRowsPerWarp; ++r)
#pragma unroll
    for (int mm = 0; mm < kMT; ++mm) {
      float v = gv_sum2(acc[r][mm]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      out[r][mm] = v;
    }
  if (lane == 0) {
#pragma unroll
    for (int r = 0; r < kGvRowsPerWarp; ++r) {
      const int n = cta_n0 + warp * kGvRowsPerWarp + r;
      if (n >= n_rows) break;
#pragma unroll
      for (int mm = 0; mm < kMT; ++mm)
        if (mm < m_rows) y[static_cast<int64_t>(mm) * ldy + n] = out[r][mm];
    }
  }
}

template <int kQT>
int launch_gemv(const float* x, int64_t ldx, const uint8_t* blocks, float* y, int64_t ldy,
                int m, int n, int k, cudaStream_t st) {
  constexpr int kBB = kQT == 0 ? B200_Q4_K_BLOCK_BYTES : B200_Q6_K_BLOCK_BYTES;
  const int64_t row_bytes = static_cast<int64_t>(k / 256) * kBB;
  const size_t w_bytes = (kGvRowsPerCta * kGvChunkBlocks * kBB + 15) / 16 * 16;
  const unsigned grid = static_cast<unsigned>((n + kGvRowsPerCta - 1) / kGvRowsPerCta);
#define B200_GEMV_CASE(MT)                                                                  \
  {                                                                                         \
    auto fn = kquant_gemv_kernel<kQT, MT>;                                                  \
    const size_t smem = w_bytes + static_cast<size_t>(MT) * kGvChunkBlocks * 256 * 4;      \
    if (smem > 48 * 1024 &&                                                                 \
        cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,               \
                             static_cast<int>(smem)) != cudaSuccess)                        \
      return B200_ERR_CUDA;                                                                 \
    fn<<<grid, kThreads, smem, st>>>(x, ldx, blocks, row_bytes, y, ldy, m, n, k);          \
  }
  if (m <= 1) B200_GEMV_CASE(1)
  else B200_GEMV_CASE(2)
#undef B200_GEMV_CASE
  return cudaGetLastError() == cudaSuccess ? B200_OK : B200_ERR_CUDA;
}

int grid_for(int64_t threads) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t want = (threads + kThreads - 1) / kThreads;
  const int64_t cap = static_cast<int64_t>(sms) * 16;
  return static_cast<int>(want < cap ? want : cap);
}

}  // namespace

extern "C" int b200_dequant_q4_k(const void* blocks, void* out, int64_t n_blocks,
                                 b200_stream_t stream) {
  if (n_blocks < 0) return B200_ERR_INVALID;
  if (n_blocks == 0) return B200_OK;
  if (!blocks || !out) return B200_ERR_INVALID;
  // 16-byte blocks base: every block (144 bytes) then starts 16-byte aligned and the
  // 8-byte quant loads are aligned.
  if ((reinterpret_cast<uintptr_t>(blocks) & 15u) || (reinterpret_cast<uintptr_t>(out) & 15u))
    return B200_ERR_INVALID;
  dequant_q4k_kernel<<<grid_for(n_blocks * 32), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(blocks), static_cast<uint4*>(out), n_blocks);
  return cudaGetLastError() == cudaSuccess ? B200_OK : B200_ERR_CUDA;
}

extern "C" int b200_dequant_q6_k(const void* blocks, void* out, int64_t n_blocks,
                                 b200_stream_t stream) {
  if (n_blocks < 0) return B200_ERR_INVALID;
  if (n_blocks == 0) return B200_OK;
  if (!blocks || !out) return B200_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(blocks) & 1u) || (reinterpret_cast<uintptr_t>(out) & 15u))
    return B200_ERR_INVALID;
  dequant_q6k_kernel<<<grid_for(n_blocks * 32), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(blocks), static_cast<uint4*>(out), n_blocks);
  return cudaGetLastError() == cudaSuccess ? B200_OK : B200_ERR_CUDA;
}

extern "C" int b200_kquant_gemv(const float* x, int64_t ldx, const void* blocks, int32_t qtype,
                                float* y, int64_t ldy, int32_t m, int32_t n, int32_t k,
                                b200_stream_t stream) {
  if (m < 0 || n < 0 || k < 0) return B200_ERR_INVALID;
  if (m == 0 || n == 0) return B200_OK;
  if (m > B200_KQUANT_GEMV_MAX_ROWS || k == 0 || k % 256 != 0) return B200_ERR_INVALID;
  if (qtype != B200_KQUANT_Q4_K && qtype != B200_KQUANT_Q6_K) return B200_ERR_INVALID;
  if (!x || !blocks || !y || ldx < k || ldy < n) return B200_ERR_INVALID;
  // x rows are read as 16-byte vectors from shared memory; the global reads are scalar
  if (reinterpret_cast<uintptr_t>(blocks) & (qtype == B200_KQUANT_Q4_K ? 15u : 1u))
    return B200_ERR_INVALID;
  auto st = static_cast<cudaStream_t>(stream);
  auto* b = static_cast<const uint8_t*>(blocks);
  return qtype == B200_KQUANT_Q4_K ? launch_gemv<0>(x, ldx, b, y, ldy, m, n, k, st)
                                   : launch_gemv<1>(x, ldx, b, y, ldy, m, n, k, st);
}
