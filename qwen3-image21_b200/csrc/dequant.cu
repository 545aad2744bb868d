// dequant.cu — GGUF k-quant (Q4_K, Q6_K) super-blocks to bf16.
//
// One warp per 256-weight super-block, one thread per 8 consecutive weights: each thread
// reads its quant bytes, the block's scale bytes and f16 super-scales (L1 serves the
// repeats), and writes one 16-byte bf16 vector, so a warp's stores are one contiguous
// 512-byte row segment.  HBM-bound: per weight 144/256 (Q4_K) or 210/256 (Q6_K) bytes in
// and 2 bytes out.
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

// Q4_K: bytes 0-1 d, 2-3 dmin, 4-15 scales, 16-143 quants.
__global__ void __launch_bounds__(kThreads) dequant_q4k_kernel(const uint8_t* blocks, uint4* out,
                                                               int64_t n_blocks) {
  const int64_t total = n_blocks * 32;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * kThreads) {
    const int64_t blk = i >> 5;
    const int t = static_cast<int>(i & 31);
    const uint8_t* b = blocks + blk * B200_Q4_K_BLOCK_BYTES;
    const uint32_t dd = *reinterpret_cast<const uint32_t*>(b);
    const float d = half_bits_to_float(dd & 0xffffu);
    const float dmin = half_bits_to_float(dd >> 16);
    uint8_t sc_bytes[12];
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      const uint32_t w = *reinterpret_cast<const uint32_t*>(b + 4 + 4 * k);
#pragma unroll
      for (int e = 0; e < 4; ++e) sc_bytes[4 * k + e] = static_cast<uint8_t>(w >> (8 * e));
    }
    const int chunk = t >> 3;          // 64-weight chunk
    const int w0 = (t & 7) * 8;        // first weight within the chunk
    const int hi = w0 >= 32;           // high nibbles: the chunk's second 32 weights
    const int l0 = w0 & 31;
    const int is = 2 * chunk + hi;     // sub-block of 32
    uint32_t sc, mn;
    if (is < 4) {
      sc = sc_bytes[is] & 63u;
      mn = sc_bytes[is + 4] & 63u;
    } else {
      sc = (sc_bytes[is + 4] & 0xFu) | ((sc_bytes[is - 4] >> 6) << 4);
      mn = (sc_bytes[is + 4] >> 4) | ((sc_bytes[is] >> 6) << 4);
    }
    const float d1 = __fmul_rn(d, static_cast<float>(sc));
    const float m1 = __fmul_rn(dmin, static_cast<float>(mn));
    const uint2 q8 = *reinterpret_cast<const uint2*>(b + 16 + 32 * chunk + l0);
    const uint32_t qw[2] = {q8.x, q8.y};
    float y[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const uint32_t byte = (qw[e >> 2] >> (8 * (e & 3))) & 0xFFu;
      const uint32_t q = hi ? (byte >> 4) : (byte & 0xFu);
      y[e] = __fsub_rn(__fmul_rn(d1, static_cast<float>(q)), m1);
    }
    out[i] = pack8_bf16(y);
  }
}

// Q6_K: bytes 0-127 ql, 128-191 qh, 192-207 int8 scales, 208-209 d.  The block is only
// 2-byte aligned (210 bytes), so bytes are read as 16-bit words.
__device__ __forceinline__ uint32_t load_u16(const uint8_t* p) {
  return *reinterpret_cast<const uint16_t*>(p);
}

__global__ void __launch_bounds__(kThreads) dequant_q6k_kernel(const uint8_t* blocks, uint4* out,
                                                               int64_t n_blocks) {
  const int64_t total = n_blocks * 32;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * kThreads) {
    const int64_t blk = i >> 5;
    const int t = static_cast<int>(i & 31);
    const uint8_t* b = blocks + blk * B200_Q6_K_BLOCK_BYTES;
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
    float y[8];
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
        const int q = static_cast<int>(lo | (hb << 4)) - 32;
        y[e + k] = __fmul_rn(ds, static_cast<float>(q));
      }
    }
    out[i] = pack8_bf16(y);
  }
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
