// block_ops.cu — the elementwise steps of the single-stream block between its GEMMs
// (src/transformer.rs:396-427), for the denoising loop around the attention path:
//   residual_adaln_kernel  x += tanh(gate) * y ; out = LayerNorm(x) * (1 + scale)
//   swiglu_kernel          h = silu(gate) * proj
// Both are HBM-bound streams: 16-byte vector loads and stores, one pass over the data,
// modulation rows (gate, 1 + scale) held in registers across the rows a CTA handles.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "../../include/b200_block_ops.h"

namespace {

constexpr int kThreads = 256;
constexpr int kRowsPerCta = 8;   // rows of one CTA; modulation loaded once per sequence
constexpr int kMaxCols = 8192;

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();  // red[] is reused by consecutive reductions
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < kThreads / 32; ++w) t += red[w];
  return t;
}

__device__ __forceinline__ uint2 pack4_bf16(float a, float b, float c, float d) {
  __nv_bfloat162 lo = __floats2bfloat162_rn(a, b), hi = __floats2bfloat162_rn(c, d);
  return make_uint2(*reinterpret_cast<uint32_t*>(&lo), *reinterpret_cast<uint32_t*>(&hi));
}

__device__ __forceinline__ float4 unpack4_bf16(uint2 u) {
  return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u),
                     __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xffff0000u));
}

struct ResidualAdaLnParams {
  float* x;
  const uint2* y;      // bf16 x4 per element group, or null
  const float* gate;
  const float* scale;
  uint2* out;          // bf16 x4, or null
  int64_t rows, rows_per_mod, mod_stride;
  int cols;
  float eps;
};

// Thread i owns float4 groups i, i + 256, ... (NV of them) of every row of its CTA.  The
// kernel is latency-bound (two block reductions per row), so up to 4096 columns the
// register cap of 4 CTAs per SM pays (15 % faster at 4096 columns than 3 CTAs per SM).
template <int NV>
__global__ void __launch_bounds__(kThreads, NV <= 4 ? 4 : 1)
    residual_adaln_kernel(ResidualAdaLnParams p) {
  __shared__ float red[kThreads / 32];
  const int groups = p.cols >> 2;
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * kRowsPerCta;
  float4 tg[NV], sc[NV];
  int64_t mod_row = -1;
  for (int rr = 0; rr < kRowsPerCta; ++rr) {
    const int64_t r = r0 + rr;
    if (r >= p.rows) break;  // uniform over the CTA
    const int64_t m = r / p.rows_per_mod;
    if (m != mod_row) {
      mod_row = m;
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        const int g = threadIdx.x + i * kThreads;
        if (g < groups) {
          if (p.y) {
            const float4 gv = reinterpret_cast<const float4*>(p.gate + m * p.mod_stride)[g];
            tg[i] = make_float4(tanhf(gv.x), tanhf(gv.y), tanhf(gv.z), tanhf(gv.w));
          }
          if (p.out) {
            const float4 sv = reinterpret_cast<const float4*>(p.scale + m * p.mod_stride)[g];
            sc[i] = make_float4(1.f + sv.x, 1.f + sv.y, 1.f + sv.z, 1.f + sv.w);
          }
        }
      }
    }
    float4* xr = reinterpret_cast<float4*>(p.x + r * p.cols);
    float4 xv[NV];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int g = threadIdx.x + i * kThreads;
      if (g < groups) {
        xv[i] = xr[g];
        if (p.y) {
          const float4 yv = unpack4_bf16(p.y[r * groups + g]);
          xv[i].x = fmaf(tg[i].x, yv.x, xv[i].x);
          xv[i].y = fmaf(tg[i].y, yv.y, xv[i].y);
          xv[i].z = fmaf(tg[i].z, yv.z, xv[i].z);
          xv[i].w = fmaf(tg[i].w, yv.w, xv[i].w);
          xr[g] = xv[i];
        }
        s += (xv[i].x + xv[i].y) + (xv[i].z + xv[i].w);
      } else {
        xv[i] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    if (!p.out) continue;
    const float inv_n = 1.f / static_cast<float>(p.cols);
    const float mean = block_sum(s, red) * inv_n;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int g = threadIdx.x + i * kThreads;
      if (g < groups) {
        const float a = xv[i].x - mean, b = xv[i].y - mean, c = xv[i].z - mean, d = xv[i].w - mean;
        q += (a * a + b * b) + (c * c + d * d);
      }
    }
    const float rstd = rsqrtf(block_sum(q, red) * inv_n + p.eps);
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int g = threadIdx.x + i * kThreads;
      if (g < groups)
        p.out[r * groups + g] = pack4_bf16((xv[i].x - mean) * rstd * sc[i].x,
                                           (xv[i].y - mean) * rstd * sc[i].y,
                                           (xv[i].z - mean) * rstd * sc[i].z,
                                           (xv[i].w - mean) * rstd * sc[i].w);
    }
  }
}

// One thread per 8 outputs; gate columns [0, F), proj columns [F, 2F) of each gp row.
__global__ void __launch_bounds__(kThreads) swiglu_kernel(const uint4* gp, uint4* h,
                                                          int64_t rows, int f8) {
  const int64_t n = rows * f8;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * kThreads) {
    const int64_t r = i / f8;
    const int j = static_cast<int>(i - r * f8);
    const uint4 g = gp[r * 2 * f8 + j];
    const uint4 u = gp[r * 2 * f8 + f8 + j];
    const uint32_t gw[4] = {g.x, g.y, g.z, g.w}, uw[4] = {u.x, u.y, u.z, u.w};
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float g0 = __uint_as_float(gw[k] << 16), g1 = __uint_as_float(gw[k] & 0xffff0000u);
      const float u0 = __uint_as_float(uw[k] << 16), u1 = __uint_as_float(uw[k] & 0xffff0000u);
      const float a0 = g0 / (1.f + __expf(-g0)), a1 = g1 / (1.f + __expf(-g1));
      __nv_bfloat162 v = __floats2bfloat162_rn(a0 * u0, a1 * u1);
      o[k] = *reinterpret_cast<uint32_t*>(&v);
    }
    h[i] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

int sm_count() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

}  // namespace

extern "C" int b200_residual_adaln(float* x, const void* y, const float* gate, const float* scale,
                                   void* out, int64_t rows, int32_t cols, int64_t rows_per_mod,
                                   int64_t mod_stride, float eps, b200_stream_t stream) {
  if (rows < 0 || cols <= 0 || cols % 4 != 0 || cols > kMaxCols) return B200_ERR_INVALID;
  if (rows == 0) return B200_OK;
  if (!x || (!y && !out) || (y && !gate) || (out && !scale)) return B200_ERR_INVALID;
  if (rows_per_mod <= 0 || mod_stride < 0 || mod_stride % 4 != 0) return B200_ERR_INVALID;
  const void* ptrs[] = {x, y, gate, scale, out};
  for (const void* ptr : ptrs)
    if (ptr && !aligned16(ptr)) return B200_ERR_INVALID;
  if (!(eps >= 0.f) || !std::isfinite(eps)) return B200_ERR_INVALID;
  ResidualAdaLnParams p{x, static_cast<const uint2*>(y), gate, scale, static_cast<uint2*>(out),
                        rows, rows_per_mod, mod_stride, cols, eps};
  const int64_t blocks = (rows + kRowsPerCta - 1) / kRowsPerCta;
  if (blocks > 0x7fffffff) return B200_ERR_INVALID;
  const int nv = (cols / 4 + kThreads - 1) / kThreads;
  auto s = static_cast<cudaStream_t>(stream);
  const dim3 grid(static_cast<unsigned>(blocks));
  if (nv <= 1) residual_adaln_kernel<1><<<grid, kThreads, 0, s>>>(p);
  else if (nv <= 2) residual_adaln_kernel<2><<<grid, kThreads, 0, s>>>(p);
  else if (nv <= 4) residual_adaln_kernel<4><<<grid, kThreads, 0, s>>>(p);
  else residual_adaln_kernel<8><<<grid, kThreads, 0, s>>>(p);
  return cudaGetLastError() == cudaSuccess ? B200_OK : B200_ERR_CUDA;
}

extern "C" int b200_swiglu(const void* gp, void* h, int64_t rows, int32_t ffn,
                           b200_stream_t stream) {
  if (rows < 0 || ffn <= 0 || ffn % 8 != 0) return B200_ERR_INVALID;
  if (rows == 0) return B200_OK;
  if (!gp || !h || !aligned16(gp) || !aligned16(h)) return B200_ERR_INVALID;
  const int f8 = ffn / 8;
  const int64_t n = rows * f8;
  // Enough CTAs to fill every SM several times over; the loop strides the rest.
  const int64_t want = (n + kThreads - 1) / kThreads;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 16;
  const unsigned blocks = static_cast<unsigned>(want < cap ? want : cap);
  swiglu_kernel<<<blocks, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(gp), static_cast<uint4*>(h), rows, f8);
  return cudaGetLastError() == cudaSuccess ? B200_OK : B200_ERR_CUDA;
}
