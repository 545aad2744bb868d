/* b200_attn_fwd called from plain C, as a native host (the engine's Rust crate) calls it:
 * device buffers from the CUDA runtime, the library's host mirrors for the layout and the
 * RoPE rows, one call on the default stream, then the output against the C oracle
 * (oracle/cpu_attention.c, compiled into this test) at the north-star tolerance.
 * Built and run by tests/test_c_abi.py on a GPU; exits non-zero on failure. */
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "b200_attn.h"

int oracle_attention_forward(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                             const uint16_t* prefix_k, const uint16_t* prefix_v,
                             const float* wq, const float* wk, float eps, const float* pe,
                             const int32_t* prefix_valid, float scale, int B, int T, int H,
                             int P, int D, float* out, int threads);

#define CHECK(cond)                                                        \
  do {                                                                     \
    if (!(cond)) {                                                         \
      fprintf(stderr, "check failed at line %d: %s\n", __LINE__, #cond);   \
      return 1;                                                            \
    }                                                                      \
  } while (0)
#define CUDA(call) CHECK((call) == cudaSuccess)

static uint64_t rng_state = 0x9E3779B97F4A7C15ull;
static double uniform(void) {
  rng_state = rng_state * 6364136223846793005ull + 1442695040888963407ull;
  return ((rng_state >> 11) + 0.5) * (1.0 / 9007199254740992.0);
}
static float normal(void) {
  return (float)(sqrt(-2.0 * log(uniform())) * cos(6.283185307179586 * uniform()));
}
static uint16_t to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}
static float from_bf16(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}
static void fill(uint16_t* x, size_t n) {
  for (size_t i = 0; i < n; ++i) x[i] = to_bf16(normal());
}

int main(void) {
  enum { B = 2, T = 300, H = 4, P = 200, D = 128, GH = 15, GW = 20 };
  const int32_t prefix_valid[B] = {200, 137};
  const size_t n_qkv = (size_t)B * T * H * D, n_pre = (size_t)B * H * P * D;
  uint16_t *q = malloc(2 * n_qkv), *k = malloc(2 * n_qkv), *v = malloc(2 * n_qkv);
  uint16_t *pk = malloc(2 * n_pre), *pv = malloc(2 * n_pre), *out_bits = malloc(2 * n_qkv);
  float *wq = malloc(4 * D), *wk = malloc(4 * D), *want = malloc(4 * n_qkv);
  CHECK(q && k && v && pk && pv && out_bits && wq && wk && want);
  fill(q, n_qkv);
  fill(k, n_qkv);
  fill(v, n_qkv);
  fill(pk, n_pre);
  fill(pv, n_pre);
  for (int i = 0; i < D; ++i) {
    wq[i] = 1.f + 0.1f * normal();
    wk[i] = 1.f + 0.1f * normal();
  }

  /* The layout (P text tokens, a GH x GW target grid) and its RoPE rows, from the
   * library's host mirrors; the step's rows are [P, P + T). */
  int64_t ids[P + T];
  uint8_t pad[P + T];
  int32_t shapes[3 * 4], len = 0, prefix = 0, target = 0;
  CHECK(b200_joint_layout(P, NULL, NULL, 0, GH, GW, P + T, ids, pad, shapes, &len, &prefix,
                          &target) == B200_OK);
  CHECK(len == P + T && prefix == P && target == T);
  const int32_t axes[3] = {16, 56, 56};
  float* pe_all = malloc(sizeof(float) * (P + T) * D);
  CHECK(pe_all);
  CHECK(b200_rope_pe(shapes, 1, pad, P + T, axes, 1e4f, pe_all) == B200_OK);
  const float* pe = pe_all + (size_t)P * D;

  /* Device side through the C ABI. */
  void *dq, *dk, *dv, *dpk, *dpv, *dout, *dws;
  float *dwq, *dwk, *dpe;
  b200_kv_desc* ddesc;
  int32_t* dstatus;
  CUDA(cudaMalloc(&dq, 2 * n_qkv));
  CUDA(cudaMalloc(&dk, 2 * n_qkv));
  CUDA(cudaMalloc(&dv, 2 * n_qkv));
  CUDA(cudaMalloc(&dpk, 2 * n_pre));
  CUDA(cudaMalloc(&dpv, 2 * n_pre));
  CUDA(cudaMalloc(&dout, 2 * n_qkv));
  CUDA(cudaMalloc((void**)&dwq, 4 * D));
  CUDA(cudaMalloc((void**)&dwk, 4 * D));
  CUDA(cudaMalloc((void**)&dpe, 4 * (size_t)T * D));
  CUDA(cudaMalloc((void**)&ddesc, sizeof(b200_kv_desc) * B));
  CUDA(cudaMalloc((void**)&dstatus, 4));
  CUDA(cudaMemcpy(dq, q, 2 * n_qkv, cudaMemcpyHostToDevice));
  CUDA(cudaMemcpy(dk, k, 2 * n_qkv, cudaMemcpyHostToDevice));
  CUDA(cudaMemcpy(dv, v, 2 * n_qkv, cudaMemcpyHostToDevice));
  CUDA(cudaMemcpy(dpk, pk, 2 * n_pre, cudaMemcpyHostToDevice));
  CUDA(cudaMemcpy(dpv, pv, 2 * n_pre, cudaMemcpyHostToDevice));
  CUDA(cudaMemcpy(dwq, wq, 4 * D, cudaMemcpyHostToDevice));
  CUDA(cudaMemcpy(dwk, wk, 4 * D, cudaMemcpyHostToDevice));
  CUDA(cudaMemcpy(dpe, pe, 4 * (size_t)T * D, cudaMemcpyHostToDevice));
  b200_kv_desc desc[B];
  for (int b = 0; b < B; ++b) {
    desc[b].prefix_valid = prefix_valid[b];
    desc[b].target_valid = T;
  }
  CUDA(cudaMemcpy(ddesc, desc, sizeof(desc), cudaMemcpyHostToDevice));
  CUDA(cudaMemset(dstatus, 0, 4));

  b200_attn_args a;
  memset(&a, 0, sizeof(a));
  a.batch = B;
  a.heads = H;
  a.head_dim = D;
  a.target_len = T;
  a.prefix_len = P;
  a.q = dq;
  a.k = dk;
  a.v = dv;
  a.prefix_k = dpk;
  a.prefix_v = dpv;
  a.norm_q_w = dwq;
  a.norm_k_w = dwk;
  a.norm_eps = 1e-6f;
  a.pe = dpe;
  a.desc = ddesc;
  a.scale = 1.f / sqrtf((float)D);
  a.out = dout;
  a.status = dstatus;
  size_t ws_bytes = 0;
  CHECK(b200_attn_workspace_bytes(&a, &ws_bytes) == B200_OK);
  CUDA(cudaMalloc(&dws, ws_bytes));
  a.workspace = dws;
  a.workspace_bytes = ws_bytes;
  const int rc = b200_attn_fwd(&a, NULL);
  if (rc != B200_OK) fprintf(stderr, "b200_attn_fwd: %s\n", b200_strerror(rc));
  CHECK(rc == B200_OK);
  CUDA(cudaDeviceSynchronize());
  int32_t status = -1;
  CUDA(cudaMemcpy(&status, dstatus, 4, cudaMemcpyDeviceToHost));
  CHECK(status == 0);
  CUDA(cudaMemcpy(out_bits, dout, 2 * n_qkv, cudaMemcpyDeviceToHost));

  /* The oracle on the same values. */
  CHECK(oracle_attention_forward(q, k, v, pk, pv, wq, wk, 1e-6f, pe, prefix_valid, a.scale, B,
                                 T, H, P, D, want, 0) == 0);
  double num = 0.0, den = 0.0, max_abs = 0.0;
  for (size_t i = 0; i < n_qkv; ++i) {
    const double g = from_bf16(out_bits[i]), w = want[i], e = fabs(g - w);
    CHECK(isfinite(g));
    num += e * e;
    den += w * w;
    if (e > max_abs) max_abs = e;
  }
  const double rel = sqrt(num / den);
  printf("c gpu parity: rel_l2=%.3e max_abs=%.3e\n", rel, max_abs);
  CHECK(rel <= 5e-3 && max_abs <= 2e-2);
  printf("c abi gpu ok\n");
  return 0;
}
