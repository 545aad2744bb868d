/*
 * cpu_attention.c — C restatement of the reference's CPU joint-attention path.
 * TEST / BASELINE INFRASTRUCTURE ONLY: the checker and the timed CPU baseline
 * ("port": the reference is Rust/candle and cannot be built in this image).  The
 * product library never links or calls this file.
 *
 * Follows, in float32:
 *   - candle_nn::RmsNorm, eps 1e-6           src/transformer.rs:141-145, 179-180
 *   - apply_rope / rope_i (interleaved pairs) src/rope.rs:222-228 (formula: 324-349)
 *   - Tensor::cat(prefix, step) of K and V    src/transformer.rs:186-189
 *   - chunked_attention                       src/transformer.rs:259-296:
 *       q pre-scaled (275), S = q k^T (281), additive -inf mask (284-287),
 *       f32 row softmax (292), P v (293).
 * The reference's query chunk (256 MiB of scores, line 273) bounds memory only; every
 * query row is computed exactly as without chunking, so rows are processed in blocks of
 * QBLOCK per thread here.  Threads: OpenMP over (batch, head, query block).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define QBLOCK 32

static float bf16_to_f32(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* one (b, h) slice: q [Sq][D] (already scaled), kt [D][Skv], v [Skv][D] -> o [Sq][D] */
static void attend_block(const float* q, const float* kt, const float* v, float* o,
                         int rows, int skv, int kvalid, int d, float* s) {
  for (int i = 0; i < rows; ++i) {
    float* si = s + (size_t)i * skv;
    for (int j = 0; j < skv; ++j) si[j] = 0.f;
    for (int c = 0; c < d; ++c) {
      const float qc = q[(size_t)i * d + c];
      const float* kr = kt + (size_t)c * skv;
      for (int j = 0; j < skv; ++j) si[j] += qc * kr[j];
    }
    for (int j = kvalid; j < skv; ++j) si[j] = -INFINITY; /* additive -inf mask */
    float mx = -INFINITY;
    for (int j = 0; j < skv; ++j) mx = si[j] > mx ? si[j] : mx;
    float sum = 0.f;
    for (int j = 0; j < skv; ++j) {
      si[j] = expf(si[j] - mx);
      sum += si[j];
    }
    const float inv = 1.f / sum;
    for (int j = 0; j < skv; ++j) si[j] *= inv;
    float* oi = o + (size_t)i * d;
    for (int c = 0; c < d; ++c) oi[c] = 0.f;
    for (int j = 0; j < skv; ++j) {
      const float p = si[j];
      const float* vr = v + (size_t)j * d;
      for (int c = 0; c < d; ++c) oi[c] += p * vr[c];
    }
  }
}

/*
 * chunked_attention on float32 [B,H,Sq,D] / [B,H,Skv,D] with key_len[b] valid leading
 * keys (NULL = all).  out [B,H,Sq,D].  Returns 0.
 */
int oracle_chunked_attention(const float* q, const float* k, const float* v, float* out,
                             int B, int H, int Sq, int Skv, int D, float scale,
                             const int32_t* key_len, int threads) {
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#endif
  const size_t nbh = (size_t)B * H;
  float* kt_all = (float*)malloc(sizeof(float) * nbh * (size_t)D * Skv);
  if (!kt_all) return -1;
#pragma omp parallel for schedule(static)
  for (long bh = 0; bh < (long)nbh; ++bh) {
    const float* kb = k + (size_t)bh * Skv * D;
    float* kt = kt_all + (size_t)bh * D * Skv;
    for (int j = 0; j < Skv; ++j)
      for (int c = 0; c < D; ++c) kt[(size_t)c * Skv + j] = kb[(size_t)j * D + c];
  }
  const int nqb = (Sq + QBLOCK - 1) / QBLOCK;
  int rc = 0;
#pragma omp parallel
  {
    float* s = (float*)malloc(sizeof(float) * (size_t)QBLOCK * Skv);
    float* qs = (float*)malloc(sizeof(float) * (size_t)QBLOCK * D);
    if (!s || !qs) {
#pragma omp atomic write
      rc = -1;
    } else {
#pragma omp for schedule(dynamic, 1)
      for (long it = 0; it < (long)(nbh * nqb); ++it) {
        const long bh = it / nqb;
        const int qb = (int)(it % nqb);
        const int b = (int)(bh / H);
        const int r0 = qb * QBLOCK;
        const int rows = Sq - r0 < QBLOCK ? Sq - r0 : QBLOCK;
        const int kvalid = key_len ? key_len[b] : Skv;
        const float* qb_ptr = q + ((size_t)bh * Sq + r0) * D;
        for (int i = 0; i < rows * D; ++i) qs[i] = qb_ptr[i] * scale; /* q.affine(scale) */
        attend_block(qs, kt_all + (size_t)bh * D * Skv, v + (size_t)bh * Skv * D,
                     out + ((size_t)bh * Sq + r0) * D, rows, Skv, kvalid, D, s);
      }
    }
    free(s);
    free(qs);
  }
  free(kt_all);
  return rc;
}

/*
 * The full span b200_attn_fwd replaces, on bf16 inputs (as uint16 bit patterns):
 *   q,k,v [B,T,H,D] raw projections; prefix_k/v [B,H,P,D]; norm weights [D] f32;
 *   pe [T,D] f32 interleaved (cos, sin); prefix_valid [B] or NULL.
 * out [B,T,H*D] float32.  Work buffers are allocated here (baseline code).
 */
int oracle_attention_forward(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                             const uint16_t* prefix_k, const uint16_t* prefix_v,
                             const float* wq, const float* wk, float eps, const float* pe,
                             const int32_t* prefix_valid, float scale, int B, int T, int H,
                             int P, int D, float* out, int threads) {
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#endif
  const int L = P + T;
  const size_t nbh = (size_t)B * H;
  float* qh = (float*)malloc(sizeof(float) * nbh * T * D);
  float* kh = (float*)malloc(sizeof(float) * nbh * L * D);
  float* vh = (float*)malloc(sizeof(float) * nbh * L * D);
  float* oh = (float*)malloc(sizeof(float) * nbh * T * D);
  int32_t* klen = (int32_t*)malloc(sizeof(int32_t) * (B > 0 ? B : 1));
  if (!qh || !kh || !vh || !oh || !klen) {
    free(qh); free(kh); free(vh); free(oh); free(klen);
    return -1;
  }
  /* prefix rows of K/V (cat, src/transformer.rs:186-189); cast bf16 -> f32 (43-45) */
#pragma omp parallel for schedule(static)
  for (long bh = 0; bh < (long)nbh; ++bh)
    for (int r = 0; r < P; ++r)
      for (int c = 0; c < D; ++c) {
        const size_t src = ((size_t)bh * P + r) * D + c;
        const size_t dst = ((size_t)bh * L + r) * D + c;
        kh[dst] = bf16_to_f32(prefix_k[src]);
        vh[dst] = bf16_to_f32(prefix_v[src]);
      }
  /* RMSNorm (q, k) + RoPE, transpose to [B,H,S,D] */
#pragma omp parallel for schedule(static)
  for (long row = 0; row < (long)B * T * H; ++row) {
    const int h = (int)(row % H);
    const int t = (int)((row / H) % T);
    const int b = (int)(row / ((long)H * T));
    const size_t src = (size_t)row * D;
    float xq[256], xk[256];
    float ssq = 0.f, ssk = 0.f;
    for (int c = 0; c < D; ++c) {
      xq[c] = bf16_to_f32(q[src + c]);
      xk[c] = bf16_to_f32(k[src + c]);
      ssq += xq[c] * xq[c];
      ssk += xk[c] * xk[c];
    }
    const float dq = sqrtf(ssq / (float)D + eps), dk = sqrtf(ssk / (float)D + eps);
    for (int c = 0; c < D; ++c) {
      xq[c] = xq[c] / dq * wq[c];
      xk[c] = xk[c] / dk * wk[c];
    }
    const size_t qd = (((size_t)b * H + h) * T + t) * D;
    const size_t kd = (((size_t)b * H + h) * L + P + t) * D;
    for (int i = 0; i < D / 2; ++i) {
      const float cs = pe[(size_t)t * D + 2 * i], sn = pe[(size_t)t * D + 2 * i + 1];
      const float q0 = xq[2 * i], q1 = xq[2 * i + 1], k0 = xk[2 * i], k1 = xk[2 * i + 1];
      qh[qd + 2 * i] = q0 * cs - q1 * sn;
      qh[qd + 2 * i + 1] = q0 * sn + q1 * cs;
      kh[kd + 2 * i] = k0 * cs - k1 * sn;
      kh[kd + 2 * i + 1] = k0 * sn + k1 * cs;
      vh[kd + 2 * i] = bf16_to_f32(v[src + 2 * i]);
      vh[kd + 2 * i + 1] = bf16_to_f32(v[src + 2 * i + 1]);
    }
  }
  int rc = 0;
  if (!prefix_valid) {
    for (int b = 0; b < B; ++b) klen[b] = L;
    rc = oracle_chunked_attention(qh, kh, vh, oh, B, H, T, L, D, scale, klen, threads);
  } else {
    /* A padded prefix suffix: compact the valid keys to [prefix[:pv]; step].  Key order
       is kept and masked keys contribute exactly 0 after the -inf mask, so softmax and
       P v over the compacted list equal the masked computation over [prefix; step]. */
    for (int b = 0; b < B; ++b) {
      const int pv = prefix_valid[b];
      for (int h = 0; h < H; ++h) {
        float* kb = kh + ((size_t)b * H + h) * L * D;
        float* vb = vh + ((size_t)b * H + h) * L * D;
        memmove(kb + (size_t)pv * D, kb + (size_t)P * D, sizeof(float) * (size_t)T * D);
        memmove(vb + (size_t)pv * D, vb + (size_t)P * D, sizeof(float) * (size_t)T * D);
      }
      klen[b] = pv + T;
    }
    rc = oracle_chunked_attention(qh, kh, vh, oh, B, H, T, L, D, scale, klen, threads);
  }
  /* [B,H,T,D] -> [B,T,H*D] (src/transformer.rs:193) */
#pragma omp parallel for schedule(static)
  for (long row = 0; row < (long)B * T * H; ++row) {
    const int h = (int)(row % H);
    const int t = (int)((row / H) % T);
    const int b = (int)(row / ((long)H * T));
    memcpy(out + (size_t)row * D, oh + (((size_t)b * H + h) * T + t) * D, sizeof(float) * D);
  }
  free(qh); free(kh); free(vh); free(oh); free(klen);
  return rc;
}

int oracle_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
