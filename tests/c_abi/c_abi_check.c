/* The C ABI from plain C11: every public header compiles as C, the library links, and
 * its host-side entry points give the reference's known answers without a GPU.
 * Built and run by tests/test_c_abi.py; exits non-zero on the first failed check. */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include "b200_attn.h"
#include "b200_block_ops.h"
#include "b200_gemm.h"
#include "b200_gguf.h"
#include "b200_tp.h"

#define CHECK(cond)                                                   \
  do {                                                                \
    if (!(cond)) {                                                    \
      fprintf(stderr, "check failed at line %d: %s\n", __LINE__, #cond); \
      return 1;                                                       \
    }                                                                 \
  } while (0)

int main(void) {
  CHECK(b200_abi_version() == B200_ATTN_ABI_VERSION);
  CHECK(strcmp(b200_strerror(B200_OK), "ok") == 0);
  CHECK(b200_attn_strerror(B200_ERR_INVALID) == b200_strerror(B200_ERR_INVALID));

  /* JointLayout::new known answer (src/joint_layout.rs:133-139): 3 text tokens, a 2x2
   * target grid -> image ids -1 -1 -1 0 0 0 0, prefix 3, target 4. */
  int64_t ids[16];
  uint8_t pad[16];
  int32_t shapes[3 * 4];
  int32_t len = 0, prefix = 0, target = 0;
  CHECK(b200_joint_layout(3, NULL, NULL, 0, 2, 2, 16, ids, pad, shapes, &len, &prefix,
                          &target) == B200_OK);
  CHECK(len == 7 && prefix == 3 && target == 4);
  const int64_t want_ids[7] = {-1, -1, -1, 0, 0, 0, 0};
  for (int i = 0; i < 7; ++i) CHECK(ids[i] == want_ids[i]);

  /* Block-causal limits of that layout: text rows see [0, i+1), the image block sees
   * itself whole. */
  int32_t limits[7];
  CHECK(b200_block_causal_limits(ids, 7, limits) == B200_OK);
  const int32_t want_lim[7] = {1, 2, 3, 7, 7, 7, 7};
  for (int i = 0; i < 7; ++i) CHECK(limits[i] == want_lim[i]);

  /* RoPE rows: position 0 of every axis gives (cos, sin) = (1, 0). */
  const int32_t axes[3] = {16, 56, 56};
  static float pe[7 * 128];
  CHECK(b200_rope_pe(shapes, 1, pad, 7, axes, 1e4f, pe) == B200_OK);
  for (int i = 0; i < 64; ++i) CHECK(fabsf(pe[2 * i] - 1.f) < 1e-6f && fabsf(pe[2 * i + 1]) < 1e-6f);

  /* key_valid -> descriptors: the last 2 of 5 prefix keys padded. */
  uint8_t kv[8] = {1, 1, 1, 0, 0, 1, 1, 1};
  b200_kv_desc desc;
  CHECK(b200_key_valid_to_desc(kv, 1, 5, 3, &desc) == B200_OK);
  CHECK(desc.prefix_valid == 3 && desc.target_valid == 3);
  kv[1] = 0; /* a hole inside the prefix is not representable */
  CHECK(b200_key_valid_to_desc(kv, 1, 5, 3, &desc) == B200_ERR_LAYOUT);

  /* Workspace sizing and argument checks before any device work. */
  b200_attn_args a;
  memset(&a, 0, sizeof(a));
  a.batch = 1;
  a.heads = 32;
  a.head_dim = 128;
  a.target_len = 4096;
  size_t ws = 0;
  CHECK(b200_attn_workspace_bytes(&a, &ws) == B200_OK);
  CHECK(ws == (size_t)2 * 32 * 4096 * 128 * 2 + B200_ATTN_SPLIT_WORKSPACE_BYTES);
  CHECK(b200_attn_fwd(&a, NULL) == B200_ERR_INVALID); /* null tensors */
  CHECK(b200_gemm(NULL, 0, NULL, 0, NULL, 0, 1, 1, 1, B200_GEMM_STORE_BF16, NULL, NULL) ==
        B200_ERR_INVALID);
  CHECK(b200_tp_destroy(NULL) == B200_ERR_INVALID);
  CHECK(b200_dequant_q4_k(NULL, NULL, 1, NULL) == B200_ERR_INVALID);
  CHECK(b200_swiglu(NULL, NULL, 1, 8, NULL) == B200_ERR_INVALID);

  printf("c abi ok\n");
  return 0;
}
