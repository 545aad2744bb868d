// host_layout.cpp — host-side C++ mirrors of the reference's layout, RoPE-table and mask
// code that feed the attention path (no device work):
//   b200_joint_layout       JointLayout::new            src/joint_layout.rs:52-103
//   b200_rope_positions     EmbedNd::forward positions  src/rope.rs:118-172
//   b200_rope_pe            EmbedNd::new + forward      src/rope.rs:37-211
//   b200_key_valid_to_desc  key_valid (cached step)     src/transformer.rs:642-649, 736-745
//   b200_block_causal_limits block-causal mask as row limits  src/attention_mask.rs:18-66
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>

#include "../../include/b200_attn.h"

namespace {

constexpr int64_t kTableNeg = 1024;   // src/rope.rs:44-47
constexpr int64_t kTablePos = 8192;   // src/rope.rs:43
constexpr int kTokensPerSlot = 4;     // src/joint_layout.rs:10

}  // namespace

extern "C" int b200_joint_layout(int32_t text_len, const uint8_t* text_image_mask,
                                 const int32_t* cond_shapes, int32_t n_cond, int32_t target_h,
                                 int32_t target_w, int32_t cap, int64_t* image_ids,
                                 uint8_t* image_pad_mask, int32_t* img_shapes, int32_t* len_out,
                                 int32_t* prefix_len_out, int32_t* target_len_out) {
  if (text_len < 0 || n_cond < 0 || target_h < 0 || target_w < 0 || cap < 0)
    return B200_ERR_INVALID;
  if (n_cond > 0 && !cond_shapes) return B200_ERR_INVALID;
  if (!len_out || !prefix_len_out || !target_len_out) return B200_ERR_INVALID;
  // Pieces: kind 0 = text [start, len), 1 = condition image `index`, 2 = target.
  struct Piece { int kind, start, len; };
  std::vector<Piece> pieces;
  int i = 0, next_image = 0;
  auto slot = [&](int k) { return text_image_mask && text_image_mask[k] != 0; };
  while (i < text_len) {
    if (!slot(i)) {
      int len = 0;
      while (i + len < text_len && !slot(i + len)) ++len;
      pieces.push_back({0, i, len});
      i += len;
      continue;
    }
    // Blocks are delimited by token counts, so adjacent images stay separate blocks.
    if (next_image >= n_cond) return B200_ERR_LAYOUT;  // more slots than images
    const int h = cond_shapes[2 * next_image], w = cond_shapes[2 * next_image + 1];
    if (h < 0 || w < 0) return B200_ERR_INVALID;
    const int needed = h * w / kTokensPerSlot;
    int have = 0;
    for (int k = i; k < i + needed && k < text_len; ++k) have += slot(k) ? 1 : 0;
    if ((h * w) % kTokensPerSlot != 0 || have != needed) return B200_ERR_LAYOUT;
    pieces.push_back({1, next_image, 0});
    ++next_image;
    i += needed;
  }
  if (next_image != n_cond) return B200_ERR_LAYOUT;  // images without slots
  pieces.push_back({2, 0, 0});

  int64_t total = 0;
  for (const Piece& p : pieces) {
    if (p.kind == 0) total += p.len;
    else if (p.kind == 1) total += static_cast<int64_t>(cond_shapes[2 * p.start]) * cond_shapes[2 * p.start + 1];
    else total += static_cast<int64_t>(target_h) * target_w;
  }
  const int64_t target_len = static_cast<int64_t>(target_h) * target_w;
  *len_out = static_cast<int32_t>(total);
  *prefix_len_out = static_cast<int32_t>(total - target_len);
  *target_len_out = static_cast<int32_t>(target_len);
  if (img_shapes) {
    for (int c = 0; c < n_cond; ++c) {
      img_shapes[3 * c] = 1;
      img_shapes[3 * c + 1] = cond_shapes[2 * c];
      img_shapes[3 * c + 2] = cond_shapes[2 * c + 1];
    }
    img_shapes[3 * n_cond] = 1;
    img_shapes[3 * n_cond + 1] = target_h;
    img_shapes[3 * n_cond + 2] = target_w;
  }
  if (!image_ids && !image_pad_mask) return B200_OK;
  if (total > cap) return B200_ERR_INVALID;
  int64_t pos = 0;
  for (const Piece& p : pieces) {
    int64_t len;
    int64_t id;
    if (p.kind == 0) { len = p.len; id = -1; }
    else if (p.kind == 1) { len = static_cast<int64_t>(cond_shapes[2 * p.start]) * cond_shapes[2 * p.start + 1]; id = p.start; }
    else { len = target_len; id = n_cond; }
    for (int64_t k = 0; k < len; ++k, ++pos) {
      if (image_ids) image_ids[pos] = id;
      if (image_pad_mask) image_pad_mask[pos] = id >= 0 ? 1 : 0;
    }
  }
  return B200_OK;
}

extern "C" int b200_rope_positions(const int32_t* img_shapes, int32_t n_shapes,
                                   const uint8_t* image_pad_mask, int32_t seq_len,
                                   int64_t* pos_out) {
  if (n_shapes < 0 || seq_len < 0 || (n_shapes > 0 && !img_shapes)) return B200_ERR_INVALID;
  if (seq_len > 0 && (!image_pad_mask || !pos_out)) return B200_ERR_INVALID;
  int64_t cursor = 0, position = 0, n = 0;
  auto push = [&](int64_t f, int64_t hh, int64_t ww) -> bool {
    if (n >= seq_len) return false;
    pos_out[3 * n] = f;
    pos_out[3 * n + 1] = hh;
    pos_out[3 * n + 2] = ww;
    ++n;
    return true;
  };
  for (int s = 0; s < n_shapes; ++s) {
    const int64_t frame = img_shapes[3 * s], height = img_shapes[3 * s + 1], width = img_shapes[3 * s + 2];
    if (frame < 0 || height < 0 || width < 0) return B200_ERR_INVALID;
    int64_t block_start = seq_len;
    for (int64_t k = cursor; k < seq_len; ++k)
      if (image_pad_mask[k]) { block_start = k; break; }
    for (int64_t k = cursor; k < block_start; ++k) {  // text: advance all three axes
      if (!push(position, position, position)) return B200_ERR_LAYOUT;
      ++position;
    }
    cursor = block_start;
    const int64_t block_tokens = frame * height * width;
    const int64_t frame_pos = position;  // frame frozen at the running position
    position += height > width ? height : width;
    const int64_t h_start = -(height - height / 2), w_start = -(width - width / 2);
    // The reference emits `frame*height*width` frame entries but one h/w grid; for
    // frame == 1 (every block the layout produces) they coincide token by token.
    if (frame != 1 && block_tokens != height * width) return B200_ERR_LAYOUT;
    for (int64_t hh = 0; hh < height; ++hh)
      for (int64_t ww = 0; ww < width; ++ww)
        if (!push(frame_pos, h_start + hh, w_start + ww)) return B200_ERR_LAYOUT;
    cursor += block_tokens;
  }
  for (int64_t k = cursor; k < seq_len; ++k) {
    if (!push(position, position, position)) return B200_ERR_LAYOUT;
    ++position;
  }
  return n == seq_len ? B200_OK : B200_ERR_LAYOUT;
}

extern "C" int b200_rope_pe(const int32_t* img_shapes, int32_t n_shapes,
                            const uint8_t* image_pad_mask, int32_t seq_len, const int32_t axes[3],
                            float theta, float* pe_out) {
  if (!axes || seq_len < 0 || (seq_len > 0 && !pe_out)) return B200_ERR_INVALID;
  for (int a = 0; a < 3; ++a)
    if (axes[a] <= 0 || axes[a] % 2 != 0) return B200_ERR_INVALID;
  if (!(theta > 0.f)) return B200_ERR_INVALID;
  std::vector<int64_t> pos(static_cast<size_t>(seq_len) * 3);
  int rc = b200_rope_positions(img_shapes, n_shapes, image_pad_mask, seq_len, pos.data());
  if (rc != B200_OK) return rc;
  const int width = axes[0] + axes[1] + axes[2];
  // inv_freq_i = exp(i * (-2 ln(theta) / dim)) in f32 (src/rope.rs:52-58); the angle is
  // position * inv_freq in f32 (rope.rs:60-63); cos / sin of the f32 angle (rope.rs:92-96).
  std::vector<float> inv[3];
  for (int a = 0; a < 3; ++a) {
    const int half = axes[a] / 2;
    const float coef = static_cast<float>(-2.0 * std::log(static_cast<double>(theta)) / axes[a]);
    inv[a].resize(half);
    for (int i = 0; i < half; ++i) inv[a][i] = std::exp(static_cast<float>(i) * coef);
  }
  for (int64_t t = 0; t < seq_len; ++t) {
    float* row = pe_out + t * width;
    int col = 0;
    for (int a = 0; a < 3; ++a) {
      const int64_t p = pos[3 * t + a];
      if (p < -kTableNeg || p >= kTablePos) return B200_ERR_LAYOUT;  // outside the tables
      const float pf = static_cast<float>(p);
      for (size_t i = 0; i < inv[a].size(); ++i) {
        const float ang = pf * inv[a][i];
        row[col++] = std::cos(ang);
        row[col++] = std::sin(ang);
      }
    }
  }
  return B200_OK;
}

extern "C" int b200_key_valid_to_desc(const uint8_t* key_valid, int32_t batch,
                                      int32_t prefix_len, int32_t target_len,
                                      b200_kv_desc* desc_out) {
  if (batch < 0 || prefix_len < 0 || target_len < 0) return B200_ERR_INVALID;
  if (batch > 0 && (!key_valid || !desc_out)) return B200_ERR_INVALID;
  const int64_t L = static_cast<int64_t>(prefix_len) + target_len;
  for (int b = 0; b < batch; ++b) {
    const uint8_t* row = key_valid + b * L;
    int32_t pv = 0;
    while (pv < prefix_len && row[pv]) ++pv;
    for (int64_t k = pv; k < prefix_len; ++k)
      if (row[k]) return B200_ERR_LAYOUT;  // a hole inside the prefix
    for (int64_t k = prefix_len; k < L; ++k)
      if (!row[k]) return B200_ERR_LAYOUT;  // target keys are always valid in the reference
    desc_out[b].prefix_valid = pv;
    desc_out[b].target_valid = target_len;
  }
  return B200_OK;
}

extern "C" int b200_block_causal_limits(const int64_t* image_ids, int32_t len,
                                        int32_t* limits_out) {
  if (len < 0 || (len > 0 && (!image_ids || !limits_out))) return B200_ERR_INVALID;
  int32_t i = 0;
  while (i < len) {
    if (image_ids[i] < 0) {  // text: causal
      limits_out[i] = i + 1;
      ++i;
      continue;
    }
    int32_t e = i;  // image block [i, e): every token sees the whole block and all before it
    while (e < len && image_ids[e] == image_ids[i]) ++e;
    for (int32_t r = i; r < e; ++r) limits_out[r] = e;
    i = e;
  }
  return B200_OK;
}

extern "C" const char* b200_strerror(int status) {
  switch (status) {
    case B200_OK: return "ok";
    case B200_ERR_INVALID: return "invalid argument (null, negative size or misaligned pointer)";
    case B200_ERR_UNSUPPORTED: return "unsupported (head_dim must be 128; device must be sm_100)";
    case B200_ERR_CUDA: return "CUDA runtime or driver call failed";
    case B200_ERR_WORKSPACE: return "workspace missing or too small";
    case B200_ERR_LAYOUT: return "layout or mask not representable";
    case B200_ERR_DEVICE_TIMEOUT: return "a device-side wait ran out";
    default: return "unknown status";
  }
}

extern "C" const char* b200_attn_strerror(int status) { return b200_strerror(status); }

extern "C" int b200_abi_version(void) { return B200_ATTN_ABI_VERSION; }
