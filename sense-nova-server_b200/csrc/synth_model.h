// The tensors of a synthetic model, in the naming and shapes of the reference's
// converter (convert.rs:228-313 `plan`, :205-226 `plan_mtp`), with the value rule of
// each f32 segment. Shared by the GPU engine's generator and the CPU checker so both
// build the same model from a seed.
#pragma once
#include <stddef.h>
#include <stdint.h>

#include <string>

#include "snl_b200.h"

namespace snl_synth {

struct Seg {
  uint32_t sub;  // sub-stream of the tensor's key
  size_t n;      // elements
  float mult, offset;
};

inline size_t q_dim(const snl_model_config& c) { return (size_t)c.n_heads * c.head_dim; }
inline size_t kv_dim(const snl_model_config& c) { return (size_t)c.n_kv_heads * c.head_dim; }
inline size_t lin_value_dim(const snl_model_config& c) { return (size_t)c.lin_v_heads * c.lin_v_dim; }
inline size_t conv_dim(const snl_model_config& c) {
  return 2 * (size_t)c.lin_k_heads * c.lin_k_dim + lin_value_dim(c);
}
inline size_t lin_proj_rows(const snl_model_config& c) {
  return conv_dim(c) + lin_value_dim(c) + 2 * (size_t)c.lin_v_heads;
}
inline size_t attn_proj_rows(const snl_model_config& c) { return 2 * q_dim(c) + 2 * kv_dim(c); }
inline bool is_mhc(const snl_model_config& c, size_t l) {
  return c.mhc_start >= 0 && (size_t)c.mhc_start <= l && l < (size_t)c.mhc_end;
}

// quant(name, dtype, rows, cols) for block-quantized matrices; vec(name, segs, nseg)
// for f32 tensors made of consecutive segments.
template <class Q, class V>
void for_each_tensor(const snl_model_config& c, bool mtp, int quant, Q&& qf, V&& vf) {
  const size_t h = c.hidden, I = c.intermediate;
  qf(std::string("embed"), (int)SNL_Q8_0, (size_t)c.vocab, h);
  qf(std::string("lm_head"), (int)SNL_Q8_0, (size_t)c.vocab, h);
  Seg nrm[1] = {{0, h, 0.1f, 0.f}};
  vf(std::string("norm"), nrm, 1);
  for (size_t i = 0; i < c.n_layers; i++) {
    const std::string L = "l" + std::to_string(i) + ".";
    vf(L + "in_ln", nrm, 1);
    vf(L + "post_ln", nrm, 1);
    if (c.full_attention[i]) {
      Seg qk[1] = {{0, 2 * (size_t)c.head_dim, 0.1f, 0.f}};
      vf(L + "qk_norm", qk, 1);
      qf(L + "qkv", quant, attn_proj_rows(c), h);
      qf(L + "o_proj", quant, h, q_dim(c));
    } else {
      const size_t cd = conv_dim(c), nv = c.lin_v_heads;
      // conv1d w | A_log | dt_bias | norm w (convert.rs:248-258)
      Seg lin[4] = {{0, cd * 4, 0.5f, 0.f}, {1, nv, 0.1f, 0.f}, {2, nv, 0.1f, 0.f}, {3, (size_t)c.lin_v_dim, 0.1f, 1.0f}};
      vf(L + "lin", lin, 4);
      qf(L + "in_proj", (int)SNL_Q8_0, lin_proj_rows(c), h);  // always 8-bit (convert.rs:286-298)
      qf(L + "out_proj", quant, h, lin_value_dim(c));
    }
    if (is_mhc(c, i)) {
      // router weight [8, 2H] then bias [8] (convert.rs:260-272, layers.wgsl:78-86)
      Seg mh[2] = {{0, 8 * 2 * h, 0.02f, 0.f}, {1, 8, 0.1f, 0.f}};
      vf(L + "mhc_attn", mh, 2);
      vf(L + "mhc_ffn", mh, 2);
    }
    qf(L + "gate_up", quant, 2 * I, h);
    qf(L + "down", quant, h, I);
  }
  if (mtp) {
    qf(std::string("mtp.fc_e"), (int)SNL_Q8_0, h, h);
    qf(std::string("mtp.fc_h"), (int)SNL_Q8_0, h, h);
    for (const char* n : {"mtp.norm_e", "mtp.norm_h", "mtp.norm", "mtp.in_ln", "mtp.post_ln"}) vf(std::string(n), nrm, 1);
    Seg qk[1] = {{0, 2 * (size_t)c.head_dim, 0.1f, 0.f}};
    vf(std::string("mtp.qk_norm"), qk, 1);
    qf(std::string("mtp.qkv"), (int)SNL_Q8_0, attn_proj_rows(c), h);
    qf(std::string("mtp.o_proj"), (int)SNL_Q8_0, h, q_dim(c));
    qf(std::string("mtp.gate_up"), (int)SNL_Q8_0, 2 * I, h);
    qf(std::string("mtp.down"), (int)SNL_Q8_0, h, I);
  }
}

}  // namespace snl_synth
