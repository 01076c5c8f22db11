// myai.cpp — .myai header parsing and tensor offset arithmetic.
// Follows src/model/header.rs:40-133, src/model/config.rs:40-69 and
// src/model/weight_index.rs:85-263 field for field; the body order and sizes
// must agree byte for byte because the file is shared with the reference.
#include "myai.h"

#include <cstdio>
#include <cstring>

namespace chalot {

static uint32_t rd32(const uint8_t* p) {
  return uint32_t(p[0]) | (uint32_t(p[1]) << 8) | (uint32_t(p[2]) << 16) |
         (uint32_t(p[3]) << 24);
}
static void wr32(uint8_t* p, uint32_t v) {
  p[0] = uint8_t(v);
  p[1] = uint8_t(v >> 8);
  p[2] = uint8_t(v >> 16);
  p[3] = uint8_t(v >> 24);
}

bool parse_header(const uint8_t* d, size_t len, FileHeader* h, std::string* err) {
  if (len < 128) {  // engine.rs:98-100
    if (err) *err = "File too small for header";
    return false;
  }
  FileHeader o;
  o.magic = rd32(d + 0);
  o.version = rd32(d + 4);
  o.dim = rd32(d + 8);
  o.hidden_dim = rd32(d + 12);
  o.n_layers = rd32(d + 16);
  o.n_heads = rd32(d + 20);
  o.vocab_size = rd32(d + 24);
  o.flags = rd32(d + 28);
  if (o.version >= 2 && len >= kHeaderSize) {  // header.rs:62-69
    o.n_experts = rd32(d + 128);
    o.top_k = rd32(d + 132);
    o.int4_group_size = rd32(d + 136);
    o.depth_router_layer = rd32(d + 140);
    o.max_seq_len = rd32(d + 144);
    o.rope_theta_x100 = rd32(d + 148);
  }
  char buf[96];
  if (o.magic != kMyaiMagic) {  // header.rs:102-104
    std::snprintf(buf, sizeof buf, "Bad magic: 0x%08X", o.magic);
    if (err) *err = buf;
    return false;
  }
  if (o.version == 0 || o.version > 2) {  // header.rs:105-107
    std::snprintf(buf, sizeof buf, "Unsupported version: %u", o.version);
    if (err) *err = buf;
    return false;
  }
  *h = o;
  return true;
}

void write_header(const FileHeader& h, uint8_t* b) {
  std::memset(b, 0, kHeaderSize);
  wr32(b + 0, h.magic);
  wr32(b + 4, h.version);
  wr32(b + 8, h.dim);
  wr32(b + 12, h.hidden_dim);
  wr32(b + 16, h.n_layers);
  wr32(b + 20, h.n_heads);
  wr32(b + 24, h.vocab_size);
  wr32(b + 28, h.flags);
  wr32(b + 128, h.n_experts);
  wr32(b + 132, h.top_k);
  wr32(b + 136, h.int4_group_size);
  wr32(b + 140, h.depth_router_layer);
  wr32(b + 144, h.max_seq_len);
  wr32(b + 148, h.rope_theta_x100);
}

ModelConfig config_from_header(const FileHeader& h) {
  ModelConfig c;
  c.dim = h.dim;
  c.hidden_dim = h.hidden_dim;
  c.n_layers = h.n_layers;
  c.n_heads = h.n_heads;
  c.head_dim = h.n_heads ? h.dim / h.n_heads : 0;
  c.vocab_size = h.vocab_size;
  c.n_experts = h.n_experts >= 2 ? h.n_experts : 1;
  size_t top_k = h.top_k >= 1 ? h.top_k : (c.n_experts < 2 ? c.n_experts : 2);
  c.top_k = top_k < c.n_experts ? top_k : c.n_experts;
  c.int4_group_size = h.int4_group_size > 0 ? h.int4_group_size : kDefaultInt4Group;
  c.max_seq_len = h.max_seq_len > 0 ? h.max_seq_len : kDefaultMaxSeq;
  c.depth_router_layer = h.depth_router_layer;
  // header.rs:127-133: the field holds theta*100, 0 selects 10000.
  c.rope_theta = h.rope_theta_x100 == 0 ? 10000.0f : float(h.rope_theta_x100) / 100.0f;
  return c;
}

size_t WeightIndex::expert_weight_bytes() const {
  size_t s = 0;
  for (const auto& l : layers)
    for (const auto& e : l.experts) s += e.bytes();
  return s;
}

WeightIndex build_index(const ModelConfig& cfg) {
  const size_t dim = cfg.dim, hidden = cfg.hidden_dim, vocab = cfg.vocab_size;
  const size_t group = cfg.int4_group_size;
  WeightIndex w;
  // weight_index.rs:92: the 256-byte header whenever MoE or int4 is in use.
  w.header_bytes = (cfg.is_moe() || group > 0) ? kHeaderSize : 128;
  size_t cur = w.header_bytes;
  w.embed_offset = cur;
  w.embed_bytes = vocab * dim;
  cur += w.embed_bytes;
  w.embed_scales_offset = cur;
  cur += vocab * 4;

  const size_t g = group ? group : 1;
  const size_t n_groups_dim = (dim + g - 1) / g;
  const size_t n_groups_hidden = (hidden + g - 1) / g;
  const size_t packed_dim = (dim + 1) / 2;
  const size_t packed_hidden = (hidden + 1) / 2;
  w.layers.resize(cfg.n_layers);
  for (auto& l : w.layers) {  // weight_index.rs:164-263
    l.rms_attn_offset = cur;
    cur += dim * 4;
    l.attn_qkv_offset = cur;
    l.attn_qkv_bytes = 3 * dim * dim;
    cur += l.attn_qkv_bytes;
    l.attn_qkv_scales_offset = cur;
    cur += 3 * dim * 4;
    l.attn_out_offset = cur;
    l.attn_out_bytes = dim * dim;
    cur += l.attn_out_bytes;
    l.attn_out_scales_offset = cur;
    cur += dim * 4;
    l.rms_ffn_offset = cur;
    cur += dim * 4;
    if (cfg.n_experts >= 2) {
      l.router_w_offset = cur;
      cur += cfg.n_experts * dim * 4;
      l.router_b_offset = cur;
      cur += cfg.n_experts * 4;
      l.router_bytes = cfg.n_experts * dim * 4 + cfg.n_experts * 4;
    }
    l.experts.resize(cfg.n_experts);
    for (auto& e : l.experts) {
      e.gate_up_offset = cur;
      e.gate_up_packed_bytes = 2 * hidden * packed_dim;
      cur += e.gate_up_packed_bytes;
      e.gate_up_scales_offset = cur;
      e.gate_up_scales_count = 2 * hidden * n_groups_dim;
      cur += e.gate_up_scales_count * 4;
      e.down_offset = cur;
      e.down_packed_bytes = dim * packed_hidden;
      cur += e.down_packed_bytes;
      e.down_scales_offset = cur;
      e.down_scales_count = dim * n_groups_hidden;
      cur += e.down_scales_count * 4;
    }
  }
  if (cfg.depth_router_layer > 0) {  // weight_index.rs:117-133
    w.depth_router_w1_offset = cur;
    cur += dim * kDepthRouterHidden * 4;
    w.depth_router_b1_offset = cur;
    cur += kDepthRouterHidden * 4;
    w.depth_router_w2_offset = cur;
    cur += kDepthRouterHidden * 4;
    w.depth_router_b2_offset = cur;
    cur += 4;
    w.depth_router_bytes = cur - w.depth_router_w1_offset;
  }
  w.final_norm_offset = cur;
  cur += dim * 4;
  w.output_proj_offset = cur;
  w.output_proj_bytes = vocab * dim;
  cur += w.output_proj_bytes;
  w.output_proj_scales_offset = cur;
  cur += vocab * 4;
  w.total_bytes = cur;
  return w;
}

}  // namespace chalot
