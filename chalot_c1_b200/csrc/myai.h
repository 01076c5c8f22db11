// myai.h — the .myai v1/v2 weight-file format: header, runtime config and the
// byte offset of every tensor in the file.
//
// The on-disk format is the reference's and is read unchanged:
//   header      src/model/header.rs:40-71 (u32 LE fields; v2 fields at 128..152)
//   validation  src/model/header.rs:101-109 (magic "MYAI", version 1 or 2)
//   defaults    src/model/config.rs:40-69 (n_experts<2 -> 1, top_k default,
//               group 0 -> 64, max_seq 0 -> 512, rope_theta u32/100, 0 -> 10000)
//   offsets     src/model/weight_index.rs:85-263 (body order, sizes)
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

namespace chalot {

constexpr uint32_t kMyaiMagic = 0x4D594149u;  // "MYAI" read little-endian
constexpr size_t kHeaderSize = 256;           // v2 header (v1 files use 128)
constexpr size_t kDefaultMaxSeq = 512;        // src/model/constants.rs:7
constexpr size_t kDefaultInt4Group = 64;      // src/tensor/quantization.rs:110
constexpr size_t kDepthRouterHidden = 32;     // src/model/constants.rs:8
constexpr float kAttnLogitCap = 30.0f;        // src/model/constants.rs:10

struct FileHeader {
  uint32_t magic = 0, version = 0, dim = 0, hidden_dim = 0, n_layers = 0,
           n_heads = 0, vocab_size = 0, flags = 0;
  uint32_t n_experts = 0, top_k = 0, int4_group_size = 0,
           depth_router_layer = 0, max_seq_len = 0, rope_theta_x100 = 0;
};

// Parses the first `len` bytes of a file. Returns false with a message when
// the buffer is shorter than 128 bytes, the magic is wrong or the version is
// not 1 or 2 (the same conditions Engine::load rejects).
bool parse_header(const uint8_t* data, size_t len, FileHeader* out, std::string* err);
// Serialises a header into 256 bytes (src/model/header.rs:73-94).
void write_header(const FileHeader& h, uint8_t* buf256);

struct ModelConfig {
  size_t dim = 0, hidden_dim = 0, n_layers = 0, n_heads = 0, head_dim = 0,
         vocab_size = 0, max_seq_len = 0, n_experts = 1, top_k = 1,
         int4_group_size = kDefaultInt4Group, depth_router_layer = 0;
  float rope_theta = 10000.0f;
  bool is_moe() const { return n_experts >= 2; }
};

ModelConfig config_from_header(const FileHeader& h);

struct ExpertIndex {
  size_t gate_up_offset = 0, gate_up_packed_bytes = 0;
  size_t gate_up_scales_offset = 0, gate_up_scales_count = 0;
  size_t down_offset = 0, down_packed_bytes = 0;
  size_t down_scales_offset = 0, down_scales_count = 0;
  size_t bytes() const {
    return gate_up_packed_bytes + gate_up_scales_count * 4 + down_packed_bytes +
           down_scales_count * 4;
  }
};

struct LayerIndex {
  size_t rms_attn_offset = 0;
  size_t attn_qkv_offset = 0, attn_qkv_bytes = 0, attn_qkv_scales_offset = 0;
  size_t attn_out_offset = 0, attn_out_bytes = 0, attn_out_scales_offset = 0;
  size_t rms_ffn_offset = 0;
  size_t router_w_offset = 0, router_b_offset = 0, router_bytes = 0;
  std::vector<ExpertIndex> experts;
};

struct WeightIndex {
  size_t header_bytes = 0;
  size_t embed_offset = 0, embed_bytes = 0, embed_scales_offset = 0;
  std::vector<LayerIndex> layers;
  size_t depth_router_w1_offset = 0, depth_router_b1_offset = 0,
         depth_router_w2_offset = 0, depth_router_b2_offset = 0,
         depth_router_bytes = 0;
  size_t final_norm_offset = 0;
  size_t output_proj_offset = 0, output_proj_bytes = 0,
         output_proj_scales_offset = 0;
  size_t total_bytes = 0;
  size_t expert_weight_bytes() const;
};

WeightIndex build_index(const ModelConfig& cfg);

}  // namespace chalot
