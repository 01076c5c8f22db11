// capi.cpp — host-only part of the C ABI: error reporting, the .myai writer
// and header inspection.
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "capi_internal.h"
#include "myai.h"

namespace chalot {

namespace {
thread_local std::string g_last_error;
}

int set_error(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

void clear_error() { g_last_error.clear(); }

}  // namespace chalot

using namespace chalot;

extern "C" {

__attribute__((visibility("default"))) const char* chalot_last_error(void) {
  return g_last_error.c_str();
}

__attribute__((visibility("default"))) int chalot_abi_version(void) { return 100; }

__attribute__((visibility("default"))) int chalot_myai_write_synthetic(const char* path,
                                                                       const chalot_synth_spec* spec) {
  if (!path || !spec) return set_error(CHALOT_ERR_ARG, "null argument");
  std::string err;
  int rc = write_synthetic(path, *spec, &err);
  if (rc != CHALOT_OK) return set_error(rc, err);
  clear_error();
  return CHALOT_OK;
}

__attribute__((visibility("default"))) int chalot_myai_inspect(const char* path,
                                                               chalot_model_config* out) {
  if (!path || !out) return set_error(CHALOT_ERR_ARG, "null argument");
  FILE* f = std::fopen(path, "rb");
  if (!f) return set_error(CHALOT_ERR_IO, std::string("open: ") + path);
  uint8_t hdr[kHeaderSize];
  size_t n = std::fread(hdr, 1, sizeof hdr, f);
  std::fclose(f);
  FileHeader h;
  std::string err;
  if (!parse_header(hdr, n, &h, &err)) return set_error(CHALOT_ERR_FORMAT, err);
  ModelConfig c = config_from_header(h);
  WeightIndex w = build_index(c);
  std::memset(out, 0, sizeof *out);
  out->dim = uint32_t(c.dim);
  out->hidden_dim = uint32_t(c.hidden_dim);
  out->n_layers = uint32_t(c.n_layers);
  out->n_heads = uint32_t(c.n_heads);
  out->head_dim = uint32_t(c.head_dim);
  out->vocab_size = uint32_t(c.vocab_size);
  out->max_seq_len = uint32_t(c.max_seq_len);
  out->n_experts = uint32_t(c.n_experts);
  out->top_k = uint32_t(c.top_k);
  out->int4_group_size = uint32_t(c.int4_group_size);
  out->depth_router_layer = uint32_t(c.depth_router_layer);
  out->rope_theta = c.rope_theta;
  out->total_bytes = w.total_bytes;
  out->expert_bytes = w.layers.empty() || w.layers[0].experts.empty() ? 0 : w.layers[0].experts[0].bytes();
  clear_error();
  return CHALOT_OK;
}

// Checks a whole .myai file against what the reference's loader and the
// header fields imply: magic and version (header.rs:102-107), the flag bits
// (bit 0 quantized, bit 1 int4, bit 2 MoE; header.rs:40-71), the reserved
// bytes 32-127 of a v2 header (the reference writers leave them zero; a writer
// that packs the v2 fields right after the v1 ones, as train_distill.py:898-915
// does, leaves them there and max_seq_len in the flags word), the shape, and the
// exact file size from the tensor offsets (weight_index.rs:85-263), where
// validate_myai.py:99-129 accepts anything within a factor of two.
__attribute__((visibility("default"))) int chalot_myai_validate(const char* path, char* report, size_t cap) {
  if (!path) return set_error(CHALOT_ERR_ARG, "null argument");
  std::vector<std::string> errs, notes;
  FILE* f = std::fopen(path, "rb");
  if (!f) return set_error(CHALOT_ERR_IO, std::string("open: ") + path);
  uint8_t hdr[kHeaderSize];
  std::memset(hdr, 0, sizeof hdr);
  const size_t n = std::fread(hdr, 1, sizeof hdr, f);
  std::fseek(f, 0, SEEK_END);
  const long fsize = std::ftell(f);
  std::fclose(f);
  FileHeader h;
  std::string err;
  char buf[256];
  if (!parse_header(hdr, n, &h, &err)) {
    errs.push_back(err);
  } else {
    if (h.flags & ~0x7u) {
      std::snprintf(buf, sizeof buf,
                    "flags 0x%X set bits beyond quantized/int4/moe (0x7); a value like %u there is usually "
                    "max_seq_len written into the flags word",
                    h.flags, h.flags);
      errs.push_back(buf);
    }
    if (h.version >= 2) {
      int first = -1;
      for (int i = 32; i < 128; ++i)
        if (hdr[i]) {
          first = i;
          break;
        }
      if (first >= 0) {
        auto u = [&](int off) { return uint32_t(hdr[off]) | (uint32_t(hdr[off + 1]) << 8) |
                                       (uint32_t(hdr[off + 2]) << 16) | (uint32_t(hdr[off + 3]) << 24); };
        std::snprintf(buf, sizeof buf,
                      "reserved header bytes 32-127 are not zero (first at %d; u32 at 32..52: %u %u %u %u %u "
                      "%u): the v2 fields n_experts, top_k, group, depth_router_layer, max_seq_len, rope_theta*100 "
                      "belong at offsets 128-151",
                      first, u(32), u(36), u(40), u(44), u(48), u(52));
        errs.push_back(buf);
      }
      if (h.n_experts > 4096) {
        std::snprintf(buf, sizeof buf, "n_experts %u above 4096", h.n_experts);
        errs.push_back(buf);
      } else if (h.n_experts == 1) {  // header.rs:17: is_moe = n_experts >= 2, so 1 loads as dense
        notes.push_back("n_experts 1: read as a dense model (MoE needs 2 or more)");
      }
      if (h.n_experts >= 2 && (h.top_k == 0 || h.top_k > h.n_experts)) {
        std::snprintf(buf, sizeof buf, "top_k %u outside [1, n_experts = %u]", h.top_k, h.n_experts);
        errs.push_back(buf);
      }
      if ((h.flags & 0x4u) && h.n_experts < 2) errs.push_back("the MoE flag is set but n_experts < 2");
    }
    if (!h.dim || !h.hidden_dim || !h.n_layers || !h.n_heads || !h.vocab_size) {
      errs.push_back("a zero dimension (dim, hidden_dim, n_layers, n_heads, vocab_size)");
    } else if (h.dim % h.n_heads) {
      std::snprintf(buf, sizeof buf, "dim %u is not a multiple of n_heads %u", h.dim, h.n_heads);
      errs.push_back(buf);
    }
    if (errs.empty()) {
      const ModelConfig c = config_from_header(h);
      const WeightIndex w = build_index(c);
      if ((size_t)fsize < w.total_bytes) {
        std::snprintf(buf, sizeof buf, "file is %ld bytes; the header's shape needs %zu (%zu missing)", fsize,
                      w.total_bytes, w.total_bytes - (size_t)fsize);
        errs.push_back(buf);
      } else if ((size_t)fsize > w.total_bytes) {
        std::snprintf(buf, sizeof buf, "%zu bytes after the last tensor (the weights end at %zu)",
                      (size_t)fsize - w.total_bytes, w.total_bytes);
        notes.push_back(buf);
      }
    }
  }
  std::string rep;
  for (const auto& e : errs) rep += "error: " + e + "\n";
  for (const auto& e : notes) rep += "note: " + e + "\n";
  if (report && cap) {
    const size_t k = std::min(cap - 1, rep.size());
    std::memcpy(report, rep.data(), k);
    report[k] = 0;
  }
  if (!errs.empty()) return set_error(CHALOT_ERR_FORMAT, rep);
  clear_error();
  return CHALOT_OK;
}

}  // extern "C"
