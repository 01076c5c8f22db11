// capi.cpp — host-only part of the C ABI: error reporting, the .myai writer
// and header inspection.
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

}  // extern "C"
