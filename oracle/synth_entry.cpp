// synth_entry.cpp — the synthetic .myai writer exported from the oracle
// library (test infrastructure), so that the CPU reference arm of the
// benchmark can write its model without loading the CUDA library. It is
// compiled from the same source files as the library's writer
// (chalot_c1_b200/csrc/myai*.cpp, same compiler flags), so the files are
// byte-identical (tests/test_oracle.py checks this).
#include <string>

#include "capi_internal.h"

extern "C" __attribute__((visibility("default"))) int orc_write_synthetic(const char* path,
                                                                          const chalot_synth_spec* spec) {
  if (!path || !spec) return CHALOT_ERR_ARG;
  std::string err;
  return chalot::write_synthetic(path, *spec, &err);
}
