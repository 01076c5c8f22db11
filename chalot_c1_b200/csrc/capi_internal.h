// capi_internal.h — status codes and the per-thread error message shared by
// every translation unit behind the C ABI.
#pragma once

#include <string>

#include "../../include/chalot_b200.h"

namespace chalot {

// Records `msg` as the calling thread's last error and returns `code`.
int set_error(int code, const std::string& msg);
void clear_error();

int write_synthetic(const char* path, const chalot_synth_spec& spec, std::string* err);

}  // namespace chalot
