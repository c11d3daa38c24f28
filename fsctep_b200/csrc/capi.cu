// Library-level C ABI: error reporting and capability queries.
#include <string>

#include "common.cuh"

namespace fsc {

static thread_local std::string g_last_error;

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

}  // namespace fsc

extern "C" {

const char* fsc_last_error(void) { return fsc::g_last_error.c_str(); }

int fsc_version(void) { return 1; }

int fsc_has_cuda(void) { return 1; }

}  // extern "C"
