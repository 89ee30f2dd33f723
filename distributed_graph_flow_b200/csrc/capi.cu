// Error plumbing and version query of the dgfx C ABI.
#include <string>

#include "common.cuh"

namespace dgfx {
namespace {
thread_local std::string g_last_error;
}  // namespace

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

}  // namespace dgfx

extern "C" const char* dgfx_last_error(void) { return dgfx::g_last_error.c_str(); }
extern "C" int dgfx_version(void) { return 100; }
