// Error reporting and version entry points of the C ABI.
#include "common.cuh"

namespace kb {
namespace {
thread_local char g_last_error[512] = "";
}

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

}  // namespace kb

extern "C" const char* kadllm_last_error(void) { return kb::g_last_error; }
extern "C" int kadllm_abi_version(void) { return 1; }
