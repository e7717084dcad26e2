// Error reporting shared by every C-ABI entry point.  Each entry point clears
// the thread's message, validates its arguments, and either enqueues work and
// returns ASTERQ_OK or returns a negative status with a message.
#include <string.h>

#include "asterq_internal.h"

namespace asterq {

static thread_local char g_last_error[512] = {0};

int set_error(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return status;
}

void clear_error() { g_last_error[0] = '\0'; }

int check_launch(const char* what) {
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return set_error(ASTERQ_ERR_CUDA, "%s: %s", what, cudaGetErrorString(err));
  return ASTERQ_OK;
}

}  // namespace asterq

extern "C" int asterq_version(void) { return ASTERQ_VERSION; }

extern "C" const char* asterq_last_error(void) { return asterq::g_last_error; }
