// Status codes, thread-local last-error message and version of libmkv.
#include <cstdarg>
#include <cstdio>

#include "mkv_common.cuh"

namespace mkv {

static thread_local char g_last_error[512] = {0};

int set_error(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return status;
}

void clear_error() { g_last_error[0] = 0; }

int cuda_status(cudaError_t err, const char* what) {
  if (err == cudaSuccess) return MKV_OK;
  return set_error(MKV_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(err),
                   cudaGetErrorString(err));
}

}  // namespace mkv

extern "C" const char* mkv_version(void) { return "0.2.0"; }

// Hash of the sources and compiler flags this library was built from (set by build.py).
#ifndef MKV_SOURCE_HASH
#define MKV_SOURCE_HASH "unknown"
#endif
extern "C" const char* mkv_source_hash(void) { return MKV_SOURCE_HASH; }

extern "C" const char* mkv_status_string(int status) {
  switch (status) {
    case MKV_OK: return "MKV_OK";
    case MKV_ERR_INVALID_ARGUMENT: return "MKV_ERR_INVALID_ARGUMENT";
    case MKV_ERR_UNSUPPORTED: return "MKV_ERR_UNSUPPORTED";
    case MKV_ERR_WORKSPACE: return "MKV_ERR_WORKSPACE";
    case MKV_ERR_CUDA: return "MKV_ERR_CUDA";
    default: return "MKV_ERR_UNKNOWN";
  }
}

extern "C" const char* mkv_last_error(void) { return mkv::g_last_error; }
