// Status codes, thread-local last-error message and version of libmkv.
#include <cuda.h>

#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <set>
#include <tuple>

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

namespace {
typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long*);
std::once_flag g_ctx_once;
CtxGetCurrentFn g_ctx_get_current = nullptr;
CtxGetIdFn g_ctx_get_id = nullptr;

void resolve_ctx_calls() {
  void* f = nullptr;
  cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
  if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
      q == cudaDriverEntryPointSuccess)
    g_ctx_get_current = (CtxGetCurrentFn)f;
  f = nullptr;
  q = cudaDriverEntryPointSymbolNotFound;
  if (cudaGetDriverEntryPoint("cuCtxGetId", &f, cudaEnableDefault, &q) == cudaSuccess &&
      q == cudaDriverEntryPointSuccess)
    g_ctx_get_id = (CtxGetIdFn)f;
}

std::mutex g_smem_mu;
std::set<std::tuple<const void*, unsigned long long, int>> g_smem_done;
}  // namespace

int current_context_id(unsigned long long* id) {
  std::call_once(g_ctx_once, resolve_ctx_calls);
  *id = 0;
  if (!g_ctx_get_current || !g_ctx_get_id)
    return set_error(MKV_ERR_CUDA, "cuCtxGetCurrent / cuCtxGetId are unavailable");
  CUcontext ctx = nullptr;
  if (g_ctx_get_current(&ctx) != CUDA_SUCCESS)
    return set_error(MKV_ERR_CUDA, "cuCtxGetCurrent failed");
  if (ctx == nullptr) return MKV_OK;
  if (g_ctx_get_id(ctx, id) != CUDA_SUCCESS) return set_error(MKV_ERR_CUDA, "cuCtxGetId failed");
  return MKV_OK;
}

int ensure_dynamic_smem(const void* func, int bytes, const char* what) {
  if (bytes <= 48 * 1024) return MKV_OK;
  unsigned long long id = 0;
  int st = current_context_id(&id);
  if (st != MKV_OK) return st;
  std::lock_guard<std::mutex> lock(g_smem_mu);
  if (id != 0 && g_smem_done.count(std::make_tuple(func, id, bytes))) return MKV_OK;
  cudaError_t e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return cuda_status(e, what);
  if (id == 0) {  // the runtime has just made the primary context current
    st = current_context_id(&id);
    if (st != MKV_OK) return st;
  }
  if (id != 0) g_smem_done.insert(std::make_tuple(func, id, bytes));
  return MKV_OK;
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
