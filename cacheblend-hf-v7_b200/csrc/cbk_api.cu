// C-ABI glue: per-thread error text, launch checks, per-device kernel attributes.
#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "cbk_common.cuh"

namespace cbk {

static thread_local char g_err[512] = "";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    return set_error(CBK_ERR_CUDA, "%s launch failed: %s", what, cudaGetErrorString(e));
  return CBK_OK;
}

// cudaFuncSetAttribute applies to the current device; remember per (function, device).
int ensure_smem_attr(const void* func, int bytes) {
  static std::mutex mu;
  static const void* funcs[64];
  static uint64_t done[64];
  static int n_funcs = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return set_error(CBK_ERR_CUDA, "cudaGetDevice failed");
  std::lock_guard<std::mutex> lock(mu);
  int slot = -1;
  for (int i = 0; i < n_funcs; ++i)
    if (funcs[i] == func) slot = i;
  if (slot < 0) {
    if (n_funcs == 64) return set_error(CBK_ERR_CUDA, "attribute table full");
    slot = n_funcs++;
    funcs[slot] = func;
    done[slot] = 0;
  }
  if (!(done[slot] & (1ull << dev))) {
    const cudaError_t e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess)
      return set_error(CBK_ERR_CUDA, "cudaFuncSetAttribute(%d bytes) failed: %s", bytes,
                       cudaGetErrorString(e));
    done[slot] |= 1ull << dev;
  }
  return CBK_OK;
}

}  // namespace cbk

extern "C" const char* cbk_last_error(void) { return cbk::g_err; }
extern "C" int cbk_abi_version(void) { return CBK_ABI_VERSION; }
