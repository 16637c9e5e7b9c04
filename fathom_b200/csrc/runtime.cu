// Error reporting, ABI version and pinned mapped host memory.
#include "common.cuh"

namespace fathom {

static thread_local char g_last_error[512] = "";

int set_error(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return status;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(FATHOM_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return FATHOM_OK;
}

}  // namespace fathom

using namespace fathom;

extern "C" const char* fathom_last_error(void) { return g_last_error; }

extern "C" int fathom_abi_version(void) { return 1; }

extern "C" int fathom_host_alloc_mapped(size_t bytes, void** host_ptr, void** dev_ptr) {
  FATHOM_REQUIRE(host_ptr && dev_ptr, FATHOM_ERR_NULL, "host_alloc_mapped: NULL output pointer");
  FATHOM_REQUIRE(bytes > 0, FATHOM_ERR_SHAPE, "host_alloc_mapped: zero bytes");
  *host_ptr = nullptr;
  *dev_ptr = nullptr;
  void* h = nullptr;
  cudaError_t e = cudaHostAlloc(&h, bytes, cudaHostAllocPortable | cudaHostAllocMapped);
  if (e != cudaSuccess)
    return set_error(FATHOM_ERR_CUDA, "cudaHostAlloc(%zu bytes) failed: %s", bytes, cudaGetErrorString(e));
  void* d = nullptr;
  e = cudaHostGetDevicePointer(&d, h, 0);
  if (e != cudaSuccess) {
    cudaFreeHost(h);
    return set_error(FATHOM_ERR_CUDA, "cudaHostGetDevicePointer failed: %s", cudaGetErrorString(e));
  }
  *host_ptr = h;
  *dev_ptr = d;
  return FATHOM_OK;
}

extern "C" int fathom_host_free(void* host_ptr) {
  if (!host_ptr) return FATHOM_OK;
  cudaError_t e = cudaFreeHost(host_ptr);
  if (e != cudaSuccess) return set_error(FATHOM_ERR_CUDA, "cudaFreeHost failed: %s", cudaGetErrorString(e));
  return FATHOM_OK;
}
