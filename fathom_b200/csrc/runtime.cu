// Error reporting, ABI version and pinned mapped host memory.
#include "common.cuh"

#include <sys/mman.h>
#include <string.h>

#include <mutex>
#include <unordered_map>

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

extern "C" int fathom_abi_version(void) { return 2; }

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

namespace {
std::mutex g_reg_mutex;
struct Mapping {
  void* base;    // what mmap returned
  size_t span;   // what was mapped
  size_t size;   // the registered, 2 MB-aligned part
};
std::unordered_map<void*, Mapping> g_registered;   // mmap'd + cudaHostRegister'ed allocations
constexpr size_t HUGE_PAGE = 2u << 20;
}  // namespace

extern "C" int fathom_host_alloc_mapped_ex(size_t bytes, int flags, void** host_ptr, void** dev_ptr) {
  if (!(flags & FATHOM_HOST_HUGEPAGES)) return fathom_host_alloc_mapped(bytes, host_ptr, dev_ptr);
  FATHOM_REQUIRE(host_ptr && dev_ptr, FATHOM_ERR_NULL, "host_alloc_mapped_ex: NULL output pointer");
  FATHOM_REQUIRE(bytes > 0, FATHOM_ERR_SHAPE, "host_alloc_mapped_ex: zero bytes");
  *host_ptr = nullptr;
  *dev_ptr = nullptr;
  const size_t size = (bytes + HUGE_PAGE - 1) / HUGE_PAGE * HUGE_PAGE;
  const size_t span = size + HUGE_PAGE;     // room to start on a 2 MB boundary
  void* base = mmap(nullptr, span, PROT_READ | PROT_WRITE, MAP_PRIVATE | MAP_ANONYMOUS, -1, 0);
  if (base == MAP_FAILED) return set_error(FATHOM_ERR_CUDA, "host_alloc_mapped_ex: mmap(%zu) failed", span);
  void* h = reinterpret_cast<void*>((reinterpret_cast<uintptr_t>(base) + HUGE_PAGE - 1) & ~(uintptr_t)(HUGE_PAGE - 1));
  madvise(h, size, MADV_HUGEPAGE);   // a hint: the kernel may still use 4 KB pages
  memset(h, 0, size);                // fault the pages in before pinning
  cudaError_t e = cudaHostRegister(h, size, cudaHostRegisterMapped | cudaHostRegisterPortable);
  if (e != cudaSuccess) {
    munmap(base, span);
    return set_error(FATHOM_ERR_CUDA, "cudaHostRegister(%zu bytes) failed: %s", size, cudaGetErrorString(e));
  }
  void* d = nullptr;
  e = cudaHostGetDevicePointer(&d, h, 0);
  if (e != cudaSuccess) {
    cudaHostUnregister(h);
    munmap(base, span);
    return set_error(FATHOM_ERR_CUDA, "cudaHostGetDevicePointer failed: %s", cudaGetErrorString(e));
  }
  {
    std::lock_guard<std::mutex> lk(g_reg_mutex);
    g_registered[h] = Mapping{base, span, size};
  }
  *host_ptr = h;
  *dev_ptr = d;
  return FATHOM_OK;
}

extern "C" int fathom_host_free(void* host_ptr) {
  if (!host_ptr) return FATHOM_OK;
  Mapping m{nullptr, 0, 0};
  {
    std::lock_guard<std::mutex> lk(g_reg_mutex);
    auto it = g_registered.find(host_ptr);
    if (it != g_registered.end()) {
      m = it->second;
      g_registered.erase(it);
    }
  }
  if (m.base) {
    cudaError_t e = cudaHostUnregister(host_ptr);
    munmap(m.base, m.span);
    if (e != cudaSuccess) return set_error(FATHOM_ERR_CUDA, "cudaHostUnregister failed: %s", cudaGetErrorString(e));
    return FATHOM_OK;
  }
  cudaError_t e = cudaFreeHost(host_ptr);
  if (e != cudaSuccess) return set_error(FATHOM_ERR_CUDA, "cudaFreeHost failed: %s", cudaGetErrorString(e));
  return FATHOM_OK;
}
