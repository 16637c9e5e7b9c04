// Shared helpers for the fathom_b200 CUDA library (sm_100a).
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdio.h>
#include <stdarg.h>

#include "../../include/fathom_b200.h"

namespace fathom {

constexpr int BLK = 64;     // tokens per block (one scale per block and channel)
constexpr int D = 128;      // head dimension of the store
constexpr int NPLANES = 4;  // 4-bit codes -> 4 bit planes

// Records a formatted message for fathom_last_error() and returns `status`.
int set_error(int status, const char* fmt, ...);

// Checks the launch status of the kernels just enqueued.
int check_launch(const char* what);

__host__ __device__ inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Order-preserving map float -> uint32 (larger float -> larger key; NaN above +inf).
__device__ __forceinline__ uint32_t f2key(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key2f(uint32_t k) {
  uint32_t u = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
  return __uint_as_float(u);
}
constexpr uint32_t KEY_NEG_INF = 0x007FFFFFu;   // f2key(-inf)

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

}  // namespace fathom

#define FATHOM_REQUIRE(cond, status, ...)                    \
  do {                                                       \
    if (!(cond)) return ::fathom::set_error((status), __VA_ARGS__); \
  } while (0)
