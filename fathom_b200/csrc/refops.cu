// The reference module's torch helpers on the logical (code, block scale) layout, in CUDA:
//   dequant_planes         kernels/bitplane.py:34-42
//   scan_planes_reference  kernels/bitplane.py:357-363
//   scan_chan4_reference   kernels/bitplane.py:365-370
// These are the dense definitions of what the plane store and the scans compute; callers of the
// reference use them to check a store or to score without a plan.  Each value follows the
// reference's expression order in fp32:
//   val = ((c >> (4 - t)) + 0.5 - 2^(t-1)) * s / 2^(t-1)     (0 where t == 0)
// with the division done as an IEEE division, so dequant_planes is bit-exact.  The scans sum
// q[g][j] * val over the channels in ascending order with fused multiply-adds (the reference runs
// a matrix product whose order is the BLAS library's; both are fp32 sums of the same products).
#include "common.cuh"

namespace fathom {
namespace {

__device__ __forceinline__ float load_scale(const void* scales, int scales_f32, int64_t i) {
  return scales_f32 ? static_cast<const float*>(scales)[i]
                    : __half2float(__ushort_as_half(static_cast<const uint16_t*>(scales)[i]));
}

// t outside 0..4 is clamped (plans never hold other depths)
__device__ __forceinline__ float dequant_value(uint32_t code, int t, float s) {
  if (t <= 0) return 0.0f;
  t = t > NPLANES ? NPLANES : t;
  const float half = __uint_as_float((uint32_t)(127 + t - 1) << 23);   // 2^(t-1), exact
  const float ct = (float)(code >> (NPLANES - t));
  return __fdiv_rn(__fmul_rn(__fsub_rn(__fadd_rn(ct, 0.5f), half), s), half);
}

// One thread per (row, token, channel) element.
__global__ void dequant_kernel(const uint8_t* __restrict__ code, const void* __restrict__ scales, int scales_f32,
                               int64_t rows, int64_t n, const int32_t* __restrict__ t, int64_t t_stride_row,
                               float* __restrict__ out) {
  const int64_t total = rows * n * D;
  const int64_t nb = cdiv(n, BLK);
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t j = e % D;
    const int64_t tok = (e / D) % n;
    const int64_t r = e / (D * n);
    const int tj = t[r * t_stride_row + j];
    const float s = load_scale(scales, scales_f32, (r * nb + tok / BLK) * D + j);
    out[e] = dequant_value(code[e], tj, s);
  }
}

// CTA = 128 tokens of one row; thread = one token, all G query heads.  The CTA stages the row's
// queries, depths and the scales of its (at most 3) blocks in shared memory; the thread reads its
// token's 128 codes with 16-byte loads.  chan4 = 1: every channel at depth 4, multiplied by the
// channel's active flag (as the reference multiplies the dequantised keys by active.float()).
template <int G>
__global__ void __launch_bounds__(128) ref_scan_kernel(const float* __restrict__ q, const uint8_t* __restrict__ code,
                                                       const void* __restrict__ scales, int scales_f32, int64_t n,
                                                       const int32_t* __restrict__ t, const uint8_t* __restrict__ active,
                                                       int chan4, float* __restrict__ out) {
  __shared__ float s_q[G][D];
  __shared__ int s_t[D];
  __shared__ float s_on[D];
  __shared__ float s_sc[3][D];
  const int64_t r = blockIdx.y;
  const int64_t tok0 = (int64_t)blockIdx.x * 128;
  const int64_t nb = cdiv(n, BLK);
  const int64_t blk0 = tok0 / BLK;
  for (int e = threadIdx.x; e < G * D; e += blockDim.x) s_q[e / D][e % D] = q[r * G * D + e];
  for (int j = threadIdx.x; j < D; j += blockDim.x) {
    s_t[j] = chan4 ? NPLANES : t[r * D + j];
    s_on[j] = chan4 ? (active[r * D + j] ? 1.0f : 0.0f) : 1.0f;
  }
  for (int e = threadIdx.x; e < 3 * D; e += blockDim.x) {
    const int64_t b = blk0 + e / D;
    s_sc[e / D][e % D] = b < nb ? load_scale(scales, scales_f32, (r * nb + b) * D + e % D) : 0.0f;
  }
  __syncthreads();
  const int64_t tok = tok0 + threadIdx.x;
  if (tok >= n) return;
  const int sb = (int)(tok / BLK - blk0);
  float acc[G];
#pragma unroll
  for (int g = 0; g < G; ++g) acc[g] = 0.0f;
  const uint4* row = reinterpret_cast<const uint4*>(code + (r * n + tok) * D);
  for (int c = 0; c < D / 16; ++c) {
    const uint4 v = row[c];
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int u = 0; u < 16; ++u) {
      const int j = c * 16 + u;
      const int tj = s_t[j];
      if (tj <= 0) continue;
      float val = dequant_value((w[u >> 2] >> (8 * (u & 3))) & 0xFFu, tj, s_sc[sb][j]);
      if (chan4) val = __fmul_rn(val, s_on[j]);
#pragma unroll
      for (int g = 0; g < G; ++g) acc[g] = fmaf(s_q[g][j], val, acc[g]);
    }
  }
#pragma unroll
  for (int g = 0; g < G; ++g) out[(r * G + g) * n + tok] = acc[g];
}

int ref_scan(const float* q, int64_t BH, int G, int64_t n, const uint8_t* code, const void* scales, int scales_f32,
             const int32_t* t, const uint8_t* active, int chan4, float* out, cudaStream_t st) {
  FATHOM_REQUIRE(q && code && scales && out && (chan4 ? active != nullptr : t != nullptr), FATHOM_ERR_NULL,
                 "scan reference: NULL pointer");
  FATHOM_REQUIRE(BH >= 1 && BH <= 65535 && n >= 1, FATHOM_ERR_SHAPE, "scan reference: bad shape");
  FATHOM_REQUIRE(G >= 1 && G <= 8, FATHOM_ERR_UNSUPPORTED, "scan reference: G must be in 1..8 (got %d)", G);
  FATHOM_REQUIRE((reinterpret_cast<uintptr_t>(code) & 15) == 0, FATHOM_ERR_SHAPE,
                 "scan reference: codes must be 16-byte aligned");
  dim3 grid((unsigned)cdiv(n, 128), (unsigned)BH);
#define FATHOM_REF_CASE(GG)                                                                                \
  case GG:                                                                                                 \
    ref_scan_kernel<GG><<<grid, 128, 0, st>>>(q, code, scales, scales_f32, n, t, active, chan4, out); \
    break;
  switch (G) {
    FATHOM_REF_CASE(1)
    FATHOM_REF_CASE(2)
    FATHOM_REF_CASE(3)
    FATHOM_REF_CASE(4)
    FATHOM_REF_CASE(5)
    FATHOM_REF_CASE(6)
    FATHOM_REF_CASE(7)
    FATHOM_REF_CASE(8)
  }
#undef FATHOM_REF_CASE
  return check_launch(chan4 ? "scan_chan4_reference" : "scan_planes_reference");
}

}  // namespace
}  // namespace fathom

using namespace fathom;

extern "C" int fathom_dequant_planes(const uint8_t* code, const void* scales, int scales_f32, int64_t rows, int64_t n,
                                     const int32_t* t, int64_t t_stride_row, float* out, void* stream) {
  FATHOM_REQUIRE(code && scales && t && out, FATHOM_ERR_NULL, "dequant_planes: NULL pointer");
  FATHOM_REQUIRE(rows >= 1 && n >= 1 && (t_stride_row == 0 || t_stride_row == D), FATHOM_ERR_SHAPE,
                 "dequant_planes: bad shape (rows=%lld n=%lld t_stride_row=%lld)", (long long)rows, (long long)n,
                 (long long)t_stride_row);
  const int64_t total = rows * n * D;
  const int64_t blocks = cdiv(total, 256) < 148 * 16 ? cdiv(total, 256) : 148 * 16;
  dequant_kernel<<<(unsigned)blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(code, scales, scales_f32, rows,
                                                                                        n, t, t_stride_row, out);
  return check_launch("dequant_planes");
}

extern "C" int fathom_scan_planes_reference(const float* q, int64_t BH, int G, int64_t n, const uint8_t* code,
                                            const void* scales, int scales_f32, const int32_t* t, float* scores,
                                            void* stream) {
  return ref_scan(q, BH, G, n, code, scales, scales_f32, t, nullptr, 0, scores, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int fathom_scan_chan4_reference(const float* q, int64_t BH, int G, int64_t n, const uint8_t* code,
                                           const void* scales, int scales_f32, const uint8_t* active, float* scores,
                                           void* stream) {
  return ref_scan(q, BH, G, n, code, scales, scales_f32, nullptr, active, 1, scores,
                  reinterpret_cast<cudaStream_t>(stream));
}
