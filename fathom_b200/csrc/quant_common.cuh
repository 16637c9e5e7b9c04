// 4-bit block quantiser + bit-plane packer over one staged 64 x 128 fp32 tile, shared by the plain
// store build (pack.cu) and the KLT-rotated store build (klt.cu).
//
// Reference semantics (kernels/bitplane.py):
//   quantise_u4   :23-32  amax per (64-token block, channel), clamp >= 1e-8, rounded to fp16 when the
//                         scale dtype is fp16, s = amax/8, code = clamp(floor(x/s), -8, 7) + 8
//   pack_planes   :44-50  bit i of plane word (block b, channel j, plane p) = bit (3-p) of the
//                         code of token 64b+i; pad tokens have code 0
//   to_superblocks:60-65  [nblk][D][4] -> [nsb][D][4][SUB]; pad blocks are zero
#pragma once
#include "common.cuh"

namespace fathom {

template <typename T> __device__ __forceinline__ float load_elem(const T* p);
template <> __device__ __forceinline__ float load_elem<float>(const float* p) { return __ldg(p); }
template <> __device__ __forceinline__ float load_elem<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat162float(*p);
}
template <> __device__ __forceinline__ float load_elem<__half>(const __half* p) { return __half2float(*p); }

// Code of x for step s = amax/8: clamp(floor(x/s), -8, 7) + 8 with IEEE division.  A NaN
// quotient (0/0: the fp16 amax underflowed to 0) gives 0 -- the value torch's NaN -> uint8
// conversion yields on the reference's CPU path.
__device__ __forceinline__ int code_of(float x, float s) {
  float qv = __fdiv_rn(x, s);
  if (qv != qv) return 0;
  float f = fminf(fmaxf(floorf(qv), -8.0f), 7.0f);
  return (int)f + 8;
}

// Block scales, codes and plane words of the staged tile (tile[r][c] = value of token 64*blk + r,
// channel c; pad tokens hold 0).  Called by all 256 threads of the CTA; only reads the tile.  Writes
// scales_blk / scales_k / planes32 / code where given.  Ends after a barrier only when `code` is
// written, so a caller that re-stages the tile must synchronise first.
__device__ __forceinline__ void quantise_tile(const float (*tile)[D + 1], float* s_step, uint8_t (*s_code)[D],
                                              int64_t bh, int64_t blk, int64_t n, int64_t nblk, int64_t nsb,
                                              int64_t sub, int amax_f16, uint8_t* __restrict__ code,
                                              void* __restrict__ scales_blk, int scales_blk_f32,
                                              uint32_t* __restrict__ planes32, uint16_t* __restrict__ scales_k) {
  const int tid = threadIdx.x;
  const bool real_blk = blk < nblk;
  const int64_t tok0 = blk * BLK;
  const int64_t sb = blk / sub, s_in = blk - sb * sub;
  if (tid < D) {
    float a = 0.0f;
#pragma unroll 8
    for (int r = 0; r < BLK; ++r) a = fmaxf(a, fabsf(tile[r][tid]));
    a = fmaxf(a, 1e-8f);
    const __half a16 = __float2half_rn(a);
    const float aq = amax_f16 ? __half2float(a16) : a;
    s_step[tid] = aq * 0.125f;  // exact: power-of-two scaling
    if (real_blk && scales_blk) {
      const int64_t o = (bh * nblk + blk) * D + tid;
      if (scales_blk_f32) reinterpret_cast<float*>(scales_blk)[o] = aq;
      else reinterpret_cast<__half*>(scales_blk)[o] = a16;
    }
    if (scales_k) scales_k[((bh * nsb + sb) * D + tid) * sub + s_in] = real_blk ? __half_as_ushort(a16) : (uint16_t)0;
  }
  __syncthreads();

  const int warp = tid >> 5, lane = tid & 31;
  const int h = warp & 1;           // token half of the block: tokens 32h .. 32h+31
  const int c0 = (warp >> 1) * 32;  // 32 channels per warp pair
  const int r = h * 32 + lane;
  const bool tok_ok = real_blk && (tok0 + r) < n;
  for (int jj = 0; jj < 32; ++jj) {
    const int j = c0 + jj;
    const int c = tok_ok ? code_of(tile[r][j], s_step[j]) : 0;
    s_code[r][j] = (uint8_t)c;
    if (planes32) {
      const uint32_t b0 = __ballot_sync(0xffffffffu, (c >> 3) & 1);
      const uint32_t b1 = __ballot_sync(0xffffffffu, (c >> 2) & 1);
      const uint32_t b2 = __ballot_sync(0xffffffffu, (c >> 1) & 1);
      const uint32_t b3 = __ballot_sync(0xffffffffu, c & 1);
      if (lane < NPLANES) {
        const uint32_t b = lane == 0 ? b0 : lane == 1 ? b1 : lane == 2 ? b2 : b3;
        planes32[((((bh * nsb + sb) * D + j) * NPLANES + lane) * sub + s_in) * 2 + h] = b;
      }
    }
  }
  if (code && real_blk) {
    __syncthreads();
    const int64_t ntok = (n - tok0) < BLK ? (n - tok0) : BLK;
    uint32_t* dst = reinterpret_cast<uint32_t*>(code + (bh * n + tok0) * D);
    const uint32_t* src = reinterpret_cast<const uint32_t*>(&s_code[0][0]);
    for (int e = tid; e < ntok * (D / 4); e += blockDim.x) dst[e] = src[e];
  }
}

}  // namespace fathom
