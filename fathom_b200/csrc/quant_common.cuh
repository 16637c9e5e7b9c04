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

constexpr int QS = D + 4;        // row stride of a staged tile: 16-byte aligned rows, conflict-free columns

// Block scales, codes and plane words of the staged tile (tile[r][c] = value of token 64*blk + r,
// channel c; pad tokens hold 0).  Called by all 256 threads of the CTA; thread (c, h) owns channel c
// and the 32 tokens of half h: its 32 values are read once into registers (column reads, conflict-free
// with the QS stride), the two halves' absmax meet in s_half, and the thread forms its four 32-bit
// plane half-words in registers.  Writes scales_blk / scales_k / planes32 / code where given.  Ends
// after a barrier only when `code` is written, so a caller that re-stages the tile (or s_half)
// must synchronise first.
__device__ __forceinline__ void quantise_tile(const float (*tile)[QS], float (*s_half)[D], uint8_t (*s_code)[D],
                                              int64_t bh, int64_t blk, int64_t n, int64_t nblk, int64_t nsb,
                                              int64_t sub, int amax_f16, uint8_t* __restrict__ code,
                                              void* __restrict__ scales_blk, int scales_blk_f32,
                                              uint32_t* __restrict__ planes32, uint16_t* __restrict__ scales_k) {
  const int tid = threadIdx.x;
  const int j = tid & (D - 1), h = tid >> 7;
  const bool real_blk = blk < nblk;
  const int64_t tok0 = blk * BLK;
  const int64_t sb = blk / sub, s_in = blk - sb * sub;
  float v[32];
  float a = 0.0f;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    v[i] = tile[h * 32 + i][j];
    a = fmaxf(a, fabsf(v[i]));
  }
  s_half[h][j] = a;
  __syncthreads();
  a = fmaxf(fmaxf(s_half[0][j], s_half[1][j]), 1e-8f);
  const __half a16 = __float2half_rn(a);
  const float aq = amax_f16 ? __half2float(a16) : a;
  const float step = aq * 0.125f;  // exact: power-of-two scaling
  if (h == 0) {
    if (real_blk && scales_blk) {
      const int64_t o = (bh * nblk + blk) * D + j;
      if (scales_blk_f32) reinterpret_cast<float*>(scales_blk)[o] = aq;
      else reinterpret_cast<__half*>(scales_blk)[o] = a16;
    }
    if (scales_k) scales_k[((bh * nsb + sb) * D + j) * sub + s_in] = real_blk ? __half_as_ushort(a16) : (uint16_t)0;
  }
  // tokens of this half that exist: pad tokens (and pad blocks) have code 0
  const int64_t rem = real_blk ? n - (tok0 + h * 32) : 0;
  const int live = rem <= 0 ? 0 : (rem >= 32 ? 32 : (int)rem);
  uint32_t w0 = 0, w1 = 0, w2 = 0, w3 = 0;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const uint32_t c = i < live ? (uint32_t)code_of(v[i], step) : 0u;
    w0 |= ((c >> 3) & 1u) << i;
    w1 |= ((c >> 2) & 1u) << i;
    w2 |= ((c >> 1) & 1u) << i;
    w3 |= (c & 1u) << i;
    if (code) s_code[h * 32 + i][j] = (uint8_t)c;
  }
  if (planes32) {
    uint32_t* o = planes32 + ((((bh * nsb + sb) * D + j) * NPLANES) * sub + s_in) * 2 + h;
    const int64_t ps = sub * 2;     // words between consecutive planes of one (block, channel)
    o[0] = w0;
    o[ps] = w1;
    o[2 * ps] = w2;
    o[3 * ps] = w3;
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
