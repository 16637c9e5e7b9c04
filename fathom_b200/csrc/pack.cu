// Store build: 4-bit quantiser + bit-plane packer + superblock order, fused (the quantiser and
// packer of one tile are quant_common.cuh's quantise_tile; kernels/bitplane.py:23-65).
//
// One CTA handles one 64-token block of one (batch, kv-head) row: it stages the 64x128 tile
// in shared memory, computes the 128 block scales, then each warp forms the plane words of
// 32 tokens x 32 channels with one warp ballot per (channel, plane).
#include "quant_common.cuh"

namespace fathom {
namespace {

// 16-byte vector of T -> 16 / sizeof(T) floats into the tile row
template <typename T> struct Vec;
template <> struct Vec<float> {
  static constexpr int N = 4;
  static __device__ __forceinline__ void put(const uint4& u, float* d) {
    *reinterpret_cast<float4*>(d) = make_float4(__uint_as_float(u.x), __uint_as_float(u.y), __uint_as_float(u.z),
                                                __uint_as_float(u.w));
  }
};
template <> struct Vec<__nv_bfloat16> {
  static constexpr int N = 8;
  static __device__ __forceinline__ void put(const uint4& u, float* d) {
    // bf16 -> fp32 is exact: the 16 bits become the high half
    reinterpret_cast<float4*>(d)[0] = make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xFFFF0000u),
                                                  __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xFFFF0000u));
    reinterpret_cast<float4*>(d)[1] = make_float4(__uint_as_float(u.z << 16), __uint_as_float(u.z & 0xFFFF0000u),
                                                  __uint_as_float(u.w << 16), __uint_as_float(u.w & 0xFFFF0000u));
  }
};
template <> struct Vec<__half> {
  static constexpr int N = 8;
  static __device__ __forceinline__ void put(const uint4& u, float* d) {
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
    const float2 c = __half22float2(*reinterpret_cast<const __half2*>(&u.z));
    const float2 e = __half22float2(*reinterpret_cast<const __half2*>(&u.w));
    reinterpret_cast<float4*>(d)[0] = make_float4(a.x, a.y, b.x, b.y);
    reinterpret_cast<float4*>(d)[1] = make_float4(c.x, c.y, e.x, e.y);
  }
};

// VEC: the tile is read with 16-byte loads (every row 16-byte aligned: checked by the launcher).
template <typename T, bool VEC>
__global__ void __launch_bounds__(256) quantise_pack_kernel(
    const T* __restrict__ K, int64_t n, int64_t k_stride_bh, int64_t nblk, int64_t nsb, int64_t sub, int amax_f16,
    uint8_t* __restrict__ code, void* __restrict__ scales_blk, int scales_blk_f32, uint32_t* __restrict__ planes32,
    uint16_t* __restrict__ scales_k) {
  __shared__ __align__(16) float tile[BLK][QS];
  __shared__ float s_half[2][D];
  __shared__ __align__(16) uint8_t s_code[BLK][D];

  const int64_t blk = blockIdx.x;
  const int64_t bh = blockIdx.y;
  const int tid = threadIdx.x;
  const bool real_blk = blk < nblk;
  const int64_t tok0 = blk * BLK;
  const T* Kb = K + bh * k_stride_bh;

  if (VEC) {
    constexpr int NV = Vec<T>::N;            // elements per 16-byte vector
    constexpr int VPR = D / NV;              // vectors per row
    constexpr int PER = BLK * VPR / 256;     // vectors per thread
    uint4 u[PER];
#pragma unroll
    for (int k = 0; k < PER; ++k) {          // all loads in flight before any use
      const int e = tid + k * 256;
      const int r = e / VPR, cv = e % VPR;
      const int64_t tok = tok0 + r;
      u[k] = (real_blk && tok < n) ? __ldg(reinterpret_cast<const uint4*>(Kb + tok * D) + cv) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      const int e = tid + k * 256;
      Vec<T>::put(u[k], &tile[e / VPR][(e % VPR) * NV]);
    }
  } else {
    for (int e = tid; e < BLK * D; e += blockDim.x) {
      const int r = e >> 7, c = e & (D - 1);
      const int64_t tok = tok0 + r;
      tile[r][c] = (real_blk && tok < n) ? load_elem<T>(Kb + tok * D + c) : 0.0f;
    }
  }
  __syncthreads();

  quantise_tile(tile, s_half, s_code, bh, blk, n, nblk, nsb, sub, amax_f16, code, scales_blk, scales_blk_f32,
                planes32, scales_k);
}

__global__ void __launch_bounds__(256) pack_codes_kernel(const uint8_t* __restrict__ code, int64_t n, int64_t nblk,
                                                         int64_t nsb, int64_t sub, uint32_t* __restrict__ planes32) {
  __shared__ __align__(16) uint8_t tile[BLK][D + 4];
  const int64_t blk = blockIdx.x, bh = blockIdx.y;
  const int tid = threadIdx.x;
  const int64_t tok0 = blk * BLK;
  for (int e = tid; e < BLK * D; e += blockDim.x) {
    const int r = e >> 7, c = e & (D - 1);
    const int64_t tok = tok0 + r;
    tile[r][c] = (blk < nblk && tok < n) ? code[(bh * n + tok) * D + c] : (uint8_t)0;
  }
  __syncthreads();
  const int64_t sb = blk / sub, s_in = blk - sb * sub;
  const int warp = tid >> 5, lane = tid & 31;
  const int h = warp & 1, c0 = (warp >> 1) * 32;
  for (int jj = 0; jj < 32; ++jj) {
    const int j = c0 + jj;
    const int c = tile[h * 32 + lane][j];
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

__global__ void __launch_bounds__(D) unpack_kernel(const uint64_t* __restrict__ planes, int64_t n, int64_t nsb,
                                                   int64_t sub, uint8_t* __restrict__ code) {
  const int64_t blk = blockIdx.x, bh = blockIdx.y;
  const int j = threadIdx.x;
  const int64_t sb = blk / sub, s_in = blk - sb * sub;
  uint64_t w[NPLANES];
#pragma unroll
  for (int p = 0; p < NPLANES; ++p) w[p] = planes[(((bh * nsb + sb) * D + j) * NPLANES + p) * sub + s_in];
  const int64_t tok0 = blk * BLK;
  const int ntok = (int)((n - tok0) < BLK ? (n - tok0) : BLK);
  for (int i = 0; i < ntok; ++i) {
    const uint32_t c = (uint32_t)(((w[0] >> i) & 1) << 3 | ((w[1] >> i) & 1) << 2 | ((w[2] >> i) & 1) << 1 |
                                  ((w[3] >> i) & 1));
    code[(bh * n + tok0 + i) * D + j] = (uint8_t)c;
  }
}

__global__ void relayout_planes_kernel(const uint64_t* __restrict__ src, int64_t BH, int64_t nblk, int64_t sub_s,
                                       int64_t nsb_s, uint64_t* __restrict__ dst, int64_t sub_d, int64_t nsb_d) {
  const int64_t total = BH * nsb_d * D * NPLANES * sub_d;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    int64_t r = e;
    const int64_t s = r % sub_d; r /= sub_d;
    const int64_t p = r % NPLANES; r /= NPLANES;
    const int64_t j = r % D; r /= D;
    const int64_t sb = r % nsb_d;
    const int64_t bh = r / nsb_d;
    const int64_t blk = sb * sub_d + s;
    uint64_t v = 0;
    if (blk < nblk) {
      const int64_t sbs = blk / sub_s, ss = blk - sbs * sub_s;
      v = src[(((bh * nsb_s + sbs) * D + j) * NPLANES + p) * sub_s + ss];
    }
    dst[e] = v;
  }
}

__global__ void relayout_scales_kernel(const uint16_t* __restrict__ src, int64_t BH, int64_t nblk, int64_t sub_s,
                                       int64_t nsb_s, uint16_t* __restrict__ dst, int64_t sub_d, int64_t nsb_d) {
  const int64_t total = BH * nsb_d * D * sub_d;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    int64_t r = e;
    const int64_t s = r % sub_d; r /= sub_d;
    const int64_t j = r % D; r /= D;
    const int64_t sb = r % nsb_d;
    const int64_t bh = r / nsb_d;
    const int64_t blk = sb * sub_d + s;
    uint16_t v = 0;
    if (blk < nblk) {
      const int64_t sbs = blk / sub_s, ss = blk - sbs * sub_s;
      v = src[((bh * nsb_s + sbs) * D + j) * sub_s + ss];
    }
    dst[e] = v;
  }
}

int grid_stride_blocks(int64_t total) {
  int64_t b = cdiv(total, 256);
  return (int)(b < 148 * 32 ? (b < 1 ? 1 : b) : 148 * 32);
}

}  // namespace
}  // namespace fathom

using namespace fathom;

extern "C" int fathom_quantise_pack(const void* K, int k_dtype, int64_t BH, int64_t n, int64_t k_stride_bh,
                                    int64_t sub, int amax_f16, uint8_t* code, void* scales_blk, int scales_blk_f32,
                                    uint64_t* planes_k, uint16_t* scales_k, void* stream) {
  FATHOM_REQUIRE(K != nullptr, FATHOM_ERR_NULL, "quantise_pack: K is NULL");
  FATHOM_REQUIRE(BH >= 1 && BH <= 65535 && n >= 1 && sub >= 1, FATHOM_ERR_SHAPE,
                 "quantise_pack: need 1 <= BH <= 65535, n >= 1, sub >= 1 (BH=%lld n=%lld sub=%lld)", (long long)BH,
                 (long long)n, (long long)sub);
  FATHOM_REQUIRE(k_stride_bh >= n * D, FATHOM_ERR_SHAPE, "quantise_pack: k_stride_bh < n*128");
  FATHOM_REQUIRE((planes_k == nullptr) == (scales_k == nullptr), FATHOM_ERR_NULL,
                 "quantise_pack: planes_k and scales_k must both be given or both be NULL");
  const int64_t nblk = cdiv(n, BLK);
  const int64_t nsb = cdiv(nblk, sub);
  const int64_t grid_blocks = planes_k ? nsb * sub : nblk;
  FATHOM_REQUIRE(grid_blocks <= 0x7fffffffLL, FATHOM_ERR_SHAPE, "quantise_pack: too many blocks");
  dim3 grid((unsigned)grid_blocks, (unsigned)BH);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  uint32_t* p32 = reinterpret_cast<uint32_t*>(planes_k);
  const bool vec = (reinterpret_cast<uintptr_t>(K) & 15) == 0;
#define FATHOM_QP(TT)                                                                                                \
  {                                                                                                                 \
    const TT* Kt = static_cast<const TT*>(K);                                                                       \
    if (vec && (k_stride_bh * (int64_t)sizeof(TT)) % 16 == 0)                                                       \
      quantise_pack_kernel<TT, true><<<grid, 256, 0, st>>>(Kt, n, k_stride_bh, nblk, nsb, sub, amax_f16, code,      \
                                                           scales_blk, scales_blk_f32, p32, scales_k);              \
    else                                                                                                            \
      quantise_pack_kernel<TT, false><<<grid, 256, 0, st>>>(Kt, n, k_stride_bh, nblk, nsb, sub, amax_f16, code,     \
                                                            scales_blk, scales_blk_f32, p32, scales_k);             \
  }
  switch (k_dtype) {
    case FATHOM_DTYPE_F32:
      FATHOM_QP(float)
      break;
    case FATHOM_DTYPE_BF16:
      FATHOM_QP(__nv_bfloat16)
      break;
    case FATHOM_DTYPE_F16:
      FATHOM_QP(__half)
      break;
    default:
      return set_error(FATHOM_ERR_UNSUPPORTED, "quantise_pack: unknown k_dtype %d", k_dtype);
  }
#undef FATHOM_QP
  return check_launch("quantise_pack");
}

extern "C" int fathom_pack_codes(const uint8_t* code, int64_t BH, int64_t n, int64_t sub, uint64_t* planes_k,
                                 void* stream) {
  FATHOM_REQUIRE(code && planes_k, FATHOM_ERR_NULL, "pack_codes: NULL pointer");
  FATHOM_REQUIRE(BH >= 1 && BH <= 65535 && n >= 1 && sub >= 1, FATHOM_ERR_SHAPE, "pack_codes: bad shape");
  const int64_t nblk = cdiv(n, BLK), nsb = cdiv(nblk, sub);
  FATHOM_REQUIRE(nsb * sub <= 0x7fffffffLL, FATHOM_ERR_SHAPE, "pack_codes: too many blocks");
  dim3 grid((unsigned)(nsb * sub), (unsigned)BH);
  pack_codes_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(code, n, nblk, nsb, sub,
                                                                              reinterpret_cast<uint32_t*>(planes_k));
  return check_launch("pack_codes");
}

extern "C" int fathom_unpack_planes(const uint64_t* planes_k, int64_t BH, int64_t n, int64_t sub, uint8_t* code,
                                    void* stream) {
  FATHOM_REQUIRE(code && planes_k, FATHOM_ERR_NULL, "unpack_planes: NULL pointer");
  FATHOM_REQUIRE(BH >= 1 && BH <= 65535 && n >= 1 && sub >= 1, FATHOM_ERR_SHAPE, "unpack_planes: bad shape");
  const int64_t nblk = cdiv(n, BLK), nsb = cdiv(nblk, sub);
  FATHOM_REQUIRE(nblk <= 0x7fffffffLL, FATHOM_ERR_SHAPE, "unpack_planes: too many blocks");
  dim3 grid((unsigned)nblk, (unsigned)BH);
  unpack_kernel<<<grid, D, 0, reinterpret_cast<cudaStream_t>(stream)>>>(planes_k, n, nsb, sub, code);
  return check_launch("unpack_planes");
}

extern "C" int fathom_relayout(const uint64_t* planes_src, const uint16_t* scales_src, int64_t BH, int64_t nblk,
                               int64_t sub_src, uint64_t* planes_dst, uint16_t* scales_dst, int64_t sub_dst,
                               void* stream) {
  FATHOM_REQUIRE(BH >= 1 && nblk >= 1 && sub_src >= 1 && sub_dst >= 1, FATHOM_ERR_SHAPE, "relayout: bad shape");
  FATHOM_REQUIRE((planes_src == nullptr) == (planes_dst == nullptr) && (scales_src == nullptr) == (scales_dst == nullptr),
                 FATHOM_ERR_NULL, "relayout: source and destination must be given in pairs");
  const int64_t nsb_s = cdiv(nblk, sub_src), nsb_d = cdiv(nblk, sub_dst);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (planes_src) {
    const int64_t total = BH * nsb_d * D * NPLANES * sub_dst;
    relayout_planes_kernel<<<grid_stride_blocks(total), 256, 0, st>>>(planes_src, BH, nblk, sub_src, nsb_s, planes_dst,
                                                                      sub_dst, nsb_d);
  }
  if (scales_src) {
    const int64_t total = BH * nsb_d * D * sub_dst;
    relayout_scales_kernel<<<grid_stride_blocks(total), 256, 0, st>>>(scales_src, BH, nblk, sub_src, nsb_s, scales_dst,
                                                                      sub_dst, nsb_d);
  }
  return check_launch("relayout");
}
