// Plane-prefix key scan (PlaneStore.scan / scan_planes_cls_kernel, kernels/bitplane.py:275-338).
//
//   score[bh, g, tok] = sum_j q[bh, g, j] * s_j(blk) * (c_t(tok, j) + 1/2 - 2^(t-1)) / 2^(t-1)
//
// over the channels j of depth t = t_j >= 1, where c_t = code >> (4 - t) is read from the first
// t bit planes only.  Rewriting the dequantiser with f = 1 + c_t / 2^t (a float whose top t
// mantissa bits ARE the t plane bits, assembled with shifts and ORs and no conversion):
//
//   value_t = s * (2 f + 2^-t - 3)   =>   score = sum_j (2 q_j s_j) f_j  +  sum_j q_j s_j (2^-t - 3)
//
// so each (token, channel) costs t shift+or pairs and one FMA per query head.
//
// Work split: a warp owns a group of consecutive 64-token blocks of one (batch, kv-head) row;
// each lane owns TPL tokens of one 32-bit plane half-word (TPL = 32: 16 blocks per warp, TPL = 16:
// 8 blocks per warp, used for G > 4 to bound registers).  For a (channel, plane) a warp's loads
// are consecutive 4-byte words, i.e. fully coalesced 128-byte (or 64-byte) segments in both the
// HBM order (sub = 16) and the host run order (sub = nblk).  Every lane keeps G x TPL fp32
// accumulators in registers; the query tile and the channel lists sit in shared memory.  The
// next channel's plane words are loaded before the current channel is consumed.
#include "common.cuh"

namespace fathom {
namespace {

constexpr int WARPS = 4;

template <int G, int TPL, int C>
__device__ __forceinline__ void scan_class(float (&acc)[G][TPL], float (&cst)[G], const float (*s_q)[D],
                                           const int* s_ch, int i0, int i1, const uint32_t* __restrict__ pbase,
                                           const uint16_t* __restrict__ sbase, int64_t chan_stride32,
                                           int64_t plane_stride32, int64_t sub, int bitoff, bool active) {
  if (i0 >= i1) return;
  constexpr float KC = (C == 1 ? 0.5f : C == 2 ? 0.25f : C == 3 ? 0.125f : 0.0625f) - 3.0f;
  uint32_t wn[C];
  uint16_t sn = 0;
  {
    const int ch = s_ch[i0];
#pragma unroll
    for (int p = 0; p < C; ++p) wn[p] = active ? __ldg(pbase + ch * chan_stride32 + p * plane_stride32) : 0u;
    sn = active ? __ldg(sbase + ch * sub) : (uint16_t)0;
  }
  for (int i = i0; i < i1; ++i) {
    const int ch = s_ch[i];
    uint32_t w[C];
#pragma unroll
    for (int p = 0; p < C; ++p) w[p] = wn[p] >> bitoff;
    const float sc = __half2float(__ushort_as_half(sn));
    if (i + 1 < i1) {
      const int chn = s_ch[i + 1];
#pragma unroll
      for (int p = 0; p < C; ++p) wn[p] = active ? __ldg(pbase + chn * chan_stride32 + p * plane_stride32) : 0u;
      sn = active ? __ldg(sbase + chn * sub) : (uint16_t)0;
    }
    float W[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float qs = s_q[g][ch] * sc;
      W[g] = 2.0f * qs;
      cst[g] = fmaf(qs, KC, cst[g]);
    }
#pragma unroll
    for (int k = 0; k < TPL; ++k) {
      uint32_t bits = 0x3F800000u;
#pragma unroll
      for (int p = 0; p < C; ++p) {
        const int sh = 22 - p - k;
        const uint32_t m = sh >= 0 ? (w[p] << sh) : (w[p] >> (-sh));
        bits |= m & (1u << (22 - p));
      }
      const float f = __uint_as_float(bits);
#pragma unroll
      for (int g = 0; g < G; ++g) acc[g][k] = fmaf(W[g], f, acc[g][k]);
    }
  }
}

template <int G, int TPL>
__global__ void __launch_bounds__(WARPS * 32, 2)
    scan_kernel(const float* __restrict__ q, const int32_t* __restrict__ cls, const int32_t* __restrict__ clsn,
                int bmax, const uint32_t* __restrict__ planes32, const uint16_t* __restrict__ scales, int64_t n,
                int64_t nblk, int64_t nsb, int64_t sub, int64_t blk_begin, int64_t blk_end, int64_t grp_begin,
                float* __restrict__ out) {
  constexpr int BPW = TPL == 32 ? 16 : 8;  // blocks per warp
  __shared__ float s_q[G][D];
  __shared__ int s_ch[D];
  __shared__ int s_start[NPLANES + 1];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t bh = blockIdx.y;
  for (int e = tid; e < G * D; e += blockDim.x) s_q[e / D][e % D] = q[bh * G * D + e];
  if (tid == 0) {
    int s = 0;
    for (int c = 1; c <= NPLANES; ++c) {
      s_start[c - 1] = s;
      s += c <= bmax ? clsn[bh * bmax + c - 1] : 0;
    }
    s_start[NPLANES] = s;
  }
  __syncthreads();
  for (int c = 1; c <= bmax; ++c) {
    const int cnt = s_start[c] - s_start[c - 1];
    for (int i = tid; i < cnt; i += blockDim.x) s_ch[s_start[c - 1] + i] = cls[(bh * bmax + c - 1) * D + i];
  }
  __syncthreads();

  const int64_t grp = grp_begin + (int64_t)blockIdx.x * WARPS + warp;
  const int64_t wblk0 = grp * BPW;
  const int64_t lo = blk_begin > wblk0 ? blk_begin : wblk0;
  const int64_t hi_lim = blk_end < nblk ? blk_end : nblk;
  if (lo >= hi_lim || wblk0 + BPW <= blk_begin) return;  // whole warp outside the range

  int64_t blk, half;
  int bitoff;
  if (TPL == 32) {
    blk = wblk0 + (lane >> 1);
    half = lane & 1;
    bitoff = 0;
  } else {
    blk = wblk0 + (lane >> 2);
    half = (lane >> 1) & 1;
    bitoff = (lane & 1) * 16;
  }
  const bool active = blk >= blk_begin && blk < hi_lim;
  const int64_t bsafe = active ? blk : lo;
  const int64_t sb = bsafe / sub, s_in = bsafe - sb * sub;
  const uint32_t* pbase = planes32 + ((bh * nsb + sb) * D * NPLANES * sub + s_in) * 2 + half;
  const uint16_t* sbase = scales + (bh * nsb + sb) * D * sub + s_in;
  const int64_t plane_stride32 = sub * 2;
  const int64_t chan_stride32 = NPLANES * sub * 2;

  float acc[G][TPL];
  float cst[G];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    cst[g] = 0.0f;
#pragma unroll
    for (int k = 0; k < TPL; ++k) acc[g][k] = 0.0f;
  }
  scan_class<G, TPL, 1>(acc, cst, s_q, s_ch, s_start[0], s_start[1], pbase, sbase, chan_stride32, plane_stride32, sub,
                        bitoff, active);
  scan_class<G, TPL, 2>(acc, cst, s_q, s_ch, s_start[1], s_start[2], pbase, sbase, chan_stride32, plane_stride32, sub,
                        bitoff, active);
  scan_class<G, TPL, 3>(acc, cst, s_q, s_ch, s_start[2], s_start[3], pbase, sbase, chan_stride32, plane_stride32, sub,
                        bitoff, active);
  scan_class<G, TPL, 4>(acc, cst, s_q, s_ch, s_start[3], s_start[4], pbase, sbase, chan_stride32, plane_stride32, sub,
                        bitoff, active);
  if (!active) return;

  const int64_t tok0 = blk * BLK + half * 32 + bitoff;
  const bool full = tok0 + TPL <= n;
  const bool vec = full && (n % 4 == 0) && ((reinterpret_cast<uintptr_t>(out) & 15) == 0);
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float* o = out + (bh * G + g) * n + tok0;
    if (vec) {
#pragma unroll
      for (int k = 0; k < TPL; k += 4)
        *reinterpret_cast<float4*>(o + k) =
            make_float4(acc[g][k] + cst[g], acc[g][k + 1] + cst[g], acc[g][k + 2] + cst[g], acc[g][k + 3] + cst[g]);
    } else {
#pragma unroll
      for (int k = 0; k < TPL; ++k)
        if (tok0 + k < n) o[k] = acc[g][k] + cst[g];
    }
  }
}

template <int G, int TPL>
int launch_scan(const float* q, int64_t BH, int64_t n, int64_t nblk, int64_t nsb, int64_t sub, const int32_t* cls,
                const int32_t* clsn, int bmax, const uint32_t* planes32, const uint16_t* scales, int64_t b0, int64_t b1,
                float* out, cudaStream_t st) {
  constexpr int BPW = TPL == 32 ? 16 : 8;
  const int64_t g0 = b0 / BPW, g1 = cdiv(b1, BPW);
  const int64_t grid_x = cdiv(g1 - g0, WARPS);
  FATHOM_REQUIRE(grid_x <= 0x7fffffffLL && BH <= 65535, FATHOM_ERR_SHAPE, "scan: grid too large");
  dim3 grid((unsigned)grid_x, (unsigned)BH);
  scan_kernel<G, TPL><<<grid, WARPS * 32, 0, st>>>(q, cls, clsn, bmax, planes32, scales, n, nblk, nsb, sub, b0, b1, g0,
                                                   out);
  return check_launch("scan");
}

}  // namespace
}  // namespace fathom

using namespace fathom;

extern "C" int fathom_scan(const float* q, int64_t BH, int G, int64_t n, int64_t sub, const int32_t* cls,
                           const int32_t* clsn, int bmax, const uint64_t* planes_k, const uint16_t* scales_k,
                           int64_t blk_begin, int64_t blk_end, float* scores, void* stream) {
  FATHOM_REQUIRE(q && cls && clsn && planes_k && scales_k && scores, FATHOM_ERR_NULL, "scan: NULL pointer");
  FATHOM_REQUIRE(BH >= 1 && BH <= 65535 && n >= 1 && sub >= 1, FATHOM_ERR_SHAPE, "scan: bad shape (BH=%lld n=%lld)",
                 (long long)BH, (long long)n);
  FATHOM_REQUIRE(G >= 1 && G <= 8, FATHOM_ERR_UNSUPPORTED, "scan: G must be in 1..8 (got %d)", G);
  FATHOM_REQUIRE(bmax >= 1 && bmax <= NPLANES, FATHOM_ERR_SHAPE, "scan: bmax must be in 1..4");
  const int64_t nblk = cdiv(n, BLK), nsb = cdiv(nblk, sub);
  FATHOM_REQUIRE(blk_begin >= 0 && blk_begin <= blk_end && blk_end <= nblk, FATHOM_ERR_SHAPE,
                 "scan: block range [%lld, %lld) outside [0, %lld]", (long long)blk_begin, (long long)blk_end,
                 (long long)nblk);
  if (blk_begin == blk_end) return FATHOM_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const uint32_t* p32 = reinterpret_cast<const uint32_t*>(planes_k);
#define FATHOM_SCAN_CASE(GG, TT) \
  case GG:                       \
    return launch_scan<GG, TT>(q, BH, n, nblk, nsb, sub, cls, clsn, bmax, p32, scales_k, blk_begin, blk_end, scores, st);
  switch (G) {
    FATHOM_SCAN_CASE(1, 32)
    FATHOM_SCAN_CASE(2, 32)
    FATHOM_SCAN_CASE(3, 32)
    FATHOM_SCAN_CASE(4, 32)
    FATHOM_SCAN_CASE(5, 16)
    FATHOM_SCAN_CASE(6, 16)
    FATHOM_SCAN_CASE(7, 16)
    FATHOM_SCAN_CASE(8, 16)
  }
#undef FATHOM_SCAN_CASE
  return set_error(FATHOM_ERR_UNSUPPORTED, "scan: G=%d", G);
}
