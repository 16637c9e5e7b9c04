// Per-query reverse water-filling plan (plan_kernel + make_plan, kernels/bitplane.py:83-116).
//
// t_j = clip(rint(log4(g_j / theta)), 0, bmax), theta found by `iters` bisection steps on
// log2(theta) over [-60, 60] so that sum_j t_j <= budget (the final depths use the upper end).
// One warp per (batch, kv-head) row; lane l owns channels 4l .. 4l+3, so every compacted list
// is a warp prefix sum in channel order.  All arithmetic is float32 with explicit round-to-
// nearest intrinsics (no contraction), rint is round-half-even, and log2 is evaluated in double
// and rounded to float.
#include "common.cuh"

namespace fathom {
namespace {

constexpr int CPL = D / 32;  // channels per lane

__device__ __forceinline__ int warp_exclusive_scan(int v, int lane, int* total) {
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  *total = __shfl_sync(0xffffffffu, x, 31);
  return x - v;
}

__global__ void __launch_bounds__(128) plan_kernel(const float* __restrict__ g, const float* __restrict__ budget,
                                                   int64_t BH, int bmax, int iters, int8_t* __restrict__ t_out,
                                                   int32_t* __restrict__ pairs, int32_t* __restrict__ npairs,
                                                   int32_t* __restrict__ act, int32_t* __restrict__ nact,
                                                   int32_t* __restrict__ cls, int32_t* __restrict__ clsn) {
  const int lane = threadIdx.x & 31;
  const int64_t bh = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (bh >= BH) return;

  float lg[CPL];
#pragma unroll
  for (int i = 0; i < CPL; ++i) {
    const float gv = fmaxf(g[bh * D + lane * CPL + i], 1e-30f);
    lg[i] = (float)log2((double)gv);
  }
  const float Br = budget[bh];
  const float bm = (float)bmax;
  float lo = -60.0f, hi = 60.0f;
  for (int it = 0; it < iters; ++it) {
    const float mid = __fmul_rn(__fadd_rn(lo, hi), 0.5f);
    int cnt = 0;
#pragma unroll
    for (int i = 0; i < CPL; ++i) cnt += (int)fminf(fmaxf(rintf(__fmul_rn(__fsub_rn(lg[i], mid), 0.5f)), 0.0f), bm);
    // the depth sum is a small integer (<= 512): one warp reduction instruction, exact
    const float tot = (float)__reduce_add_sync(0xffffffffu, cnt);
    if (tot > Br) lo = mid;
    else hi = mid;
  }
  int t[CPL];
#pragma unroll
  for (int i = 0; i < CPL; ++i) t[i] = (int)fminf(fmaxf(rintf(__fmul_rn(__fsub_rn(lg[i], hi), 0.5f)), 0.0f), bm);

  const int c0 = lane * CPL;
  int cnt_act = 0, cnt_pair = 0;
#pragma unroll
  for (int i = 0; i < CPL; ++i) {
    t_out[bh * D + c0 + i] = (int8_t)t[i];
    cnt_act += t[i] > 0;
    cnt_pair += t[i];
  }

  int total;
  // active channels, ascending
  int pos = warp_exclusive_scan(cnt_act, lane, &total);
  int32_t* actb = act + bh * D;
#pragma unroll
  for (int i = 0; i < CPL; ++i)
    if (t[i] > 0) actb[pos++] = c0 + i;
#pragma unroll
  for (int i = 0; i < CPL; ++i)
    if (c0 + i >= total) actb[c0 + i] = 0;
  if (lane == 0) nact[bh] = total;

  // (channel, plane) pairs in channel order
  pos = warp_exclusive_scan(cnt_pair, lane, &total);
  const int PD = D * bmax;
  int32_t* pb = pairs + bh * PD;
#pragma unroll
  for (int i = 0; i < CPL; ++i)
    for (int p = 0; p < t[i]; ++p) pb[pos++] = (c0 + i) * bmax + p;
  for (int e = lane; e < PD; e += 32)
    if (e >= total) pb[e] = 0;
  if (lane == 0) npairs[bh] = total;

  // per-depth channel lists
  for (int c = 1; c <= bmax; ++c) {
    int cnt = 0;
#pragma unroll
    for (int i = 0; i < CPL; ++i) cnt += t[i] == c;
    pos = warp_exclusive_scan(cnt, lane, &total);
    int32_t* cb = cls + (bh * bmax + (c - 1)) * D;
#pragma unroll
    for (int i = 0; i < CPL; ++i)
      if (t[i] == c) cb[pos++] = c0 + i;
#pragma unroll
    for (int i = 0; i < CPL; ++i)
      if (c0 + i >= total) cb[c0 + i] = 0;
    if (lane == 0) clsn[bh * bmax + (c - 1)] = total;
  }
}

}  // namespace
}  // namespace fathom

using namespace fathom;

extern "C" int fathom_make_plan(const float* g, const float* budget, int64_t BH, int bmax, int iters, int8_t* t,
                                int32_t* pairs, int32_t* npairs, int32_t* act, int32_t* nact, int32_t* cls,
                                int32_t* clsn, void* stream) {
  FATHOM_REQUIRE(g && budget && t && pairs && npairs && act && nact && cls && clsn, FATHOM_ERR_NULL,
                 "make_plan: NULL pointer");
  FATHOM_REQUIRE(BH >= 1, FATHOM_ERR_SHAPE, "make_plan: BH must be >= 1");
  FATHOM_REQUIRE(bmax >= 1 && bmax <= NPLANES, FATHOM_ERR_SHAPE, "make_plan: bmax must be in 1..4 (got %d)", bmax);
  FATHOM_REQUIRE(iters >= 0, FATHOM_ERR_SHAPE, "make_plan: iters must be >= 0");
  const int64_t grid = cdiv(BH, 4);
  FATHOM_REQUIRE(grid <= 0x7fffffffLL, FATHOM_ERR_SHAPE, "make_plan: BH too large");
  plan_kernel<<<(unsigned)grid, 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(g, budget, BH, bmax, iters, t, pairs,
                                                                                    npairs, act, nact, cls, clsn);
  return check_launch("make_plan");
}
