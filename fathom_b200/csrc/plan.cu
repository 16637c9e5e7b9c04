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

// Six exclusive warp prefix sums at once (interleaved shuffles: one scan's latency); tot receives the
// warp totals.
__device__ __forceinline__ void warp_exclusive_scan6(int (&v)[6], int lane, int (&tot)[6]) {
  int x[6];
#pragma unroll
  for (int j = 0; j < 6; ++j) x[j] = v[j];
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
#pragma unroll
    for (int j = 0; j < 6; ++j) {
      const int y = __shfl_up_sync(0xffffffffu, x[j], o);
      if (lane >= o) x[j] += y;
    }
  }
#pragma unroll
  for (int j = 0; j < 6; ++j) {
    tot[j] = __shfl_sync(0xffffffffu, x[j], 31);
    v[j] = x[j] - v[j];
  }
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
  // The depth sum at a candidate mid; a small integer (<= 512): one warp reduction instruction, exact.
  // rint(x) is formed as (x + 1.5 * 2^23) - 1.5 * 2^23, which rounds half to even like rintf for
  // |x| < 2^22 (here |x| < 100; NaN and inf pass through as in rintf), and the lane's four clamped
  // depths are summed as floats: one conversion per evaluation instead of eight, whose pipe bounded
  // the loop (bisection 2.8 -> 1.8 us).
  constexpr float RINT_C = 12582912.0f;
  auto total_at = [&](float mid) {
    float cnt = 0.0f;
#pragma unroll
    for (int i = 0; i < CPL; ++i) {
      const float x = __fmul_rn(__fsub_rn(lg[i], mid), 0.5f);
      cnt = __fadd_rn(cnt, fminf(fmaxf(__fsub_rn(__fadd_rn(x, RINT_C), RINT_C), 0.0f), bm));
    }
    return (float)__reduce_add_sync(0xffffffffu, (int)cnt);
  };
  // Bisection, two steps per round: the round's mid and both mids the next step can take (lo, mid)
  // and (mid, hi) are evaluated together (three independent warp reductions in flight, where one
  // step's reduction latency bounded the loop), then the path is followed.  Every mid is formed from
  // the same (lo, hi) as in a one-step loop, so the final hi is bit for bit the same.
  float lo = -60.0f, hi = 60.0f;
  int it = 0;
  for (; it + 2 <= iters; it += 2) {
    const float m1 = __fmul_rn(__fadd_rn(lo, hi), 0.5f);
    const float mL = __fmul_rn(__fadd_rn(lo, m1), 0.5f);   // the next mid after hi = m1
    const float mH = __fmul_rn(__fadd_rn(m1, hi), 0.5f);   // the next mid after lo = m1
    const float t1 = total_at(m1), tL = total_at(mL), tH = total_at(mH);
    if (t1 > Br) {
      lo = m1;
      if (tH > Br) lo = mH;
      else hi = mH;
    } else {
      hi = m1;
      if (tL > Br) lo = mL;
      else hi = mL;
    }
  }
  if (it < iters) {
    const float mid = __fmul_rn(__fadd_rn(lo, hi), 0.5f);
    if (total_at(mid) > Br) lo = mid;
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

  // the lane's counts for the six compacted lists (active channels, pairs, the four depth classes),
  // prefix-summed over the warp together
  int sc[6] = {cnt_act, cnt_pair, 0, 0, 0, 0};
#pragma unroll
  for (int i = 0; i < CPL; ++i) {
#pragma unroll
    for (int c = 1; c <= NPLANES; ++c) sc[1 + c] += t[i] == c;
  }
  int tot6[6];
  warp_exclusive_scan6(sc, lane, tot6);
  int total = tot6[0];
  // active channels, ascending
  int pos = sc[0];
  int32_t* actb = act + bh * D;
#pragma unroll
  for (int i = 0; i < CPL; ++i)
    if (t[i] > 0) actb[pos++] = c0 + i;
#pragma unroll
  for (int i = 0; i < CPL; ++i)
    if (c0 + i >= total) actb[c0 + i] = 0;
  if (lane == 0) nact[bh] = total;

  // (channel, plane) pairs in channel order
  pos = sc[1];
  total = tot6[1];
  const int PD = D * bmax;
  int32_t* pb = pairs + bh * PD;
#pragma unroll
  for (int i = 0; i < CPL; ++i) {
#pragma unroll
    for (int p = 0; p < NPLANES; ++p)
      if (p < t[i]) pb[pos++] = (c0 + i) * bmax + p;
  }
  for (int e = lane; e < PD; e += 32)
    if (e >= total) pb[e] = 0;
  if (lane == 0) npairs[bh] = total;

  // per-depth channel lists
  for (int c = 1; c <= bmax; ++c) {
    pos = sc[1 + c];
    total = tot6[1 + c];
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
