// Internal: shared by select.cu and scan.cu (the scan writes the selection's group keys).
#pragma once
#include "common.cuh"

namespace fathom {
namespace selectk {

constexpr int HBITS = 12;
constexpr int NBINS = 1 << HBITS;
constexpr int CAP = 8192;          // candidates kept per row in the fast path
constexpr int MAX_KK = 4096;
constexpr int CHUNK = 16384;       // scores per CTA in the hist / collect passes
constexpr int HT = 512;            // threads of hist / collect CTAs
constexpr int FT = 512;            // threads of the finalize CTA

struct Workspace {
  uint32_t* hist;    // [rows][NBINS]
  uint32_t* count;   // [rows] candidates appended
  uint32_t* ticket;  // [rows] hist CTAs finished
  uint32_t* bstar;   // [rows] boundary bin
  uint64_t* cand;    // [rows][CAP]
};

constexpr size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

// hist, count and ticket start at zero; bstar and cand are written before they are read.
constexpr size_t zeroed_bytes(int64_t rows) {
  return align256(rows * NBINS * sizeof(uint32_t)) + 2 * align256(rows * sizeof(uint32_t));
}

constexpr size_t ws_bytes(int64_t rows) {
  return zeroed_bytes(rows) + align256(rows * sizeof(uint32_t)) + align256(rows * (size_t)CAP * sizeof(uint64_t));
}

// Group-maximum selection: one key per GROUP consecutive tokens of a row (the order-preserving key
// of the group's largest score), written by the scan's epilogue or by a pass over the scores.
// If at least kk groups have a key >= tau, at least kk distinct tokens do, so the boundary bin of
// the group keys bounds the kk-th largest token key from below; only the groups whose key reaches
// it are read again.  Used when the fully unmasked groups number at least 1.5 * kk.
constexpr int GROUP = 32;
constexpr int64_t n_groups(int64_t n) { return (n + GROUP - 1) / GROUP; }
constexpr size_t gkey_bytes(int64_t rows, int64_t n) { return align256(rows * n_groups(n) * sizeof(uint32_t)); }
// Workspace that serves both selection paths.
constexpr size_t select_ws_bytes(int64_t rows, int64_t n) {
  return ws_bytes(rows) > gkey_bytes(rows, n) ? ws_bytes(rows) : gkey_bytes(rows, n);
}
// Groups lying entirely inside the unmasked range [mask_lo, mask_hi) of a row of n tokens.
inline int64_t unmasked_groups(int64_t n, int64_t mask_lo, int64_t mask_hi) {
  const int64_t lo = mask_lo < 0 ? 0 : (mask_lo > n ? n : mask_lo);
  const int64_t hi = mask_hi < 0 ? 0 : (mask_hi > n ? n : mask_hi);
  const int64_t g_lo = (lo + GROUP - 1) / GROUP;
  const int64_t g_hi = hi == n ? n_groups(n) : hi / GROUP;
  return g_hi > g_lo ? g_hi - g_lo : 0;
}
inline bool group_select_applies(int64_t rows, int64_t n, int64_t kk, int64_t mask_lo, int64_t mask_hi,
                                 size_t workspace_bytes) {
  return 2 * unmasked_groups(n, mask_lo, mask_hi) >= 3 * kk && workspace_bytes >= gkey_bytes(rows, n);
}

inline Workspace carve(void* base, int64_t rows) {
  char* p = static_cast<char*>(base);
  Workspace w;
  w.hist = reinterpret_cast<uint32_t*>(p);
  p += align256(rows * NBINS * sizeof(uint32_t));
  w.count = reinterpret_cast<uint32_t*>(p);
  p += align256(rows * sizeof(uint32_t));
  w.ticket = reinterpret_cast<uint32_t*>(p);
  p += align256(rows * sizeof(uint32_t));
  w.bstar = reinterpret_cast<uint32_t*>(p);
  p += align256(rows * sizeof(uint32_t));
  w.cand = reinterpret_cast<uint64_t*>(p);
  return w;
}

// Boundary bin from a row histogram held in shared memory, with `nt` threads (multiple of 32).
// Returns (to every thread) the largest bin b with sum_{b' >= b} hist[b'] >= kk.
static __device__ int boundary_bin(const uint32_t* s_hist, int64_t kk, uint32_t* s_part, int* s_res) {
  const int nt = blockDim.x;
  const int per = NBINS / nt;
  const int t = threadIdx.x;
  uint32_t part = 0;
  for (int b = 0; b < per; ++b) part += s_hist[t * per + b];
  s_part[t] = part;
  __syncthreads();
  // inclusive suffix sums over threads (Hillis-Steele on shared memory)
  for (int o = 1; o < nt; o <<= 1) {
    const uint32_t v = (t + o < nt) ? s_part[t + o] : 0u;
    __syncthreads();
    s_part[t] += v;
    __syncthreads();
  }
  if (t == 0) *s_res = 0;
  __syncthreads();
  const uint32_t above = (t + 1 < nt) ? s_part[t + 1] : 0u;
  if (s_part[t] >= (uint32_t)kk && above < (uint32_t)kk) {
    uint32_t run = above;
    for (int b = (t + 1) * per - 1; b >= t * per; --b) {
      run += s_hist[b];
      if (run >= (uint32_t)kk) {
        *s_res = b;
        break;
      }
    }
  }
  __syncthreads();
  return *s_res;
}

// Block-wide exclusive scan of one value per thread (blockDim.x <= 1024). Returns the prefix;
// *total receives the block sum.
static __device__ uint32_t block_exclusive_scan(uint32_t v, uint32_t* s_warp, uint32_t* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  uint32_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) s_warp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    uint32_t w = lane < nw ? s_warp[lane] : 0u;
    uint32_t z = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, z, o);
      if (lane >= o) z += y;
    }
    if (lane < nw) s_warp[lane] = z - w;
    if (lane == 31) s_warp[32] = z;
  }
  __syncthreads();
  const uint32_t res = s_warp[warp] + x - v;
  *total = s_warp[32];
  __syncthreads();
  return res;
}


// Boundary bin of one row histogram (NBINS counters in global memory, read through L2), found by one
// warp: each lane sums 128 consecutive bins, a shuffle suffix-scan finds the lane holding the bin,
// which walks its bins from the top.  Returns (to every lane) the largest bin b with
// sum_{b' >= b} hist[b'] >= kk, or 0 if the row holds fewer than kk keys.
static __device__ int warp_boundary_bin(const uint32_t* hist, int64_t kk) {
  const int lane = threadIdx.x & 31;
  constexpr int PER = NBINS / 32;
  const uint4* h4 = reinterpret_cast<const uint4*>(hist + lane * PER);
  uint32_t part = 0;
#pragma unroll 8
  for (int i = 0; i < PER / 4; ++i) {
    const uint4 v = __ldcg(h4 + i);
    part += v.x + v.y + v.z + v.w;
  }
  uint32_t suffix = part;   // inclusive suffix sum over lanes >= this one
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_down_sync(0xffffffffu, suffix, o);
    if (lane + o < 32) suffix += y;
  }
  const uint32_t above = __shfl_down_sync(0xffffffffu, suffix, 1);
  const uint32_t above_l = lane < 31 ? above : 0u;
  int found = -1;
  if (suffix >= (uint32_t)kk && above_l < (uint32_t)kk) {
    uint32_t run = above_l;
    for (int b = PER - 1; b >= 0; --b) {
      run += __ldcg(hist + lane * PER + b);
      if (run >= (uint32_t)kk) {
        found = lane * PER + b;
        break;
      }
    }
  }
  const uint32_t m = __ballot_sync(0xffffffffu, found >= 0);
  return m ? __shfl_sync(0xffffffffu, found, __ffs(m) - 1) : 0;
}

// Boundary bin of a histogram in shared memory, found by the whole block (blockDim.x a multiple of 32
// that divides NBINS by a multiple of 4, at most 1024): returns to every thread the largest bin b with
// sum_{b' >= b} hist[b'] >= kk and the count strictly above b in *above_out; (0, 0) when the histogram
// holds fewer than kk.  Each thread sums NBINS/blockDim consecutive bins (16-byte loads), a block-wide
// suffix scan finds the one thread whose bins hold the crossing, which walks them.  s_tmp: 66 words.
static __device__ int block_boundary_bin(const uint32_t* hist, int64_t kk, uint32_t* s_tmp, uint32_t* above_out) {
  const int t = threadIdx.x, lane = t & 31, w = t >> 5, nw = blockDim.x >> 5;
  const int per = NBINS / blockDim.x;
  uint32_t part = 0;
  for (int i = 0; i < per; i += 4) {
    const uint4 v = *reinterpret_cast<const uint4*>(hist + t * per + i);
    part += v.x + v.y + v.z + v.w;
  }
  uint32_t suf = part;   // inclusive suffix sum over the lanes >= this one
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_down_sync(0xffffffffu, suf, o);
    if (lane + o < 32) suf += y;
  }
  if (lane == 0) s_tmp[w] = suf;
  __syncthreads();
  if (w == 0) {
    const uint32_t v = lane < nw ? s_tmp[lane] : 0u;
    uint32_t s2 = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_down_sync(0xffffffffu, s2, o);
      if (lane + o < 32) s2 += y;
    }
    s_tmp[32 + lane] = s2 - v;   // the warps above this one
    if (lane == 0) {
      s_tmp[64] = 0;
      s_tmp[65] = 0;
    }
  }
  __syncthreads();
  const uint32_t incl = suf + s_tmp[32 + w];
  const uint32_t above = incl - part;
  if (incl >= (uint32_t)kk && above < (uint32_t)kk) {
    uint32_t run = above;
    for (int i = per - 1; i >= 0; --i) {
      const uint32_t h = hist[t * per + i];
      if (run + h >= (uint32_t)kk) {
        s_tmp[64] = (uint32_t)(t * per + i);
        s_tmp[65] = run;
        break;
      }
      run += h;
    }
  }
  __syncthreads();
  const int b = (int)s_tmp[64];
  *above_out = s_tmp[65];
  __syncthreads();   // s_tmp may be reused by the caller
  return b;
}

// The whole selection over score rows: see select.cu.  With gkeys_ready the group keys are already in
// the workspace (written by the scan) and group_select_applies() held for these arguments.
int launch_select(const float* scores, int64_t rows, int64_t n, int64_t row_stride, int64_t kk, int64_t mask_lo,
                  int64_t mask_hi, int64_t index_offset, int64_t* out_idx, int64_t out_stride, float* out_scores,
                  int64_t append_sink, int64_t append_local, void* workspace, size_t workspace_bytes,
                  bool gkeys_ready, cudaStream_t st);

}  // namespace selectk
}  // namespace fathom
