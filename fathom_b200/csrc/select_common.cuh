// Internal: shared by select.cu and scan.cu (the fused scan + selection histogram).
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


// collect + finalize on a histogram (and boundary bins) already built: see select.cu.
int launch_select_tail(const float* scores, int64_t rows, int64_t n, int64_t row_stride, int64_t kk, int64_t mask_lo,
                       int64_t mask_hi, int64_t index_offset, int64_t* out_idx, int64_t out_stride,
                       float* out_scores, int64_t append_sink, int64_t append_local, const Workspace& w,
                       cudaStream_t st);

}  // namespace selectk
}  // namespace fathom
