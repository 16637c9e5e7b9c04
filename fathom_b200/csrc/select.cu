// Top-k selection over score rows: sink_local_topk (kernels/bitplane.py:372-378) and the
// merge of per-shard candidates.
//
// Output order is (score descending, index ascending); every tie is broken by the index, so
// the selection is deterministic and a context-sharded scan merges to the same list.
//
// Two paths, chosen per call (select_common.cuh: group_select_applies):
//
// Group-key path (a row has at least 1.5 kk fully unmasked 32-token groups): the scan's epilogue (or
// gmax_kernel over existing scores) writes the key of each group's largest score, then gsel_kernel,
// one CTA per row, bounds the threshold from those keys, reads only the groups that reach it and
// ranks the candidates (see gsel_kernel).
//
// Histogram path (dense k), three launches on the caller's stream:
//   1 hist      many CTAs per row: 4096-bin histogram of the top 12 bits of the order-
//               preserving key of every unmasked score (masked tokens get the key of -inf);
//               shared-memory histogram, flushed to the row's global histogram with atomics.
//               The last CTA of a row (atomic ticket; nothing waits) derives the boundary bin b*:
//               the largest bin with at least kk keys at or above it.
//   2 collect   many CTAs per row: appends every key in bins >= b* as a 64-bit candidate
//               (key << 32 | ~index), warp-aggregated atomics.  Candidates are unique and their
//               descending order is (score desc, index asc).
//   3 finalize  one CTA per row: radix select of the kk-th largest candidate on the remaining
//               52 bits (12-bit digits in shared memory, stopping as soon as the prefix holds
//               exactly the number still needed), compaction of exactly kk candidates, bitonic
//               sort of those.  A row with more candidates than the buffer holds (massive ties,
//               or kk close to n) takes an exact radix select over the whole row (12+12+8 bits)
//               and an index-ordered compaction of the keys equal to the threshold.
#include "select_common.cuh"


namespace fathom {
using namespace selectk;
namespace {

__device__ __forceinline__ uint32_t masked_key(const float* row, int64_t i, int64_t mask_lo, int64_t mask_hi) {
  return (i >= mask_lo && i < mask_hi) ? f2key(row[i]) : KEY_NEG_INF;
}

// Scores i0..i1 of a row, four at a time when the row is 16-byte aligned.
template <typename F>
__device__ __forceinline__ void for_each_score(const float* r, int64_t i0, int64_t i1, bool vec, F&& f) {
  if (vec) {
    for (int64_t i = i0 + 4 * (int64_t)threadIdx.x; i < i1; i += 4 * (int64_t)blockDim.x) {
      const float4 v = *reinterpret_cast<const float4*>(r + i);
      f(i, v.x);
      if (i + 1 < i1) f(i + 1, v.y);
      if (i + 2 < i1) f(i + 2, v.z);
      if (i + 3 < i1) f(i + 3, v.w);
    }
  } else {
    for (int64_t i = i0 + threadIdx.x; i < i1; i += blockDim.x) f(i, r[i]);
  }
}

__global__ void __launch_bounds__(HT) hist_kernel(const float* __restrict__ scores, int64_t n, int64_t row_stride,
                                                  int64_t kk, int64_t mask_lo, int64_t mask_hi,
                                                  uint32_t* __restrict__ ghist, uint32_t* __restrict__ ticket,
                                                  uint32_t* __restrict__ bstar) {
  __shared__ uint32_t sh[NBINS];
  __shared__ bool s_last;
  const int64_t row = blockIdx.y;
  for (int b = threadIdx.x; b < NBINS; b += HT) sh[b] = 0;
  __syncthreads();
  const float* r = scores + row * row_stride;
  const int64_t i0 = (int64_t)blockIdx.x * CHUNK;
  const int64_t i1 = i0 + CHUNK < n ? i0 + CHUNK : n;
  const bool vec = (n % 4 == 0) && (row_stride % 4 == 0) && ((reinterpret_cast<uintptr_t>(scores) & 15) == 0);
  const bool unmasked = i0 >= mask_lo && i1 <= mask_hi;
  constexpr int PER = CHUNK / HT;                  // 32 scores per thread, loaded before any atomic
  float x[PER];
#pragma unroll
  for (int u = 0; u < PER / 4; ++u) {
    const int64_t i = i0 + 4 * ((int64_t)threadIdx.x + (int64_t)u * HT);
    if (vec) {
      const float4 v = i < i1 ? *reinterpret_cast<const float4*>(r + i) : make_float4(0.f, 0.f, 0.f, 0.f);
      x[4 * u] = v.x; x[4 * u + 1] = v.y; x[4 * u + 2] = v.z; x[4 * u + 3] = v.w;
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e) x[4 * u + e] = i + e < i1 ? r[i + e] : 0.f;
    }
  }
#pragma unroll
  for (int u = 0; u < PER; ++u) {
    const int64_t i = i0 + 4 * ((int64_t)threadIdx.x + (int64_t)(u / 4) * HT) + (u % 4);
    if (i < i1) {
      const uint32_t key = (unmasked || (i >= mask_lo && i < mask_hi)) ? f2key(x[u]) : KEY_NEG_INF;
      atomicAdd(&sh[key >> (32 - HBITS)], 1u);
    }
  }
  __syncthreads();
  uint32_t* gh = ghist + row * NBINS;
  for (int b = threadIdx.x; b < NBINS; b += HT)
    if (sh[b]) atomicAdd(&gh[b], sh[b]);
  // the last CTA of the row to finish derives the boundary bin (no CTA waits for another)
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(&ticket[row], 1u) == gridDim.x - 1;
  __syncthreads();
  if (!s_last || threadIdx.x >= 32) return;
  __threadfence();
  const int bs = warp_boundary_bin(gh, kk);
  if (threadIdx.x == 0) bstar[row] = (uint32_t)bs;
}

__global__ void __launch_bounds__(HT, 2) collect_kernel(const float* __restrict__ scores, int64_t n, int64_t row_stride,
                                                     int64_t mask_lo, int64_t mask_hi,
                                                     const uint32_t* __restrict__ bstar_rows,
                                                     uint32_t* __restrict__ count, uint64_t* __restrict__ cand) {
  constexpr int PER = CHUNK / HT;           // scores per thread (32), in two rounds of 16
  constexpr int HALF = PER / 2;
  const int64_t row = blockIdx.y;
  const uint32_t bstar = bstar_rows[row];
  const float* r = scores + row * row_stride;
  const int64_t i0 = (int64_t)blockIdx.x * CHUNK;
  const int64_t i1 = i0 + CHUNK < n ? i0 + CHUNK : n;
  const int lane = threadIdx.x & 31;
  uint64_t* cr = cand + row * CAP;
  const bool vec = (n % 4 == 0) && (row_stride % 4 == 0) && ((reinterpret_cast<uintptr_t>(scores) & 15) == 0);
  const bool unmasked = i0 >= mask_lo && i1 <= mask_hi;   // the whole chunk is outside sink/local
#pragma unroll 1
  for (int round = 0; round < 2; ++round) {
    // thread t owns scores i0 + 4t + 4*HT*u + e; this pass's loads first, then the filter
    float x[HALF];
#pragma unroll
    for (int uu = 0; uu < HALF / 4; ++uu) {
      const int u = round * (HALF / 4) + uu;
      const int64_t i = i0 + 4 * ((int64_t)threadIdx.x + (int64_t)u * HT);
      if (vec) {
        const float4 v = i < i1 ? *reinterpret_cast<const float4*>(r + i) : make_float4(0.f, 0.f, 0.f, 0.f);
        x[4 * uu] = v.x; x[4 * uu + 1] = v.y; x[4 * uu + 2] = v.z; x[4 * uu + 3] = v.w;
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) x[4 * uu + e] = i + e < i1 ? r[i + e] : 0.f;
      }
    }
    uint32_t takes = 0;
#pragma unroll
    for (int v = 0; v < HALF; ++v) {
      const int u = round * (HALF / 4) + v / 4;
      const int64_t i = i0 + 4 * ((int64_t)threadIdx.x + (int64_t)u * HT) + (v % 4);
      const uint32_t key = (unmasked || (i >= mask_lo && i < mask_hi)) ? f2key(x[v]) : KEY_NEG_INF;
      if (i < i1 && (key >> (32 - HBITS)) >= bstar) takes |= 1u << v;
    }
    if (!__any_sync(0xffffffffu, takes != 0)) continue;
#pragma unroll
    for (int v = 0; v < HALF; ++v) {
      const int u = round * (HALF / 4) + v / 4;
      const int64_t i = i0 + 4 * ((int64_t)threadIdx.x + (int64_t)u * HT) + (v % 4);
      const bool take = (takes >> v) & 1u;
      const uint32_t m = __ballot_sync(0xffffffffu, take);
      if (m) {
        uint32_t pos0 = 0;
        if (lane == 0) pos0 = atomicAdd(&count[row], (uint32_t)__popc(m));
        pos0 = __shfl_sync(0xffffffffu, pos0, 0);
        if (take) {
          const uint32_t key = (unmasked || (i >= mask_lo && i < mask_hi)) ? f2key(x[v]) : KEY_NEG_INF;
          const uint32_t pos = pos0 + __popc(m & ((1u << lane) - 1));
          if (pos < CAP) cr[pos] = ((uint64_t)key << 32) | (uint32_t)(~(uint32_t)i);
        }
      }
    }
  }
}

// Bitonic sort of P (power of two) 64-bit values in shared memory, descending.
__device__ void bitonic_desc(uint64_t* s, int P) {
  for (int k = 2; k <= P; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < P; i += blockDim.x) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const uint64_t a = s[i], b = s[ixj];
          const bool desc = (i & k) == 0;
          if (desc ? (a < b) : (a > b)) {
            s[i] = b;
            s[ixj] = a;
          }
        }
      }
      __syncthreads();
    }
  }
}

__device__ __forceinline__ int next_pow2(int x) {
  int p = 1;
  while (p < x) p <<= 1;
  return p;
}

// Exact selection of the kk largest keys of one row by a single CTA (rare path).  Writes the
// selected candidates to s_out[0..kk) (unordered) as (key << 32 | ~index).
__device__ void exact_select_row(const float* r, int64_t n, int64_t kk, int64_t mask_lo, int64_t mask_hi,
                                 uint64_t* s_out, uint32_t* s_hist, uint32_t* s_part, int* s_res, uint32_t* s_warp,
                                 uint32_t* s_cnt) {
  uint32_t prefix = 0, pmask = 0;
  int64_t need = kk;
  const int shifts[3] = {20, 8, 0};
  const int widths[3] = {12, 12, 8};
  for (int lv = 0; lv < 3; ++lv) {
    const int sh = shifts[lv], nb = 1 << widths[lv];
    for (int b = threadIdx.x; b < NBINS; b += blockDim.x) s_hist[b] = 0;
    __syncthreads();
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
      const uint32_t key = masked_key(r, i, mask_lo, mask_hi);
      if ((key & pmask) == prefix) atomicAdd(&s_hist[(key >> sh) & (nb - 1)], 1u);
    }
    __syncthreads();
    const int b = boundary_bin(s_hist, need, s_part, s_res);
    // keys of this prefix in bins above b are all taken
    uint32_t above = 0;
    for (int x = threadIdx.x; x < NBINS; x += blockDim.x)
      if (x > b) above += s_hist[x];
    uint32_t tot;
    block_exclusive_scan(above, s_warp, &tot);
    need -= tot;
    prefix |= (uint32_t)b << sh;
    pmask |= (uint32_t)(nb - 1) << sh;
  }
  const uint32_t T = prefix;  // exact key of the kk-th largest; `need` keys equal to T are taken
  if (threadIdx.x == 0) *s_cnt = 0;
  __syncthreads();
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
    const uint32_t key = masked_key(r, i, mask_lo, mask_hi);
    if (key > T) s_out[atomicAdd(s_cnt, 1u)] = ((uint64_t)key << 32) | (uint32_t)(~(uint32_t)i);
  }
  __syncthreads();
  const uint32_t ngt = *s_cnt;
  // first `need` keys equal to T, in index order
  uint32_t taken = 0;
  for (int64_t base = 0; base < n && taken < (uint32_t)need; base += blockDim.x) {
    const int64_t i = base + threadIdx.x;
    const bool eq = i < n && masked_key(r, i, mask_lo, mask_hi) == T;
    uint32_t tot;
    const uint32_t pos = block_exclusive_scan(eq ? 1u : 0u, s_warp, &tot);
    if (eq && taken + pos < (uint32_t)need) s_out[ngt + taken + pos] = ((uint64_t)T << 32) | (uint32_t)(~(uint32_t)i);
    taken += tot;
  }
  __syncthreads();
}

// Radix select on 64-bit candidates held in shared memory: returns (to every thread) the
// smallest value C such that exactly kk of the n values are >= C.  The values are unique; the
// top 12 bits of the kk-th largest are `top12` and `need` of the values equal it in those bits.
// Per level one pass counts the values still matching the prefix and histograms their next digit;
// one warp then finds the digit.  It stops as soon as the prefix holds exactly `need` values.
__device__ uint64_t refine_threshold(const uint64_t* s_v, int n, uint32_t top12, int64_t need, uint32_t* s_hist,
                                     uint32_t* s_ctl, uint32_t* s_tmp) {
  uint64_t prefix = (uint64_t)top12 << 52;
  uint64_t pmask = 0xFFFull << 52;
  const int shifts[5] = {40, 28, 16, 4, 0};
  const int widths[5] = {12, 12, 12, 12, 4};
  for (int lv = 0; lv < 5; ++lv) {
    const int sh = shifts[lv], nb = 1 << widths[lv];
    for (int b = threadIdx.x; b < NBINS; b += blockDim.x) s_hist[b] = 0;
    if (threadIdx.x == 0) s_ctl[0] = 0;
    __syncthreads();
    uint32_t match = 0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const uint64_t v = s_v[i];
      if ((v & pmask) == prefix) {
        ++match;
        atomicAdd(&s_hist[(v >> sh) & (nb - 1)], 1u);
      }
    }
    match += __shfl_xor_sync(0xffffffffu, match, 16);
    match += __shfl_xor_sync(0xffffffffu, match, 8);
    match += __shfl_xor_sync(0xffffffffu, match, 4);
    match += __shfl_xor_sync(0xffffffffu, match, 2);
    match += __shfl_xor_sync(0xffffffffu, match, 1);
    if ((threadIdx.x & 31) == 0 && match) atomicAdd(&s_ctl[0], match);
    __syncthreads();
    if ((int64_t)s_ctl[0] == need) break;  // uniform: every value matching the prefix is taken
    uint32_t above;
    const int b = block_boundary_bin(s_hist, need, s_tmp, &above);
    need -= above;
    prefix |= (uint64_t)b << sh;
    pmask |= (uint64_t)(nb - 1) << sh;
    __syncthreads();  // s_ctl is rewritten by the next level
  }
  return prefix;
}

// Descending bitonic sort of P (power of two, <= blockDim.x) values, one per thread: v of thread i is
// element i.  Partners closer than a warp are exchanged with shuffles, farther ones through shared
// memory (s_x, P entries).  Returns this thread's element of the sorted order.
__device__ uint64_t bitonic_desc_regs(uint64_t v, int P, uint64_t* s_x) {
  const int i = threadIdx.x;
  for (int k = 2; k <= P; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      uint64_t other;
      if (j >= 32) {
        if (i < P) s_x[i] = v;
        __syncthreads();
        other = i < P ? s_x[i ^ j] : v;
        __syncthreads();
      } else {
        other = __shfl_xor_sync(0xffffffffu, v, j);
      }
      const bool keep_max = ((i & k) == 0) == ((i & j) == 0);
      if (i < P) v = keep_max ? (v > other ? v : other) : (v < other ? v : other);
    }
  }
  return v;
}

// Sorts the kk selected candidates of s_sel (descending: score desc, index asc) and writes the row's
// output: indices (+ index_offset), optional scores, then the appended sink and local indices.
// s_sel holds next_pow2(kk) entries; s_x is scratch of as many.
__device__ void write_sorted(uint64_t* s_sel, uint64_t* s_x, int64_t row, int64_t n, int64_t kk, int64_t index_offset,
                             int64_t* __restrict__ out_idx, int64_t out_stride, float* __restrict__ out_scores,
                             int64_t append_sink, int64_t append_local) {
  const int P = next_pow2((int)kk);
  int64_t* o = out_idx + row * out_stride;
  if (P <= (int)blockDim.x) {
    // one value per thread, sorted in registers
    uint64_t v = threadIdx.x < kk ? s_sel[threadIdx.x] : 0ull;
    __syncthreads();
    v = bitonic_desc_regs(v, P, s_x);
    if (threadIdx.x < kk) {
      o[threadIdx.x] = (int64_t)(uint32_t)(~(uint32_t)v) + index_offset;
      if (out_scores) out_scores[row * kk + threadIdx.x] = key2f((uint32_t)(v >> 32));
    }
  } else {
    for (int i = (int)kk + threadIdx.x; i < P; i += blockDim.x) s_sel[i] = 0ull;
    __syncthreads();
    bitonic_desc(s_sel, P);
    for (int i = threadIdx.x; i < kk; i += blockDim.x) {
      const uint64_t v = s_sel[i];
      o[i] = (int64_t)(uint32_t)(~(uint32_t)v) + index_offset;
      if (out_scores) out_scores[row * kk + i] = key2f((uint32_t)(v >> 32));
    }
  }
  for (int64_t i = threadIdx.x; i < append_sink; i += blockDim.x) o[kk + i] = i;
  for (int64_t i = threadIdx.x; i < append_local; i += blockDim.x) o[kk + append_sink + i] = n - append_local + i;
}

__global__ void __launch_bounds__(FT) finalize_kernel(const float* __restrict__ scores, int64_t n, int64_t row_stride,
                                                      int64_t kk, int64_t mask_lo, int64_t mask_hi,
                                                      const uint32_t* __restrict__ count,
                                                      const uint32_t* __restrict__ bstar_rows,
                                                      const uint64_t* __restrict__ cand, int64_t index_offset,
                                                      int64_t* __restrict__ out_idx, int64_t out_stride,
                                                      float* __restrict__ out_scores, int64_t append_sink,
                                                      int64_t append_local) {
  extern __shared__ uint64_t s_dyn[];  // CAP candidates, then MAX_KK selected
  uint64_t* s_buf = s_dyn;
  uint64_t* s_sel = s_dyn + CAP;
  __shared__ uint32_t s_hist[NBINS];
  __shared__ uint32_t s_part[FT];
  __shared__ uint32_t s_warp[33];
  __shared__ uint32_t s_ctl[4];
  __shared__ uint32_t s_tmp[66];
  __shared__ uint32_t s_cnt;
  __shared__ int s_res;
  const int64_t row = blockIdx.x;
  const uint32_t cnt = count[row];
  if (cnt <= (uint32_t)CAP) {
    const uint32_t top12 = bstar_rows[row];
    uint32_t above = 0;
    for (int i = threadIdx.x; i < (int)cnt; i += blockDim.x) {
      const uint64_t v = cand[row * CAP + i];
      s_buf[i] = v;
      above += (uint32_t)(v >> 52) > top12;
    }
    above += __shfl_xor_sync(0xffffffffu, above, 16);
    above += __shfl_xor_sync(0xffffffffu, above, 8);
    above += __shfl_xor_sync(0xffffffffu, above, 4);
    above += __shfl_xor_sync(0xffffffffu, above, 2);
    above += __shfl_xor_sync(0xffffffffu, above, 1);
    if (threadIdx.x == 0) s_cnt = 0;
    __syncthreads();
    if ((threadIdx.x & 31) == 0 && above) atomicAdd(&s_cnt, above);
    __syncthreads();
    const uint32_t tot = s_cnt;
    __syncthreads();
    const uint64_t C = refine_threshold(s_buf, (int)cnt, top12, kk - (int64_t)tot, s_hist, s_ctl, s_tmp);
    if (threadIdx.x == 0) s_cnt = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < (int)cnt; i += blockDim.x)
      if (s_buf[i] >= C) {
        const uint32_t pos = atomicAdd(&s_cnt, 1u);
        if (pos < (uint32_t)MAX_KK) s_sel[pos] = s_buf[i];
      }
    __syncthreads();
  } else {
    exact_select_row(scores + row * row_stride, n, kk, mask_lo, mask_hi, s_sel, s_hist, s_part, &s_res, s_warp,
                     &s_cnt);
  }
  write_sorted(s_sel, s_buf, row, n, kk, index_offset, out_idx, out_stride, out_scores, append_sink, append_local);
}

__global__ void __launch_bounds__(FT) merge_kernel(const float* __restrict__ cs, const int64_t* __restrict__ ci,
                                                   int64_t m, int64_t kk, int64_t* __restrict__ out_idx,
                                                   float* __restrict__ out_scores) {
  extern __shared__ uint64_t s_dyn[];  // CAP candidates, then MAX_KK selected
  uint64_t* s_buf = s_dyn;
  uint64_t* s_sel = s_dyn + CAP;
  __shared__ uint32_t s_hist[NBINS];
  __shared__ uint32_t s_ctl[4];
  __shared__ uint32_t s_tmp[66];
  __shared__ uint32_t s_cnt;
  const int64_t row = blockIdx.x;
  for (int b = threadIdx.x; b < NBINS; b += blockDim.x) s_hist[b] = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < m; i += blockDim.x) {
    const uint64_t v = ((uint64_t)f2key(cs[row * m + i]) << 32) | (uint32_t)(~(uint32_t)ci[row * m + i]);
    s_buf[i] = v;
    atomicAdd(&s_hist[v >> 52], 1u);
  }
  __syncthreads();
  uint32_t above;
  const uint32_t top12 = (uint32_t)block_boundary_bin(s_hist, kk, s_tmp, &above);
  const int64_t need = kk - (int64_t)above;
  const uint64_t C = refine_threshold(s_buf, (int)m, top12, need, s_hist, s_ctl, s_tmp);
  if (threadIdx.x == 0) s_cnt = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < m; i += blockDim.x)
    if (s_buf[i] >= C) {
      const uint32_t pos = atomicAdd(&s_cnt, 1u);
      if (pos < (uint32_t)MAX_KK) s_sel[pos] = s_buf[i];   // distinct indices give exactly kk
    }
  __syncthreads();
  const int P = next_pow2((int)kk);
  if (P <= FT) {
    uint64_t v = threadIdx.x < kk ? s_sel[threadIdx.x] : 0ull;
    __syncthreads();
    v = bitonic_desc_regs(v, P, s_buf);
    if (threadIdx.x < kk) {
      out_idx[row * kk + threadIdx.x] = (int64_t)(uint32_t)(~(uint32_t)v);
      if (out_scores) out_scores[row * kk + threadIdx.x] = key2f((uint32_t)(v >> 32));
    }
  } else {
    for (int i = (int)kk + threadIdx.x; i < P; i += blockDim.x) s_sel[i] = 0ull;
    __syncthreads();
    bitonic_desc(s_sel, P);
    for (int i = threadIdx.x; i < kk; i += blockDim.x) {
      const uint64_t v = s_sel[i];
      out_idx[row * kk + i] = (int64_t)(uint32_t)(~(uint32_t)v);
      if (out_scores) out_scores[row * kk + i] = key2f((uint32_t)(v >> 32));
    }
  }
}

// ---------------------------------------------------------------------------------------------
// Group-maximum selection (see select_common.cuh).

// One thread per group of GROUP scores: the largest key of the group (keys, not floats, so -0 and
// +0 order as the selection orders them).
__global__ void __launch_bounds__(256) gmax_kernel(const float* __restrict__ scores, int64_t n, int64_t row_stride,
                                                   int64_t ng, uint32_t* __restrict__ gkey) {
  const int64_t row = blockIdx.y;
  const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= ng) return;
  const float* r = scores + row * row_stride;
  const int64_t t0 = g * GROUP, t1 = t0 + GROUP < n ? t0 + GROUP : n;
  uint32_t m = 0;
  if (t1 - t0 == GROUP && (reinterpret_cast<uintptr_t>(r + t0) & 15) == 0) {
#pragma unroll
    for (int u = 0; u < GROUP / 4; ++u) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(r + t0) + u);
      m = max(m, max(max(f2key(v.x), f2key(v.y)), max(f2key(v.z), f2key(v.w))));
    }
  } else {
    for (int64_t i = t0; i < t1; ++i) m = max(m, f2key(r[i]));
  }
  gkey[row * ng + g] = m;
}

constexpr int QT = 1024;   // threads of the group-selection CTA

// One CTA per row.
//   1 two-level histogram (top 12 key bits, then the next 12 bits inside the boundary bin) of the
//     fully unmasked groups' keys (warp-aggregated shared atomics); tau = lower edge of the second
//     level's boundary bin: at least kk groups, hence kk unmasked tokens, have a key >= tau, and tau
//     lies within 2^-15 octave of the kk-th largest group key
//   2 list the groups whose key reaches tau, read their scores, keep every token with key >= tau
//     (masked tokens carry the key of -inf, as in the histogram path) as a candidate
//   3 at most 4096 candidates: a counting rank (bins of the key above tau, then a count of the larger
//     values in the candidate's bin); ranks below kk are written in place.  More: radix-refine to
//     exactly kk, then sort.
// More than CAP listed groups or candidates (massive ties) takes the exact whole-row selection.
__global__ void __launch_bounds__(QT) gsel_kernel(const float* __restrict__ scores, int64_t n, int64_t row_stride,
                                                  int64_t kk, int64_t mask_lo, int64_t mask_hi,
                                                  const uint32_t* __restrict__ gkey, int64_t ng, int64_t index_offset,
                                                  int64_t* __restrict__ out_idx, int64_t out_stride,
                                                  float* __restrict__ out_scores, int64_t append_sink,
                                                  int64_t append_local) {
  extern __shared__ uint64_t s_dyn[];  // CAP candidates, then MAX_KK selected (the group list before that)
  uint64_t* s_buf = s_dyn;
  uint64_t* s_sel = s_dyn + CAP;
  int32_t* s_glist = reinterpret_cast<int32_t*>(s_sel);   // CAP group ids; phase 2 only
  __shared__ uint32_t s_hist[NBINS];
  __shared__ uint32_t s_part[QT];
  __shared__ uint32_t s_warp[33];
  __shared__ uint32_t s_ctl[4];
  __shared__ uint32_t s_tmp[66];
  __shared__ uint32_t s_cnt, s_nq;
  __shared__ int s_res;
  const int64_t row = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31;
  const uint32_t* gk = gkey + row * ng;
  const float* r = scores + row * row_stride;
  const int64_t lo = mask_lo < 0 ? 0 : (mask_lo > n ? n : mask_lo);
  const int64_t hi = mask_hi < 0 ? 0 : (mask_hi > n ? n : mask_hi);
  const int64_t g_lo = (lo + GROUP - 1) / GROUP;
  const int64_t g_hi = hi == n ? ng : hi / GROUP;
  for (int b = tid; b < NBINS; b += QT) s_hist[b] = 0;
  if (tid == 0) {
    s_cnt = 0;
    s_nq = 0;
  }
  __syncthreads();

  // 1: histogram of the unmasked groups' keys
  constexpr int U = 8;
  for (int64_t base = 0; base < ng; base += (int64_t)QT * U) {
    uint32_t bin[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t g = base + (int64_t)u * QT + tid;
      bin[u] = (g >= g_lo && g < g_hi) ? (__ldg(gk + g) >> (32 - HBITS)) : (uint32_t)NBINS;
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint32_t peers = __match_any_sync(0xffffffffu, bin[u]);
      if (bin[u] < (uint32_t)NBINS && lane == __ffs(peers) - 1) atomicAdd(&s_hist[bin[u]], (uint32_t)__popc(peers));
    }
  }
  __syncthreads();
  uint32_t gabove;
  const uint32_t b1 = (uint32_t)block_boundary_bin(s_hist, kk, s_tmp, &gabove);   // 0: all qualify
  // second level: the next 12 bits of the group keys inside bin b1 (kk - gabove of them are needed)
  for (int b = tid; b < NBINS; b += QT) s_hist[b] = 0;
  __syncthreads();
  for (int64_t base = 0; base < ng; base += (int64_t)QT * U) {
    uint32_t bin[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t g = base + (int64_t)u * QT + tid;
      const uint32_t key = (g >= g_lo && g < g_hi) ? __ldg(gk + g) : 0u;
      bin[u] = (g >= g_lo && g < g_hi && (key >> (32 - HBITS)) == b1) ? ((key >> (32 - 2 * HBITS)) & (NBINS - 1))
                                                                      : (uint32_t)NBINS;
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (!__any_sync(0xffffffffu, bin[u] < (uint32_t)NBINS)) continue;
      const uint32_t peers = __match_any_sync(0xffffffffu, bin[u]);
      if (bin[u] < (uint32_t)NBINS && lane == __ffs(peers) - 1) atomicAdd(&s_hist[bin[u]], (uint32_t)__popc(peers));
    }
  }
  __syncthreads();
  uint32_t gabove2;
  const uint32_t b2 = (uint32_t)block_boundary_bin(s_hist, kk - (int64_t)gabove, s_tmp, &gabove2);
  // at least kk unmasked groups have a key >= tau (0 when fewer than kk groups: all qualify)
  const uint32_t tau = (b1 << (32 - HBITS)) | (b2 << (32 - 2 * HBITS));

  // 2a: the groups whose key reaches tau, in a shared list
  for (int64_t base = 0; base < ng; base += (int64_t)QT * U) {
    uint32_t q = 0;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t g = base + (int64_t)u * QT + tid;
      if (g < ng && __ldg(gk + g) >= tau) q |= 1u << u;
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const bool take = (q >> u) & 1u;
      const uint32_t m = __ballot_sync(0xffffffffu, take);
      if (m) {
        uint32_t pos0 = 0;
        if (lane == 0) pos0 = atomicAdd(&s_nq, (uint32_t)__popc(m));
        pos0 = __shfl_sync(0xffffffffu, pos0, 0);
        const uint32_t pos = pos0 + __popc(m & ((1u << lane) - 1));
        if (take && pos < (uint32_t)CAP) s_glist[pos] = (int32_t)(base + (int64_t)u * QT + tid);
      }
    }
  }
  __syncthreads();
  const uint32_t nq = s_nq;

  // 2b: one listed group per thread; its tokens with key >= tau become candidates
  if (nq <= (uint32_t)CAP) {
    for (uint32_t jb = 0; jb < nq; jb += QT) {
      const uint32_t j = jb + tid;
      uint32_t take = 0;
      int64_t t0 = 0;
      if (j < nq) {
        t0 = (int64_t)s_glist[j] * GROUP;
        const int64_t t1 = t0 + GROUP < n ? t0 + GROUP : n;
        const bool inside = t0 >= lo && t1 <= hi;
        if (t1 - t0 == GROUP && (reinterpret_cast<uintptr_t>(r + t0) & 15) == 0) {
#pragma unroll
          for (int u = 0; u < GROUP / 4; ++u) {
            const float4 v = __ldg(reinterpret_cast<const float4*>(r + t0) + u);
            const float e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              const int64_t i = t0 + 4 * u + c;
              const uint32_t key = (inside || (i >= lo && i < hi)) ? f2key(e[c]) : KEY_NEG_INF;
              if (key >= tau) take |= 1u << (4 * u + c);
            }
          }
        } else {
          for (int64_t i = t0; i < t1; ++i) {
            const uint32_t key = (i >= lo && i < hi) ? f2key(r[i]) : KEY_NEG_INF;
            if (key >= tau) take |= 1u << (int)(i - t0);
          }
        }
      }
      // warp-aggregated reservation of the candidate slots
      const uint32_t c = (uint32_t)__popc(take);
      uint32_t incl = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      uint32_t base = 0;
      if (lane == 31) base = atomicAdd(&s_cnt, incl);
      base = __shfl_sync(0xffffffffu, base, 31);
      uint32_t pos = base + incl - c;
      while (take) {
        const int b = __ffs(take) - 1;
        take &= take - 1;
        const int64_t i = t0 + b;
        const uint32_t key = (i >= lo && i < hi) ? f2key(r[i]) : KEY_NEG_INF;
        if (pos < (uint32_t)CAP) s_buf[pos] = ((uint64_t)key << 32) | (uint32_t)(~(uint32_t)i);
        ++pos;
      }
    }
  }
  __syncthreads();
  const uint32_t cnt = s_cnt;

  const bool fits = nq <= (uint32_t)CAP && cnt <= (uint32_t)CAP && cnt >= (uint32_t)kk;
  if (fits && cnt <= (uint32_t)MAX_KK) {
    // 3 (usual case): a counting rank.  Candidates go to NBINS bins of (key - tau) >> bshift, highest bin
    // first; a descending scan of the bin counts gives each bin's first rank, and a candidate's rank is
    // that plus the number of larger values in its bin (bins hold a few candidates).  Ranks < kk are
    // written straight to their output positions.
    uint32_t kmax = 0;
    for (int i = tid; i < (int)cnt; i += QT) kmax = max(kmax, (uint32_t)(s_buf[i] >> 32));
    kmax = __reduce_max_sync(0xffffffffu, kmax);
    if (lane == 0) s_tmp[tid >> 5] = kmax;
    for (int b = tid; b < NBINS; b += QT) s_hist[b] = 0;
    __syncthreads();
    kmax = s_tmp[lane];   // 32 warps
    kmax = __reduce_max_sync(0xffffffffu, kmax);
    int bshift = 0;
    while (((kmax - tau) >> bshift) >= (uint32_t)NBINS) ++bshift;
    for (int i = tid; i < (int)cnt; i += QT)
      atomicAdd(&s_hist[(NBINS - 1) - (((uint32_t)(s_buf[i] >> 32) - tau) >> bshift)], 1u);   // descending bins
    __syncthreads();
    uint32_t* s_cur = reinterpret_cast<uint32_t*>(s_buf + MAX_KK);   // bin cursors (the unused half of s_buf)
    {
      const int per = NBINS / QT;   // 4 bins per thread
      uint32_t c[NBINS / QT], tot = 0;
#pragma unroll
      for (int u = 0; u < per; ++u) {
        c[u] = s_hist[tid * per + u];
        tot += c[u];
      }
      uint32_t all;
      uint32_t start = block_exclusive_scan(tot, s_warp, &all);
#pragma unroll
      for (int u = 0; u < per; ++u) {
        s_hist[tid * per + u] = start;   // first rank of the bin
        s_cur[tid * per + u] = start;
        start += c[u];
      }
    }
    __syncthreads();
    for (int i = tid; i < (int)cnt; i += QT) {
      const uint64_t v = s_buf[i];
      const uint32_t b = (NBINS - 1) - (((uint32_t)(v >> 32) - tau) >> bshift);
      s_sel[atomicAdd(&s_cur[b], 1u)] = v;
    }
    __syncthreads();   // s_cur[b] is now the end of bin b
    int64_t* o = out_idx + row * out_stride;
    for (int i = tid; i < (int)cnt; i += QT) {
      const uint64_t v = s_buf[i];
      const uint32_t b = (NBINS - 1) - (((uint32_t)(v >> 32) - tau) >> bshift);
      uint32_t r = s_hist[b];
      for (uint32_t t = s_hist[b]; t < s_cur[b]; ++t) r += s_sel[t] > v;
      if (r < (uint32_t)kk) {
        o[r] = (int64_t)(uint32_t)(~(uint32_t)v) + index_offset;
        if (out_scores) out_scores[row * kk + r] = key2f((uint32_t)(v >> 32));
      }
    }
    for (int64_t i = tid; i < append_sink; i += QT) o[kk + i] = i;
    for (int64_t i = tid; i < append_local; i += QT) o[kk + append_sink + i] = n - append_local + i;
    return;
  }
  if (fits) {
    // 3: exactly kk of the candidates (at least kk of them exist, all distinct)
    for (int b = tid; b < NBINS; b += QT) s_hist[b] = 0;
    __syncthreads();
    for (int i = tid; i < (int)cnt; i += QT) atomicAdd(&s_hist[s_buf[i] >> 52], 1u);
    __syncthreads();
    uint32_t above;
    const uint32_t top12 = (uint32_t)block_boundary_bin(s_hist, kk, s_tmp, &above);
    const int64_t need = kk - (int64_t)above;
    const uint64_t C = refine_threshold(s_buf, (int)cnt, top12, need, s_hist, s_ctl, s_tmp);
    if (tid == 0) s_cnt = 0;
    __syncthreads();
    for (int i = tid; i < (int)cnt; i += QT)
      if (s_buf[i] >= C) {
        const uint32_t pos = atomicAdd(&s_cnt, 1u);
        if (pos < (uint32_t)MAX_KK) s_sel[pos] = s_buf[i];
      }
    __syncthreads();
  } else {
    exact_select_row(r, n, kk, mask_lo, mask_hi, s_sel, s_hist, s_part, &s_res, s_warp, &s_cnt);
  }
  write_sorted(s_sel, s_buf, row, n, kk, index_offset, out_idx, out_stride, out_scores, append_sink, append_local);
}

int run_group_select(const float* scores, int64_t rows, int64_t n, int64_t row_stride, int64_t kk, int64_t mask_lo,
                     int64_t mask_hi, int64_t index_offset, int64_t* out_idx, int64_t out_stride, float* out_scores,
                     int64_t append_sink, int64_t append_local, uint32_t* gkey, bool gkeys_ready, cudaStream_t st) {
  const int64_t ng = n_groups(n);
  if (!gkeys_ready) {
    dim3 grid((unsigned)cdiv(ng, 256), (unsigned)rows);
    gmax_kernel<<<grid, 256, 0, st>>>(scores, n, row_stride, ng, gkey);
  }
  const size_t smem = (CAP + MAX_KK) * sizeof(uint64_t);
  cudaFuncSetAttribute(gsel_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  gsel_kernel<<<(unsigned)rows, QT, smem, st>>>(scores, n, row_stride, kk, mask_lo, mask_hi, gkey, ng, index_offset,
                                                 out_idx, out_stride, out_scores, append_sink, append_local);
  return check_launch("select_topk (group keys)");
}

// collect + finalize on a histogram and boundary bins already built
int select_tail(const float* scores, int64_t rows, int64_t n, int64_t row_stride, int64_t kk, int64_t mask_lo,
                       int64_t mask_hi, int64_t index_offset, int64_t* out_idx, int64_t out_stride,
                       float* out_scores, int64_t append_sink, int64_t append_local, const Workspace& w,
                       cudaStream_t st) {
  const int64_t chunks = cdiv(n, CHUNK);
  dim3 grid((unsigned)chunks, (unsigned)rows);
  collect_kernel<<<grid, HT, 0, st>>>(scores, n, row_stride, mask_lo, mask_hi, w.bstar, w.count, w.cand);
  const size_t smem = (CAP + MAX_KK) * sizeof(uint64_t);
  cudaFuncSetAttribute(finalize_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  finalize_kernel<<<(unsigned)rows, FT, smem, st>>>(scores, n, row_stride, kk, mask_lo, mask_hi, w.count, w.bstar,
                                                     w.cand, index_offset, out_idx, out_stride, out_scores,
                                                     append_sink, append_local);
  return check_launch("select_topk");
}

int run_select(const float* scores, int64_t rows, int64_t n, int64_t row_stride, int64_t kk, int64_t mask_lo,
               int64_t mask_hi, int64_t index_offset, int64_t* out_idx, int64_t out_stride, float* out_scores,
               int64_t append_sink, int64_t append_local, void* workspace, size_t workspace_bytes, bool gkeys_ready,
               cudaStream_t st) {
  FATHOM_REQUIRE(scores && out_idx, FATHOM_ERR_NULL, "select_topk: NULL pointer");
  FATHOM_REQUIRE(rows >= 1 && rows <= 65535 && n >= 1 && n <= 0xffffffffLL, FATHOM_ERR_SHAPE,
                 "select_topk: need 1 <= rows <= 65535 and 1 <= n < 2^32");
  FATHOM_REQUIRE(kk >= 1 && kk <= MAX_KK && kk <= n, FATHOM_ERR_SHAPE, "select_topk: kk=%lld outside 1..min(4096, n=%lld)",
                 (long long)kk, (long long)n);
  FATHOM_REQUIRE(row_stride >= n && out_stride >= kk + append_sink + append_local, FATHOM_ERR_SHAPE,
                 "select_topk: bad strides");
  FATHOM_REQUIRE(workspace != nullptr, FATHOM_ERR_NULL, "select_topk: workspace is NULL");
  FATHOM_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 255) == 0, FATHOM_ERR_WORKSPACE,
                 "select_topk: workspace must be 256-byte aligned");
  if (group_select_applies(rows, n, kk, mask_lo, mask_hi, workspace_bytes))
    return run_group_select(scores, rows, n, row_stride, kk, mask_lo, mask_hi, index_offset, out_idx, out_stride,
                            out_scores, append_sink, append_local, static_cast<uint32_t*>(workspace), gkeys_ready, st);
  FATHOM_REQUIRE(!gkeys_ready, FATHOM_ERR_UNSUPPORTED, "select_topk: group keys given where they do not apply");
  FATHOM_REQUIRE(workspace_bytes >= ws_bytes(rows), FATHOM_ERR_WORKSPACE,
                 "select_topk: workspace needs %zu bytes (got %zu)", select_ws_bytes(rows, n), workspace_bytes);
  Workspace w = carve(workspace, rows);
  cudaError_t e = cudaMemsetAsync(workspace, 0, zeroed_bytes(rows), st);
  if (e != cudaSuccess) return set_error(FATHOM_ERR_CUDA, "select_topk: memset: %s", cudaGetErrorString(e));
  const int64_t chunks = cdiv(n, CHUNK);
  dim3 grid((unsigned)chunks, (unsigned)rows);
  hist_kernel<<<grid, HT, 0, st>>>(scores, n, row_stride, kk, mask_lo, mask_hi, w.hist, w.ticket, w.bstar);
  return select_tail(scores, rows, n, row_stride, kk, mask_lo, mask_hi, index_offset, out_idx, out_stride,
                            out_scores, append_sink, append_local, w, st);
}

}  // namespace

namespace selectk {
int launch_select(const float* scores, int64_t rows, int64_t n, int64_t row_stride, int64_t kk, int64_t mask_lo,
                  int64_t mask_hi, int64_t index_offset, int64_t* out_idx, int64_t out_stride, float* out_scores,
                  int64_t append_sink, int64_t append_local, void* workspace, size_t workspace_bytes,
                  bool gkeys_ready, cudaStream_t st) {
  return run_select(scores, rows, n, row_stride, kk, mask_lo, mask_hi, index_offset, out_idx, out_stride, out_scores,
                    append_sink, append_local, workspace, workspace_bytes, gkeys_ready, st);
}

}  // namespace selectk
}  // namespace fathom

using namespace fathom;

extern "C" size_t fathom_select_workspace_bytes(int64_t rows, int64_t n, int64_t kk) {
  (void)kk;
  return rows > 0 && n > 0 ? select_ws_bytes(rows, n) : 0;
}

extern "C" int fathom_select_topk(const float* scores, int64_t rows, int64_t n, int64_t row_stride, int64_t kk,
                                  int64_t mask_lo, int64_t mask_hi, int64_t index_offset, int64_t* out_idx,
                                  int64_t out_stride, float* out_scores, void* workspace, size_t workspace_bytes,
                                  void* stream) {
  return run_select(scores, rows, n, row_stride, kk, mask_lo, mask_hi, index_offset, out_idx, out_stride, out_scores,
                    0, 0, workspace, workspace_bytes, false, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int fathom_sink_local_topk(const float* scores, int64_t rows, int64_t n, int64_t k, int64_t sink,
                                      int64_t local, int64_t* idx, void* workspace, size_t workspace_bytes,
                                      void* stream) {
  FATHOM_REQUIRE(sink >= 0 && local >= 0 && k - sink - local >= 1, FATHOM_ERR_SHAPE,
                 "sink_local_topk: need k - sink - local >= 1 (k=%lld sink=%lld local=%lld)", (long long)k,
                 (long long)sink, (long long)local);
  FATHOM_REQUIRE(local <= n && sink <= n, FATHOM_ERR_SHAPE, "sink_local_topk: sink/local exceed n");
  return run_select(scores, rows, n, n, k - sink - local, sink, n - local, 0, idx, k, nullptr, sink, local, workspace,
                    workspace_bytes, false, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int fathom_merge_topk(const float* cand_scores, const int64_t* cand_idx, int64_t rows, int64_t m, int64_t kk,
                                 int64_t* out_idx, float* out_scores, void* stream) {
  FATHOM_REQUIRE(cand_scores && cand_idx && out_idx, FATHOM_ERR_NULL, "merge_topk: NULL pointer");
  FATHOM_REQUIRE(rows >= 1 && rows <= 0x7fffffffLL && m >= 1 && m <= CAP && kk >= 1 && kk <= m && kk <= MAX_KK,
                 FATHOM_ERR_SHAPE, "merge_topk: need 1 <= kk <= min(m, %d), m <= %d", MAX_KK, CAP);
  const size_t smem = (CAP + MAX_KK) * sizeof(uint64_t);
  cudaFuncSetAttribute(merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  merge_kernel<<<(unsigned)rows, FT, smem, reinterpret_cast<cudaStream_t>(stream)>>>(cand_scores, cand_idx, m, kk,
                                                                                     out_idx, out_scores);
  return check_launch("merge_topk");
}

// ---------------------------------------------------------------------------------------------
// Top-k with a library-owned scratch area: for callers that cannot allocate device memory on the
// call path (a plugin host that has handed all device memory to its own pool, or a decode loop
// that cannot accept cudaMalloc's implicit device synchronisation), and so cannot provide the
// workspace fathom_sink_local_topk asks for.  The scratch is one file-scope device array sized for
// FATHOM_STATIC_TOPK_MAX_ROWS rows; every GPU that loads this library holds it until the process
// exits.  The array is created when the CUDA module of this file is loaded on a device: with CUDA's
// default lazy module loading that is the first call on that device which touches the module (this
// entry point's address look-up, or any selection call), so such a call belongs before the host pools
// its device memory or captures a stream.  Every call on a device shares the array: calls whose GPU
// work overlaps (other streams, other host threads) race on it and must be serialised by the caller.
// Each call clears the part that has to start at zero (histograms and counters); the rest is
// overwritten before it is read.
namespace fathom {
namespace {

constexpr size_t kStaticScratchBytes = ws_bytes(FATHOM_STATIC_TOPK_MAX_ROWS);

static __device__ __align__(256) unsigned char g_topk_scratch[kStaticScratchBytes];

// Device address of g_topk_scratch on the current device.  In host code the array's name is only a
// host-side stand-in, so the address is looked up with the device current, on every call: once the
// module is loaded the look-up is a table read, and a context torn down and created again (a device
// reset) can never leave a stale address behind.
int static_scratch(void** out) {
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_topk_scratch);
  if (e != cudaSuccess || p == nullptr)
    return set_error(FATHOM_ERR_CUDA, "sink_local_topk_static: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
  *out = p;
  return FATHOM_OK;
}

}  // namespace
}  // namespace fathom

extern "C" int fathom_sink_local_topk_static(const float* scores, int64_t rows, int64_t n, int64_t k, int64_t sink,
                                             int64_t local, int64_t* idx, void* stream) {
  FATHOM_REQUIRE(rows >= 1 && rows <= FATHOM_STATIC_TOPK_MAX_ROWS, FATHOM_ERR_SHAPE,
                 "sink_local_topk_static: rows=%lld outside 1..%d (the library-owned scratch holds at most %d rows; "
                 "use fathom_sink_local_topk with a caller workspace for more)",
                 (long long)rows, FATHOM_STATIC_TOPK_MAX_ROWS, FATHOM_STATIC_TOPK_MAX_ROWS);
  FATHOM_REQUIRE(ws_bytes(rows) <= kStaticScratchBytes, FATHOM_ERR_WORKSPACE, "sink_local_topk_static: scratch too small");
  void* scratch = nullptr;
  const int r = static_scratch(&scratch);
  if (r != FATHOM_OK) return r;
  return fathom_sink_local_topk(scores, rows, n, k, sink, local, idx, scratch, kStaticScratchBytes, stream);
}
