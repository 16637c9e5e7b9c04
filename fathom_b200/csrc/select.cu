// Top-k selection over score rows: sink_local_topk (kernels/bitplane.py:372-378) and the
// merge of per-shard candidates.
//
// Output order is (score descending, index ascending); every tie is broken by the index, so
// the selection is deterministic and a context-sharded scan merges to the same list.
//
// Fast path, three launches on the caller's stream:
//   1 hist      many CTAs per row: 4096-bin histogram of the top 12 bits of the order-
//               preserving key of every unmasked score (masked tokens get the key of -inf);
//               shared-memory histogram, flushed to the row's global histogram with atomics.
//   2 collect   many CTAs per row: each finds the boundary bin b* (the largest bin with at least
//               kk keys at or above it) from the global histogram, then appends every key in
//               bins >= b* as a 64-bit (key << 32 | ~index) candidate, warp-aggregated atomics.
//   3 finalize  one CTA per row: bitonic sort of the candidates in shared memory, descending
//               on (key, ~index), then the first kk.  If a row has more candidates than the
//               buffer holds (massive ties, or kk close to n) it switches to an exact radix
//               select over the whole row (12+12+8 bits) and an index-ordered compaction of
//               the keys equal to the threshold.
#include "common.cuh"

#include <atomic>

namespace fathom {
namespace {

constexpr int HBITS = 12;
constexpr int NBINS = 1 << HBITS;
constexpr int CAP = 8192;          // candidates kept per row in the fast path
constexpr int MAX_KK = 4096;
constexpr int CHUNK = 16384;       // scores per CTA in the hist / collect passes
constexpr int HT = 512;            // threads of hist / collect CTAs
constexpr int FT = 1024;           // threads of the finalize CTA

struct Workspace {
  uint32_t* hist;   // [rows][NBINS]
  uint32_t* count;  // [rows]
  uint64_t* cand;   // [rows][CAP]
};

size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

size_t ws_bytes(int64_t rows) {
  return align256(rows * NBINS * sizeof(uint32_t)) + align256(rows * sizeof(uint32_t)) +
         align256(rows * (size_t)CAP * sizeof(uint64_t));
}

Workspace carve(void* base, int64_t rows) {
  char* p = static_cast<char*>(base);
  Workspace w;
  w.hist = reinterpret_cast<uint32_t*>(p);
  p += align256(rows * NBINS * sizeof(uint32_t));
  w.count = reinterpret_cast<uint32_t*>(p);
  p += align256(rows * sizeof(uint32_t));
  w.cand = reinterpret_cast<uint64_t*>(p);
  return w;
}

__device__ __forceinline__ uint32_t masked_key(const float* row, int64_t i, int64_t mask_lo, int64_t mask_hi) {
  return (i >= mask_lo && i < mask_hi) ? f2key(row[i]) : KEY_NEG_INF;
}

__global__ void __launch_bounds__(HT) hist_kernel(const float* __restrict__ scores, int64_t n, int64_t row_stride,
                                                  int64_t mask_lo, int64_t mask_hi, uint32_t* __restrict__ ghist) {
  __shared__ uint32_t sh[NBINS];
  const int64_t row = blockIdx.y;
  for (int b = threadIdx.x; b < NBINS; b += HT) sh[b] = 0;
  __syncthreads();
  const float* r = scores + row * row_stride;
  const int64_t i0 = (int64_t)blockIdx.x * CHUNK;
  const int64_t i1 = i0 + CHUNK < n ? i0 + CHUNK : n;
  for (int64_t i = i0 + threadIdx.x; i < i1; i += HT) atomicAdd(&sh[masked_key(r, i, mask_lo, mask_hi) >> (32 - HBITS)], 1u);
  __syncthreads();
  uint32_t* gh = ghist + row * NBINS;
  for (int b = threadIdx.x; b < NBINS; b += HT)
    if (sh[b]) atomicAdd(&gh[b], sh[b]);
}

// Boundary bin from a row histogram held in shared memory, with `nt` threads (multiple of 32).
// Returns (to every thread) the largest bin b with sum_{b' >= b} hist[b'] >= kk.
__device__ int boundary_bin(const uint32_t* s_hist, int64_t kk, uint32_t* s_part, int* s_res) {
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

__global__ void __launch_bounds__(HT) collect_kernel(const float* __restrict__ scores, int64_t n, int64_t row_stride,
                                                     int64_t kk, int64_t mask_lo, int64_t mask_hi,
                                                     const uint32_t* __restrict__ ghist, uint32_t* __restrict__ count,
                                                     uint64_t* __restrict__ cand) {
  __shared__ uint32_t s_hist[NBINS];
  __shared__ uint32_t s_part[HT];
  __shared__ int s_res;
  const int64_t row = blockIdx.y;
  for (int b = threadIdx.x; b < NBINS; b += HT) s_hist[b] = ghist[row * NBINS + b];
  __syncthreads();
  const uint32_t bstar = (uint32_t)boundary_bin(s_hist, kk, s_part, &s_res);
  const float* r = scores + row * row_stride;
  const int64_t i0 = (int64_t)blockIdx.x * CHUNK;
  const int64_t i1 = i0 + CHUNK < n ? i0 + CHUNK : n;
  const int lane = threadIdx.x & 31;
  uint64_t* cr = cand + row * CAP;
  for (int64_t base = i0; base < i1; base += HT) {
    const int64_t i = base + threadIdx.x;
    uint32_t key = 0;
    bool take = false;
    if (i < i1) {
      key = masked_key(r, i, mask_lo, mask_hi);
      take = (key >> (32 - HBITS)) >= bstar;
    }
    const uint32_t m = __ballot_sync(0xffffffffu, take);
    if (m) {
      uint32_t pos0 = 0;
      if (lane == 0) pos0 = atomicAdd(&count[row], (uint32_t)__popc(m));
      pos0 = __shfl_sync(0xffffffffu, pos0, 0);
      if (take) {
        const uint32_t pos = pos0 + __popc(m & ((1u << lane) - 1));
        if (pos < CAP) cr[pos] = ((uint64_t)key << 32) | (uint32_t)(~(uint32_t)i);
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

// Block-wide exclusive scan of one value per thread (blockDim.x <= 1024). Returns the prefix;
// *total receives the block sum.
__device__ uint32_t block_exclusive_scan(uint32_t v, uint32_t* s_warp, uint32_t* total) {
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

__global__ void __launch_bounds__(FT) finalize_kernel(const float* __restrict__ scores, int64_t n, int64_t row_stride,
                                                      int64_t kk, int64_t mask_lo, int64_t mask_hi,
                                                      const uint32_t* __restrict__ count,
                                                      const uint64_t* __restrict__ cand, int64_t index_offset,
                                                      int64_t* __restrict__ out_idx, int64_t out_stride,
                                                      float* __restrict__ out_scores, int64_t append_sink,
                                                      int64_t append_local) {
  extern __shared__ uint64_t s_buf[];  // CAP entries
  __shared__ uint32_t s_hist[NBINS];
  __shared__ uint32_t s_part[FT];
  __shared__ uint32_t s_warp[33];
  __shared__ uint32_t s_cnt;
  __shared__ int s_res;
  const int64_t row = blockIdx.x;
  const uint32_t cnt = count[row];
  int P;
  if (cnt <= (uint32_t)CAP) {
    P = next_pow2((int)cnt);
    for (int i = threadIdx.x; i < P; i += blockDim.x) s_buf[i] = i < (int)cnt ? cand[row * CAP + i] : 0ull;
    __syncthreads();
  } else {
    exact_select_row(scores + row * row_stride, n, kk, mask_lo, mask_hi, s_buf, s_hist, s_part, &s_res, s_warp, &s_cnt);
    P = next_pow2((int)kk);
    for (int i = (int)kk + threadIdx.x; i < P; i += blockDim.x) s_buf[i] = 0ull;
    __syncthreads();
  }
  bitonic_desc(s_buf, P);
  int64_t* o = out_idx + row * out_stride;
  for (int i = threadIdx.x; i < kk; i += blockDim.x) {
    const uint64_t v = s_buf[i];
    o[i] = (int64_t)(uint32_t)(~(uint32_t)v) + index_offset;
    if (out_scores) out_scores[row * kk + i] = key2f((uint32_t)(v >> 32));
  }
  for (int64_t i = threadIdx.x; i < append_sink; i += blockDim.x) o[kk + i] = i;
  for (int64_t i = threadIdx.x; i < append_local; i += blockDim.x) o[kk + append_sink + i] = n - append_local + i;
}

__global__ void __launch_bounds__(FT) merge_kernel(const float* __restrict__ cs, const int64_t* __restrict__ ci,
                                                   int64_t m, int64_t kk, int64_t* __restrict__ out_idx,
                                                   float* __restrict__ out_scores) {
  extern __shared__ uint64_t s_buf[];
  const int64_t row = blockIdx.x;
  const int P = next_pow2((int)m);
  for (int i = threadIdx.x; i < P; i += blockDim.x)
    s_buf[i] = i < m ? ((uint64_t)f2key(cs[row * m + i]) << 32) | (uint32_t)(~(uint32_t)ci[row * m + i]) : 0ull;
  __syncthreads();
  bitonic_desc(s_buf, P);
  for (int i = threadIdx.x; i < kk; i += blockDim.x) {
    const uint64_t v = s_buf[i];
    out_idx[row * kk + i] = (int64_t)(uint32_t)(~(uint32_t)v);
    if (out_scores) out_scores[row * kk + i] = key2f((uint32_t)(v >> 32));
  }
}

int run_select(const float* scores, int64_t rows, int64_t n, int64_t row_stride, int64_t kk, int64_t mask_lo,
               int64_t mask_hi, int64_t index_offset, int64_t* out_idx, int64_t out_stride, float* out_scores,
               int64_t append_sink, int64_t append_local, void* workspace, size_t workspace_bytes, cudaStream_t st) {
  FATHOM_REQUIRE(scores && out_idx, FATHOM_ERR_NULL, "select_topk: NULL pointer");
  FATHOM_REQUIRE(rows >= 1 && rows <= 65535 && n >= 1 && n <= 0xffffffffLL, FATHOM_ERR_SHAPE,
                 "select_topk: need 1 <= rows <= 65535 and 1 <= n < 2^32");
  FATHOM_REQUIRE(kk >= 1 && kk <= MAX_KK && kk <= n, FATHOM_ERR_SHAPE, "select_topk: kk=%lld outside 1..min(4096, n=%lld)",
                 (long long)kk, (long long)n);
  FATHOM_REQUIRE(row_stride >= n && out_stride >= kk + append_sink + append_local, FATHOM_ERR_SHAPE,
                 "select_topk: bad strides");
  FATHOM_REQUIRE(workspace != nullptr, FATHOM_ERR_NULL, "select_topk: workspace is NULL");
  FATHOM_REQUIRE(workspace_bytes >= ws_bytes(rows) && (reinterpret_cast<uintptr_t>(workspace) & 255) == 0,
                 FATHOM_ERR_WORKSPACE, "select_topk: workspace needs %zu bytes, 256-byte aligned (got %zu)",
                 ws_bytes(rows), workspace_bytes);
  Workspace w = carve(workspace, rows);
  cudaError_t e = cudaMemsetAsync(workspace, 0, reinterpret_cast<char*>(w.cand) - static_cast<char*>(workspace), st);
  if (e != cudaSuccess) return set_error(FATHOM_ERR_CUDA, "select_topk: memset: %s", cudaGetErrorString(e));
  const int64_t chunks = cdiv(n, CHUNK);
  dim3 grid((unsigned)chunks, (unsigned)rows);
  hist_kernel<<<grid, HT, 0, st>>>(scores, n, row_stride, mask_lo, mask_hi, w.hist);
  collect_kernel<<<grid, HT, 0, st>>>(scores, n, row_stride, kk, mask_lo, mask_hi, w.hist, w.count, w.cand);
  const size_t smem = CAP * sizeof(uint64_t);
  static bool attr_set = false;
  if (!attr_set) {
    cudaFuncSetAttribute(finalize_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    cudaFuncSetAttribute(merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    attr_set = true;
  }
  finalize_kernel<<<(unsigned)rows, FT, smem, st>>>(scores, n, row_stride, kk, mask_lo, mask_hi, w.count, w.cand,
                                                     index_offset, out_idx, out_stride, out_scores, append_sink,
                                                     append_local);
  return check_launch("select_topk");
}

}  // namespace
}  // namespace fathom

using namespace fathom;

extern "C" size_t fathom_select_workspace_bytes(int64_t rows, int64_t n, int64_t kk) {
  (void)n;
  (void)kk;
  return rows > 0 ? ws_bytes(rows) : 0;
}

extern "C" int fathom_select_topk(const float* scores, int64_t rows, int64_t n, int64_t row_stride, int64_t kk,
                                  int64_t mask_lo, int64_t mask_hi, int64_t index_offset, int64_t* out_idx,
                                  int64_t out_stride, float* out_scores, void* workspace, size_t workspace_bytes,
                                  void* stream) {
  return run_select(scores, rows, n, row_stride, kk, mask_lo, mask_hi, index_offset, out_idx, out_stride, out_scores,
                    0, 0, workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int fathom_sink_local_topk(const float* scores, int64_t rows, int64_t n, int64_t k, int64_t sink,
                                      int64_t local, int64_t* idx, void* workspace, size_t workspace_bytes,
                                      void* stream) {
  FATHOM_REQUIRE(sink >= 0 && local >= 0 && k - sink - local >= 1, FATHOM_ERR_SHAPE,
                 "sink_local_topk: need k - sink - local >= 1 (k=%lld sink=%lld local=%lld)", (long long)k,
                 (long long)sink, (long long)local);
  FATHOM_REQUIRE(local <= n && sink <= n, FATHOM_ERR_SHAPE, "sink_local_topk: sink/local exceed n");
  return run_select(scores, rows, n, n, k - sink - local, sink, n - local, 0, idx, k, nullptr, sink, local, workspace,
                    workspace_bytes, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int fathom_merge_topk(const float* cand_scores, const int64_t* cand_idx, int64_t rows, int64_t m, int64_t kk,
                                 int64_t* out_idx, float* out_scores, void* stream) {
  FATHOM_REQUIRE(cand_scores && cand_idx && out_idx, FATHOM_ERR_NULL, "merge_topk: NULL pointer");
  FATHOM_REQUIRE(rows >= 1 && rows <= 0x7fffffffLL && m >= 1 && m <= CAP && kk >= 1 && kk <= m, FATHOM_ERR_SHAPE,
                 "merge_topk: need 1 <= kk <= m <= %d", CAP);
  const size_t smem = CAP * sizeof(uint64_t);
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
// exits.  Every call on a device shares it: calls whose GPU work overlaps (other streams, other
// host threads) race on it and must be serialised by the caller.  Each call clears the part that
// has to start at zero (histograms and counters); the rest is overwritten before it is read.
namespace fathom {
namespace {

constexpr size_t static_align256(size_t x) { return (x + 255) & ~(size_t)255; }
constexpr size_t kStaticScratchBytes =
    static_align256((size_t)FATHOM_STATIC_TOPK_MAX_ROWS * NBINS * sizeof(uint32_t)) +
    static_align256((size_t)FATHOM_STATIC_TOPK_MAX_ROWS * sizeof(uint32_t)) +
    static_align256((size_t)FATHOM_STATIC_TOPK_MAX_ROWS * CAP * sizeof(uint64_t));

static __device__ __align__(256) unsigned char g_topk_scratch[kStaticScratchBytes];

constexpr int kMaxDevices = 64;
std::atomic<void*> g_topk_scratch_ptr[kMaxDevices];

// Device address of g_topk_scratch on the current device.  In host code the array's name is only a
// host-side stand-in, so the address is looked up once per device (with that device current) and
// cached; the first call on each device therefore does this set-up.
int static_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(FATHOM_ERR_CUDA, "sink_local_topk_static: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return set_error(FATHOM_ERR_UNSUPPORTED, "sink_local_topk_static: device %d", dev);
  void* p = g_topk_scratch_ptr[dev].load(std::memory_order_acquire);
  if (p == nullptr) {
    e = cudaGetSymbolAddress(&p, g_topk_scratch);
    if (e != cudaSuccess || p == nullptr)
      return set_error(FATHOM_ERR_CUDA, "sink_local_topk_static: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    g_topk_scratch_ptr[dev].store(p, std::memory_order_release);
  }
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
