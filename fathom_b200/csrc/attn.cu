// Zero-copy K/V row gather and decode attention over the selected rows
// (scripts/B_e2e_offload_v2.py:73-83 gather_rows, :226-244 offload_attn tail;
//  HBM twin scripts/B_kernel_bench.py:26-31 gather_attn).
//
// decode attention from host-resident rows, three launches (device-resident rows: one launch of
// attend_kernel<.., false>, which reads each pick's rows in place):
//   1 dedupe   one CTA per (batch, kv-head): the G*k picks go into a shared-memory hash table,
//              a block scan ranks the distinct indices; slot map (query head, pick) -> unique row,
//              the unique index list (in table order) and its length.
//   2 gather   many CTAs per (batch, kv-head): each unique K and V row is fetched ONCE from its source
//              (mapped host memory over the host link, or the device-resident recent buffer) into a
//              device staging area; 16 lanes x 16 B per 256-byte row, 4 rows in flight per lane.
//              Spreading the rows over every SM keeps enough requests in flight for the link.
//   3 attend   16 or 32 warps per (batch, query head), in one CTA or a cluster of 4 or 8 CTAs: a warp
//              takes 4 picks at a time (8 lanes x 16 dims each) from the staging area (L2-resident),
//              q.K^T / sqrt(128), an online softmax and the running weighted sum of V; the warp
//              states are merged in global warp order.  fp32 math.
// A pick outside the caller's owned index range [idx_lo, idx_hi) is skipped (context shards);
// the partial form writes the unnormalised output with its (max, sum of exp), base 2.
#include "common.cuh"

#include <stdlib.h>

#include <cooperative_groups.h>

namespace fathom {
namespace {

constexpr int DT = 1024;      // dedupe threads
constexpr int GT = 256;       // gather threads
constexpr int GROWS = 64;     // unique rows per gather CTA
constexpr int MAX_M = 16384;  // G*k per (batch, kv-head) handled by one dedupe CTA

size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = v > 0 ? v : 148;
  }
  return cached[dev];
}

// True for device (HBM) memory; false for host memory (mapped or not), managed memory and unknown pointers.
bool device_memory(const void* p) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();   // clear the error of an unregistered pointer
    return false;
  }
  return a.type == cudaMemoryTypeDevice;
}

struct DecodeWs {
  int32_t* slot;       // [BH][M] pick -> unique row (-1: not owned)
  int64_t* uniq;       // [BH][M] unique indices, ascending (-1: not owned)
  int32_t* ucount;     // [BH] number of unique indices
  uint16_t* kstage;    // [BH][M][128] bf16
  uint16_t* vstage;    // [BH][M][128] bf16
};

size_t decode_ws_bytes(int64_t BH, int64_t M) {
  return align256(BH * M * sizeof(int32_t)) + align256(BH * M * sizeof(int64_t)) + align256(BH * sizeof(int32_t)) +
         2 * align256(BH * M * D * sizeof(uint16_t));
}

DecodeWs carve(void* base, int64_t BH, int64_t M) {
  char* p = static_cast<char*>(base);
  DecodeWs w;
  w.slot = reinterpret_cast<int32_t*>(p);
  p += align256(BH * M * sizeof(int32_t));
  w.uniq = reinterpret_cast<int64_t*>(p);
  p += align256(BH * M * sizeof(int64_t));
  w.ucount = reinterpret_cast<int32_t*>(p);
  p += align256(BH * sizeof(int32_t));
  w.kstage = reinterpret_cast<uint16_t*>(p);
  p += align256(BH * M * D * sizeof(uint16_t));
  w.vstage = reinterpret_cast<uint16_t*>(p);
  return w;
}

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
    const uint32_t w = lane < nw ? s_warp[lane] : 0u;
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

constexpr uint32_t EMPTY = 0xFFFFFFFFu;
constexpr int MAX_TS = 32768;         // hash table slots (128 KB of shared memory; + M keys, 2 x NB bins)
constexpr int PICKS_PER_THREAD = MAX_M / DT;
constexpr int NB = 2048;              // rank buckets (high bits of the row index)
constexpr int MAX_PER = MAX_TS / DT;  // table slots per dedupe thread

__device__ __forceinline__ uint32_t hash_slot(uint32_t key, int log2ts) {
  return (key * 0x9E3779B1u) >> (32 - log2ts);
}

// One CTA per (batch, kv-head).  Every owned pick is inserted into an open-addressing table in
// shared memory (atomicCAS, linear probing; the table has at least twice as many slots as picks,
// so a probe sequence always ends at an empty slot or at its own key).  The distinct indices are
// then ranked in ascending order: a counting pass over NB buckets of their high bits, a block scan,
// a scatter into bucket order, and within each (small) bucket a count of the smaller keys.  The
// unique list is therefore sorted, so the gather walks the source in address order (fewer address
// translations per byte over the host link), and every rank is independent of the insert order.
// Each pick remembers its table slot and reads its rank.
__global__ void __launch_bounds__(DT) dedupe_kernel(const int64_t* __restrict__ idx, int64_t M, int64_t idx_lo,
                                                    int64_t idx_hi, int64_t row_limit, int log2ts, int bshift,
                                                    int32_t* __restrict__ slot,
                                                    int64_t* __restrict__ uniq, int32_t* __restrict__ ucount) {
  extern __shared__ uint32_t s_tab[];  // 1 << log2ts slots, then M keys in bucket order
  __shared__ uint32_t s_warp[33];
  __shared__ uint32_t s_bin[NB], s_cur[NB];
  const int64_t bh = blockIdx.x;
  const int TS = 1 << log2ts;
  uint32_t* s_sorted = s_tab + TS;
  for (int i = threadIdx.x; i < TS; i += blockDim.x) s_tab[i] = EMPTY;
  for (int b = threadIdx.x; b < NB; b += blockDim.x) s_bin[b] = 0u;
  __syncthreads();
  const int64_t* ib = idx + bh * M;
  int pos[PICKS_PER_THREAD];
  int64_t tv[PICKS_PER_THREAD];   // every pick load in flight before the first insert
#pragma unroll
  for (int u = 0; u < PICKS_PER_THREAD; ++u) {
    const int64_t i = threadIdx.x + (int64_t)u * DT;
    tv[u] = i < M ? ib[i] : -1;
  }
#pragma unroll
  for (int u = 0; u < PICKS_PER_THREAD; ++u) {
    const int64_t i = threadIdx.x + (int64_t)u * DT;
    pos[u] = -1;
    if (i < M) {
      const int64_t t = tv[u];
      if (t >= idx_lo && t < idx_hi && t - idx_lo < row_limit) {
        const uint32_t key = (uint32_t)(t - idx_lo);
        uint32_t h = hash_slot(key, log2ts);
        for (int probe = 0; probe < TS; ++probe) {
          const uint32_t old = atomicCAS(&s_tab[h], EMPTY, key);
          if (old == EMPTY || old == key) {
            pos[u] = (int)h;
            break;
          }
          h = (h + 1) & (TS - 1);
        }
      }
    }
  }
  __syncthreads();
  // ascending ranks of the distinct keys (each thread a contiguous chunk of the table)
  const int per = TS / DT > 0 ? TS / DT : 1;
  const int h0 = threadIdx.x * per;
  const int h1 = h0 + per < TS ? h0 + per : TS;
  for (int h = h0; h < h1; ++h)
    if (s_tab[h] != EMPTY) atomicAdd(&s_bin[s_tab[h] >> bshift], 1u);
  __syncthreads();
  uint32_t bsum = 0;   // bins 2t, 2t+1 of thread t (NB = 2 * DT)
  const uint32_t c0 = s_bin[2 * threadIdx.x], c1 = s_bin[2 * threadIdx.x + 1];
  uint32_t total;
  bsum = block_exclusive_scan(c0 + c1, s_warp, &total);
  s_bin[2 * threadIdx.x] = bsum;
  s_bin[2 * threadIdx.x + 1] = bsum + c0;
  s_cur[2 * threadIdx.x] = bsum;
  s_cur[2 * threadIdx.x + 1] = bsum + c0;
  __syncthreads();
  for (int h = h0; h < h1; ++h)
    if (s_tab[h] != EMPTY) s_sorted[atomicAdd(&s_cur[s_tab[h] >> bshift], 1u)] = s_tab[h];
  __syncthreads();   // s_cur[b] is now the end of bucket b
  uint32_t myrank[MAX_PER];
  int64_t* ul = uniq + bh * M;
  for (int h = h0; h < h1; ++h) {
    const uint32_t x = s_tab[h];
    if (x == EMPTY) continue;
    const uint32_t b = x >> bshift;
    uint32_t r = s_bin[b];
    for (uint32_t t = s_bin[b]; t < s_cur[b]; ++t) r += s_sorted[t] < x;
    myrank[h - h0] = r;
    ul[r] = (int64_t)x;
  }
  __syncthreads();   // every key read: the slots may now hold ranks
  for (int h = h0; h < h1; ++h)
    if (s_tab[h] != EMPTY) s_tab[h] = myrank[h - h0];
  __syncthreads();
  int32_t* sl = slot + bh * M;
#pragma unroll
  for (int u = 0; u < PICKS_PER_THREAD; ++u) {
    const int64_t i = threadIdx.x + (int64_t)u * DT;
    if (i < M) sl[i] = pos[u] >= 0 ? (int32_t)s_tab[pos[u]] : -1;
  }
  if (threadIdx.x == 0) ucount[bh] = (int32_t)total;
}

__global__ void __launch_bounds__(GT) gather_kernel(const int32_t* __restrict__ ucount, const int64_t* __restrict__ uniq,
                                                    int64_t M, const uint4* __restrict__ ksrc,
                                                    const uint4* __restrict__ vsrc, int64_t cap, int64_t rs16,
                                                    int64_t n_host,
                                                    const uint4* __restrict__ krec, const uint4* __restrict__ vrec,
                                                    int64_t recent_cap, uint4* __restrict__ kstage,
                                                    uint4* __restrict__ vstage) {
  constexpr int LPR = D * 2 / 16;          // 16 lanes x 16 B per row
  constexpr int RPP = GT / LPR;            // rows per pass
  constexpr int PASSES = GROWS / RPP;      // 4
  const int64_t bh = blockIdx.y;
  const int64_t U = ucount[bh];
  const int64_t r0 = (int64_t)blockIdx.x * GROWS;
  if (r0 >= U) return;
  const int sub = threadIdx.x % LPR;
  const int rr = threadIdx.x / LPR;
  uint4 kv[PASSES], vv[PASSES];
  int64_t rows[PASSES];
#pragma unroll
  for (int u = 0; u < PASSES; ++u) {
    const int64_t r = r0 + u * RPP + rr;
    const int64_t t = r < U ? uniq[bh * M + r] : -1;
    rows[u] = t >= 0 ? r : -1;
    if (t >= 0) {
      const uint4* kp;
      const uint4* vp;
      if (t < n_host) {  // host rows: rs16 uint4 between consecutive rows (LPR when K and V are separate)
        kp = ksrc + (bh * cap + t) * rs16;
        vp = vsrc + (bh * cap + t) * rs16;
      } else {
        kp = krec + (bh * recent_cap + (t - n_host)) * LPR;
        vp = vrec + (bh * recent_cap + (t - n_host)) * LPR;
      }
      kv[u] = kp[sub];
      vv[u] = vp[sub];
    }
  }
#pragma unroll
  for (int u = 0; u < PASSES; ++u) {
    if (rows[u] >= 0) {
      kstage[(bh * M + rows[u]) * LPR + sub] = kv[u];
      vstage[(bh * M + rows[u]) * LPR + sub] = vv[u];
    }
  }
}

// ---- attention over the picks --------------------------------------------------------------------
// Layout shared by every attention kernel (staged host rows, rows read in place, one CTA or a cluster
// of CTAs per (batch, query head)), so all of them sum in the same order and give the same bits:
//  * NW warps per (batch, query head) (16, or 32 when the heads are few; fixed by the head count, so
//    every kernel that serves a launch shape uses the same layout; the CTA split does not change the
//    sums); global warp w owns picks
//    [w * PW, w * PW + PW), PW = ceil(k / NW);
//  * a warp takes PG = 4 picks at once: lane group j (lanes 8j .. 8j + 7) takes picks j, j + 4, j + 8, ..
//    of each 32-pick chunk, and lane i of a group holds dims [16i, 16i + 16) of q, K, V and the output;
//  * a score is the group's 8 partial dots summed by 3 shuffles; q is pre-scaled by log2(e) / sqrt(128),
//    so scores are in base-2 units and weights are exp2(s - m) (the packed partials' m is base 2);
//  * each group keeps an online softmax (max, sum, 16 dims of the weighted V sum per lane), DU picks
//    per step; a warp's 4 group states are merged by two symmetric shuffle steps, then the NW warp
//    states of a (batch, query head) in global warp order.
constexpr int PG = 4;           // picks per warp instruction (lane groups of 8)
constexpr int DPL = D / 8;      // dims per lane
constexpr int DU = 2;           // picks per lane group per step
constexpr float QSCALE = (float)(1.4426950408889634 / 11.313708498984761);   // log2(e) / sqrt(128)

__device__ __forceinline__ float2 bf16x2_f2(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}

// One lane's share of its group's online softmax.
struct GroupSoftmax {
  float m = -INFINITY, l = 0.0f;
  float2 a[DPL / 2];
  __device__ __forceinline__ GroupSoftmax() {
#pragma unroll
    for (int e = 0; e < DPL / 2; ++e) a[e] = make_float2(0.0f, 0.0f);
  }

  // DU picks of the group: kr[u] / vr[u] point at this lane's 16 dims of the pick's K and V rows,
  // nullptr for a pick the group does not own.  sq: this lane's 16 pre-scaled query dims (shared).
  // Every lane of the warp calls this (the score sums shuffle across the group's lanes).
  __device__ __forceinline__ void add(const float* sq, const uint16_t* const (&kr)[DU],
                                      const uint16_t* const (&vr)[DU]) {
    uint4 kw[DU][2], vw[DU][2];
#pragma unroll
    for (int u = 0; u < DU; ++u) {
      if (kr[u] != nullptr) {
        kw[u][0] = *reinterpret_cast<const uint4*>(kr[u]);
        kw[u][1] = *reinterpret_cast<const uint4*>(kr[u] + 8);
        vw[u][0] = *reinterpret_cast<const uint4*>(vr[u]);
        vw[u][1] = *reinterpret_cast<const uint4*>(vr[u] + 8);
      } else {
        kw[u][0] = kw[u][1] = vw[u][0] = vw[u][1] = make_uint4(0, 0, 0, 0);
      }
    }
    float s[DU];
#pragma unroll
    for (int u = 0; u < DU; ++u) {
      float2 d = make_float2(0.0f, 0.0f);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float4 q0 = *reinterpret_cast<const float4*>(sq + 8 * h);
        const float4 q1 = *reinterpret_cast<const float4*>(sq + 8 * h + 4);
        d = __ffma2_rn(make_float2(q0.x, q0.y), bf16x2_f2(kw[u][h].x), d);
        d = __ffma2_rn(make_float2(q0.z, q0.w), bf16x2_f2(kw[u][h].y), d);
        d = __ffma2_rn(make_float2(q1.x, q1.y), bf16x2_f2(kw[u][h].z), d);
        d = __ffma2_rn(make_float2(q1.z, q1.w), bf16x2_f2(kw[u][h].w), d);
      }
      s[u] = d.x + d.y;
    }
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) {
#pragma unroll
      for (int u = 0; u < DU; ++u) s[u] += __shfl_xor_sync(0xffffffffu, s[u], o);
    }
    float mx = m;
#pragma unroll
    for (int u = 0; u < DU; ++u) {
      if (kr[u] == nullptr) s[u] = -INFINITY;
      mx = fmaxf(mx, s[u]);
    }
    if (mx == -INFINITY) return;   // nothing owned yet
    if (mx > m) {                  // the running max moved: rescale (a factor of exactly 1 otherwise)
      const float corr = m == -INFINITY ? 0.0f : exp2f(m - mx);
      l *= corr;
#pragma unroll
      for (int e = 0; e < DPL / 2; ++e) a[e] = make_float2(a[e].x * corr, a[e].y * corr);
      m = mx;
    }
#pragma unroll
    for (int u = 0; u < DU; ++u) {
      const float p = s[u] == -INFINITY ? 0.0f : exp2f(s[u] - m);
      l += p;
      const float2 pp = make_float2(p, p);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        a[4 * h + 0] = __ffma2_rn(pp, bf16x2_f2(vw[u][h].x), a[4 * h + 0]);
        a[4 * h + 1] = __ffma2_rn(pp, bf16x2_f2(vw[u][h].y), a[4 * h + 1]);
        a[4 * h + 2] = __ffma2_rn(pp, bf16x2_f2(vw[u][h].z), a[4 * h + 2]);
        a[4 * h + 3] = __ffma2_rn(pp, bf16x2_f2(vw[u][h].w), a[4 * h + 3]);
      }
    }
  }

  // Merges the 4 group states of the warp (lanes i, i + 8, i + 16, i + 24 hold the same dims); every
  // lane ends with the warp's state.  Each step is symmetric in its two states (two rounded products,
  // then their sum), so all groups hold the same bits.
  __device__ __forceinline__ void merge_groups() {
#pragma unroll
    for (int o = 8; o < 32; o <<= 1) {
      const float mo = __shfl_xor_sync(0xffffffffu, m, o);
      const float lo = __shfl_xor_sync(0xffffffffu, l, o);
      const float M = fmaxf(m, mo);
      const float e1 = m == -INFINITY ? 0.0f : exp2f(m - M);
      const float e2 = mo == -INFINITY ? 0.0f : exp2f(mo - M);
      l = __fadd_rn(__fmul_rn(l, e1), __fmul_rn(lo, e2));
#pragma unroll
      for (int e = 0; e < DPL / 2; ++e) {
        const float ox = __shfl_xor_sync(0xffffffffu, a[e].x, o);
        const float oy = __shfl_xor_sync(0xffffffffu, a[e].y, o);
        a[e] = make_float2(__fadd_rn(__fmul_rn(a[e].x, e1), __fmul_rn(ox, e2)),
                           __fadd_rn(__fmul_rn(a[e].y, e1), __fmul_rn(oy, e2)));
      }
      m = M;
    }
  }
};

// Where the picks' rows are.  Staged: slot s >= 0 of the staging area (host rows after dedupe + gather).
// In place: pick t in [idx_lo, idx_hi), row r = t - idx_lo below n_host + recent_cap: row r of the
// source (r < n_host, row_stride elements apart) or row r - n_host of the recent buffer.
struct PickRows {
  const int64_t* idx;       // in place: [BH*G][k] picks
  const int32_t* slot;      // staged: [BH][M] pick -> staging slot
  const uint16_t* ksrc;     // staged: kstage [BH][M][128]; in place: the K source
  const uint16_t* vsrc;
  int64_t M, cap, row_stride, n_host, recent_cap, idx_lo, idx_hi;
  const uint16_t* krec;
  const uint16_t* vrec;
};

// NW warps per (batch, query head), CWW per CTA, CS = NW / CWW CTAs (one cluster) per (batch, query
// head): global warp gw = rank * CWW + warp.  Every warp stores its state into the shared memory of the
// cluster's first CTA (distributed shared memory; its own when CS = 1), which merges the NW states in
// global warp order and writes the output or the packed partial [BH*G][130] = (sum_r 2^(s_r - m) V_r,
// m, l), m in base-2 units.
template <int NW, int CWW, bool STAGED>
__global__ void __launch_bounds__(CWW * 32, 32 / CWW) attend_kernel(const float* __restrict__ q, int G, int64_t k,
                                                                    PickRows pr, float* __restrict__ out_f32,
                                                                    uint16_t* __restrict__ out_bf16,
                                                                    float* __restrict__ out_packed) {
  namespace cg = cooperative_groups;
  constexpr int CS = NW / CWW;
  cg::cluster_group cluster = cg::this_cluster();
  __shared__ __align__(16) float s_q[D];
  __shared__ float s_m[NW], s_l[NW];               // the cluster's first CTA: every warp's state
  __shared__ __align__(16) float s_acc[NW][D];
  const unsigned crank = CS == 1 ? 0u : cluster.block_rank();
  const int64_t bhg = blockIdx.x / CS;
  const int64_t bh = bhg / G;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int grp = lane >> 3, sl = lane & 7;
  const int gw = (int)crank * CWW + warp;
  for (int d = tid; d < D; d += CWW * 32) s_q[d] = q[bhg * D + d] * QSCALE;
  __syncthreads();
  const float* sq = s_q + sl * DPL;
  const int64_t PW = (k + NW - 1) / NW;
  const int64_t p0 = (int64_t)gw * PW;
  const int64_t p1 = p0 + PW < k ? p0 + PW : k;
  GroupSoftmax st;
  for (int64_t c0 = p0; c0 < p1; c0 += 32) {   // uniform per warp
    // this lane's pick of the chunk: its staging slot or row (< 2^32 - 1, checked by the launcher), -1
    // when not owned
    int32_t mine = -1;
    if (c0 + lane < p1) {
      if constexpr (STAGED) {
        mine = pr.slot[bh * pr.M + (bhg % G) * k + c0 + lane];
      } else {
        const int64_t t = pr.idx[bhg * k + c0 + lane];
        if (t >= pr.idx_lo && t < pr.idx_hi && t - pr.idx_lo < pr.n_host + pr.recent_cap)
          mine = (int32_t)(uint32_t)(t - pr.idx_lo);
      }
    }
    const int nc = (int)(p1 - c0 < 32 ? p1 - c0 : 32);
    for (int s0 = 0; s0 < nc; s0 += PG * DU) {   // uniform per warp
      const uint16_t* kr[DU];
      const uint16_t* vr[DU];
#pragma unroll
      for (int u = 0; u < DU; ++u) {
        const int src = s0 + u * PG + grp;
        int32_t rr = __shfl_sync(0xffffffffu, mine, src & 31);
        if (src >= nc) rr = -1;
        kr[u] = vr[u] = nullptr;
        if (rr != -1) {
          if constexpr (STAGED) {
            const int64_t off = (bh * pr.M + rr) * D + sl * DPL;
            kr[u] = pr.ksrc + off;
            vr[u] = pr.vsrc + off;
          } else {
            const int64_t r = (int64_t)(uint32_t)rr;
            if (r < pr.n_host) {
              const int64_t off = (bh * pr.cap + r) * pr.row_stride + sl * DPL;
              kr[u] = pr.ksrc + off;
              vr[u] = pr.vsrc + off;
            } else {
              const int64_t off = (bh * pr.recent_cap + r - pr.n_host) * D + sl * DPL;
              kr[u] = pr.krec + off;
              vr[u] = pr.vrec + off;
            }
          }
        }
      }
      st.add(sq, kr, vr);
    }
  }
  st.merge_groups();
  // each warp stores its state into the first CTA's shared memory (distributed shared memory stores)
  float* dm = s_m;
  float* dl = s_l;
  float* da = &s_acc[0][0];
  if constexpr (CS > 1) {
    dm = cluster.map_shared_rank(s_m, 0);
    dl = cluster.map_shared_rank(s_l, 0);
    da = cluster.map_shared_rank(&s_acc[0][0], 0);
  }
  if (lane == 0) {
    dm[gw] = st.m;
    dl[gw] = st.l;
  }
  if (lane < 8) {
    float4* dst = reinterpret_cast<float4*>(da + gw * D + sl * DPL);
#pragma unroll
    for (int e = 0; e < DPL / 4; ++e)
      dst[e] = make_float4(st.a[2 * e].x, st.a[2 * e].y, st.a[2 * e + 1].x, st.a[2 * e + 1].y);
  }
  if constexpr (CS == 1) __syncthreads();
  else cluster.sync();   // every warp's state is in the first CTA's shared memory
  if (crank != 0) return;
  for (int d = tid; d < D; d += CWW * 32) {
    float Mx = -INFINITY;
#pragma unroll 8
    for (int w = 0; w < NW; ++w) Mx = fmaxf(Mx, s_m[w]);
    float L = 0.0f, O = 0.0f;
#pragma unroll 8
    for (int w = 0; w < NW; ++w) {
      const float e = s_m[w] == -INFINITY ? 0.0f : exp2f(s_m[w] - Mx);
      L = fmaf(s_l[w], e, L);
      O = fmaf(s_acc[w][d], e, O);
    }
    if (out_packed) {
      float* pk = out_packed + bhg * (D + 2);
      pk[d] = O;
      if (d == 0) {
        pk[D] = Mx;
        pk[D + 1] = L;
      }
    } else {
      const float o = O / L;
      if (out_f32) out_f32[bhg * D + d] = o;
      if (out_bf16) out_bf16[bhg * D + d] = __bfloat16_as_ushort(__float2bfloat16_rn(o));
    }
  }
}

// Warps and CTAs per (batch, query head) for `rows` of them: 32 warps in a cluster of 8 CTAs for fewer
// than SMs / 4 heads (latency: short per-group pick chains), 16 warps in a cluster of 4 up to 2 x SMs
// heads, one CTA of 16 warps beyond (measured on config-1, config-3 and 360-head launches).
// FATHOM_ATTN_NW (16 or 32) and FATHOM_ATTN_CS (1, 2, 4 or 8) override (tuning).
void attend_shape(int64_t rows, int* nw, int* cs) {
  const int64_t sms = sm_count();
  *nw = rows * 4 >= sms ? 16 : 32;
  *cs = rows >= 2 * sms ? 1 : rows * 4 >= sms ? 4 : 8;
  if (const char* e = getenv("FATHOM_ATTN_NW")) *nw = atoi(e) == 32 ? 32 : 16;
  if (const char* e = getenv("FATHOM_ATTN_CS")) {
    const int v = atoi(e);
    *cs = (v == 1 || v == 2 || v == 4 || v == 8) ? v : *cs;
  }
}

template <int NW, bool STAGED>
cudaError_t launch_attend_nw(cudaLaunchConfig_t* cfg, int cs, const float* q, int G, int64_t k, const PickRows& pr,
                             float* out_f32, uint16_t* out_bf16, float* out_packed) {
  cfg->blockDim = dim3((unsigned)(NW / cs * 32));
  switch (cs) {
    case 1: return cudaLaunchKernelEx(cfg, attend_kernel<NW, NW, STAGED>, q, G, k, pr, out_f32, out_bf16, out_packed);
    case 2:
      return cudaLaunchKernelEx(cfg, attend_kernel<NW, NW / 2, STAGED>, q, G, k, pr, out_f32, out_bf16, out_packed);
    case 4:
      return cudaLaunchKernelEx(cfg, attend_kernel<NW, NW / 4, STAGED>, q, G, k, pr, out_f32, out_bf16, out_packed);
    default:
      return cudaLaunchKernelEx(cfg, attend_kernel<NW, NW / 8, STAGED>, q, G, k, pr, out_f32, out_bf16, out_packed);
  }
}

template <bool STAGED>
int launch_attend(const float* q, int64_t BH, int G, int64_t k, const PickRows& pr, float* out_f32,
                  uint16_t* out_bf16, float* out_packed, cudaStream_t st) {
  const int64_t rows = BH * G;
  int nw = 16, cs = 1;
  attend_shape(rows, &nw, &cs);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(rows * cs));
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)cs;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = cs > 1 ? 1 : 0;
  const cudaError_t e = nw == 32 ? launch_attend_nw<32, STAGED>(&cfg, cs, q, G, k, pr, out_f32, out_bf16, out_packed)
                                 : launch_attend_nw<16, STAGED>(&cfg, cs, q, G, k, pr, out_f32, out_bf16, out_packed);
  if (e != cudaSuccess) return set_error(FATHOM_ERR_CUDA, "decode_attention: launch: %s", cudaGetErrorString(e));
  return check_launch("decode_attention");
}

// out = sum_p o_p 2^(m_p - M) / sum_p l_p 2^(m_p - M), M = max_p m_p: log-sum-exp merge of the
// partial attention of P context shards (m in base-2 units).  One CTA of 128 threads per (batch,
// query head).
__global__ void __launch_bounds__(D) combine_kernel(const float* __restrict__ parts, int64_t P, int64_t rows,
                                                    float* __restrict__ out_f32, uint16_t* __restrict__ out_bf16) {
  const int64_t row = blockIdx.x;
  const int t = threadIdx.x;
  constexpr int W = D + 2;  // packed part: o[128], m, l
  float M = -INFINITY;
  for (int64_t p = 0; p < P; ++p) M = fmaxf(M, parts[(p * rows + row) * W + D]);
  float L = 0.0f, acc = 0.0f;
  for (int64_t p = 0; p < P; ++p) {
    const float* pp = parts + (p * rows + row) * W;
    const float m = pp[D];
    const float w = m == -INFINITY ? 0.0f : exp2f(m - M);
    L = fmaf(pp[D + 1], w, L);
    acc = fmaf(pp[t], w, acc);
  }
  const float o = acc / L;
  if (out_f32) out_f32[row * D + t] = o;
  if (out_bf16) out_bf16[row * D + t] = __bfloat16_as_ushort(__float2bfloat16_rn(o));
}

__global__ void gather_rows_kernel(const uint4* __restrict__ src, int64_t cap, const int32_t* __restrict__ idx,
                                   int64_t R, int lpr, uint4* __restrict__ dst) {
  const int64_t bh = blockIdx.y;
  const int rows_per_cta = blockDim.x / lpr;
  const int64_t r = (int64_t)blockIdx.x * rows_per_cta + threadIdx.x / lpr;
  const int sub = threadIdx.x % lpr;
  if (r >= R || threadIdx.x >= rows_per_cta * lpr) return;
  const int32_t t = idx[bh * R + r];
  if (t < 0 || t >= cap) return;  // skipped: no traffic (negative) or outside the source rows
  dst[(bh * R + r) * lpr + sub] = src[(bh * cap + t) * lpr + sub];
}


int run_decode(const float* q, int64_t BH, int G, const int64_t* idx, int64_t k, const uint16_t* K_src,
               const uint16_t* V_src, int64_t cap, int64_t kv_row_stride, int64_t n_host, const uint16_t* K_recent,
               const uint16_t* V_recent,
               int64_t recent_cap, int64_t idx_lo, int64_t idx_hi, float* out_f32, uint16_t* out_bf16,
               float* out_packed, void* workspace, size_t workspace_bytes, cudaStream_t st) {
  FATHOM_REQUIRE(q && idx && K_src && V_src && workspace, FATHOM_ERR_NULL, "decode_attention: NULL pointer");
  FATHOM_REQUIRE(out_f32 || out_bf16 || out_packed, FATHOM_ERR_NULL, "decode_attention: no output");
  FATHOM_REQUIRE(BH >= 1 && BH <= 65535 && G >= 1 && k >= 1 && n_host >= 0 && n_host <= cap && idx_lo <= idx_hi,
                 FATHOM_ERR_SHAPE, "decode_attention: bad shape");
  const int64_t M = (int64_t)G * k;
  FATHOM_REQUIRE(M <= MAX_M, FATHOM_ERR_UNSUPPORTED, "decode_attention: G*k=%lld exceeds %d", (long long)M, MAX_M);
  FATHOM_REQUIRE(recent_cap == 0 || (K_recent && V_recent), FATHOM_ERR_NULL,
                 "decode_attention: recent buffers missing");
  FATHOM_REQUIRE(workspace_bytes >= decode_ws_bytes(BH, M) && (reinterpret_cast<uintptr_t>(workspace) & 255) == 0,
                 FATHOM_ERR_WORKSPACE, "decode_attention: workspace needs %zu bytes, 256-byte aligned",
                 decode_ws_bytes(BH, M));
  FATHOM_REQUIRE((reinterpret_cast<uintptr_t>(K_src) & 15) == 0 && (reinterpret_cast<uintptr_t>(V_src) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(q) & 15) == 0,
                 FATHOM_ERR_SHAPE, "decode_attention: q and the K/V sources must be 16-byte aligned");
  FATHOM_REQUIRE(cap < 0xFFFFFFFFLL && n_host + recent_cap < 0xFFFFFFFFLL, FATHOM_ERR_UNSUPPORTED,
                 "decode_attention: row indices must fit 32 bits");
  if (kv_row_stride == 0) kv_row_stride = D;
  FATHOM_REQUIRE(kv_row_stride >= D && kv_row_stride % 8 == 0, FATHOM_ERR_SHAPE,
                 "decode_attention: kv_row_stride must be >= 128 and a multiple of 8 elements");
  if (device_memory(K_src) && device_memory(V_src) &&
      (recent_cap == 0 || (device_memory(K_recent) && device_memory(V_recent)))) {
    // rows already in HBM: each pick's rows are read in place (one launch; the workspace is unused)
    FATHOM_REQUIRE(recent_cap == 0 || ((reinterpret_cast<uintptr_t>(K_recent) & 15) == 0 &&
                                       (reinterpret_cast<uintptr_t>(V_recent) & 15) == 0),
                   FATHOM_ERR_SHAPE, "decode_attention: the recent buffers must be 16-byte aligned");
    const PickRows pr{idx, nullptr, K_src, V_src, 0, cap, kv_row_stride, n_host, recent_cap, idx_lo, idx_hi,
                      K_recent, V_recent};
    return launch_attend<false>(q, BH, G, k, pr, out_f32, out_bf16, out_packed, st);
  }
  DecodeWs w = carve(workspace, BH, M);
  int log2ts = 10;
  while ((1 << log2ts) < 2 * M) ++log2ts;           // load factor <= 1/2
  FATHOM_REQUIRE((1 << log2ts) <= MAX_TS, FATHOM_ERR_UNSUPPORTED, "decode_attention: too many picks");
  const size_t smem = sizeof(uint32_t) * (((size_t)1 << log2ts) + (size_t)M);   // table + keys in bucket order
  cudaFuncSetAttribute(dedupe_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  int bshift = 0;   // NB buckets cover the readable rows [0, n_host + recent_cap)
  while (((n_host + recent_cap - 1) >> bshift) >= NB) ++bshift;
  // picks at or beyond the readable rows (n_host host rows + recent_cap device rows) are ignored
  dedupe_kernel<<<(unsigned)BH, DT, smem, st>>>(idx, M, idx_lo, idx_hi, n_host + recent_cap, log2ts, bshift, w.slot,
                                                w.uniq, w.ucount);
  dim3 ggrid((unsigned)cdiv(M, GROWS), (unsigned)BH);
  gather_kernel<<<ggrid, GT, 0, st>>>(w.ucount, w.uniq, M, reinterpret_cast<const uint4*>(K_src),
                                      reinterpret_cast<const uint4*>(V_src), cap, kv_row_stride / 8, n_host,
                                      reinterpret_cast<const uint4*>(K_recent),
                                      reinterpret_cast<const uint4*>(V_recent), recent_cap,
                                      reinterpret_cast<uint4*>(w.kstage), reinterpret_cast<uint4*>(w.vstage));
  const int r = check_launch("decode_attention (dedupe, gather)");
  if (r != FATHOM_OK) return r;
  const PickRows pr{nullptr, w.slot, w.kstage, w.vstage, M, 0, 0, 0, 0, 0, 0, nullptr, nullptr};
  return launch_attend<true>(q, BH, G, k, pr, out_f32, out_bf16, out_packed, st);
}

}  // namespace
}  // namespace fathom

using namespace fathom;

extern "C" size_t fathom_decode_workspace_bytes(int64_t BH, int G, int64_t k) {
  if (BH <= 0 || G <= 0 || k <= 0) return 0;
  return decode_ws_bytes(BH, (int64_t)G * k);
}

extern "C" int fathom_decode_attention(const float* q, int64_t BH, int G, const int64_t* idx, int64_t k,
                                       const uint16_t* K_src, const uint16_t* V_src, int64_t cap,
                                       int64_t kv_row_stride, int64_t n_host, const uint16_t* K_recent,
                                       const uint16_t* V_recent, int64_t recent_cap, float* out_f32,
                                       uint16_t* out_bf16, void* workspace, size_t workspace_bytes, void* stream) {
  return run_decode(q, BH, G, idx, k, K_src, V_src, cap, kv_row_stride, n_host, K_recent, V_recent, recent_cap, 0,
                    INT64_MAX,
                    out_f32, out_bf16, nullptr, workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int fathom_decode_attention_partial(const float* q, int64_t BH, int G, const int64_t* idx, int64_t k,
                                               const uint16_t* K_src, const uint16_t* V_src, int64_t cap,
                                               int64_t kv_row_stride, int64_t idx_lo, int64_t idx_hi,
                                               float* out_packed, void* workspace, size_t workspace_bytes,
                                               void* stream) {
  FATHOM_REQUIRE(out_packed, FATHOM_ERR_NULL, "decode_attention_partial: NULL output");
  FATHOM_REQUIRE(idx_hi - idx_lo <= cap, FATHOM_ERR_SHAPE, "decode_attention_partial: owned range exceeds cap");
  return run_decode(q, BH, G, idx, k, K_src, V_src, cap, kv_row_stride, idx_hi - idx_lo, nullptr, nullptr, 0, idx_lo,
                    idx_hi, nullptr,
                    nullptr, out_packed, workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" size_t fathom_decode_partial_workspace_bytes(int64_t BH, int G, int64_t k) {
  if (BH <= 0 || G <= 0 || k <= 0) return 0;
  return decode_ws_bytes(BH, (int64_t)G * k);
}

extern "C" int fathom_attention_combine(const float* parts, int64_t P, int64_t rows, float* out_f32, uint16_t* out_bf16,
                                        void* stream) {
  FATHOM_REQUIRE(parts && (out_f32 || out_bf16), FATHOM_ERR_NULL, "attention_combine: NULL pointer");
  FATHOM_REQUIRE(P >= 1 && rows >= 1 && rows <= 0x7fffffffLL, FATHOM_ERR_SHAPE, "attention_combine: bad shape");
  combine_kernel<<<(unsigned)rows, D, 0, reinterpret_cast<cudaStream_t>(stream)>>>(parts, P, rows, out_f32, out_bf16);
  return check_launch("attention_combine");
}

extern "C" int fathom_gather_rows(const uint16_t* src, int64_t cap, const int32_t* idx, int64_t BH, int64_t R, int64_t Dm,
                                  uint16_t* dst, void* stream) {
  FATHOM_REQUIRE(src && idx && dst, FATHOM_ERR_NULL, "gather_rows: NULL pointer");
  FATHOM_REQUIRE(BH >= 1 && BH <= 65535 && R >= 1 && Dm >= 8 && (Dm * 2) % 16 == 0 && Dm * 2 / 16 <= 256,
                 FATHOM_ERR_SHAPE, "gather_rows: need D*2 a multiple of 16 (D <= 2048)");
  FATHOM_REQUIRE((reinterpret_cast<uintptr_t>(src) & 15) == 0 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0,
                 FATHOM_ERR_SHAPE, "gather_rows: src/dst must be 16-byte aligned");
  const int lpr = (int)(Dm * 2 / 16);
  const int rows_per_cta = 256 / lpr;
  dim3 grid((unsigned)cdiv(R, rows_per_cta), (unsigned)BH);
  gather_rows_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const uint4*>(src), cap, idx, R, lpr, reinterpret_cast<uint4*>(dst));
  return check_launch("gather_rows");
}
