// Zero-copy K/V row gather and decode attention over the selected rows
// (scripts/B_e2e_offload_v2.py:73-83 gather_rows, :226-244 offload_attn tail;
//  HBM twin scripts/B_kernel_bench.py:26-31 gather_attn).
//
// decode attention from host-resident rows, three launches (device-resident rows: one launch of
// attend_direct_kernel or attend_direct_cluster_kernel, which read each pick's rows in place):
//   1 dedupe   one CTA per (batch, kv-head): the G*k picks go into a shared-memory hash table,
//              a block scan ranks the distinct indices; slot map (query head, pick) -> unique row,
//              the unique index list (in table order) and its length.
//   2 gather   many CTAs per (batch, kv-head): each unique K and V row is fetched ONCE from its source
//              (mapped host memory over the host link, or the device-resident recent buffer) into a
//              device staging area; 16 lanes x 16 B per 256-byte row, 4 rows in flight per lane.
//              Spreading the rows over every SM keeps enough requests in flight for the link.
//   3 attend   one CTA of 32 warps per (batch, query head): each warp takes 4 picks at a time from
//              the staging area (L2-resident), q.K^T / sqrt(128), an online softmax and the running
//              weighted sum of V; the 16 warp states are merged in shared memory.  fp32 math.
// A pick outside the caller's owned index range [idx_lo, idx_hi) is skipped (context shards);
// the partial form writes the unnormalised output with its (max, sum of exp).
#include "common.cuh"

#include <cooperative_groups.h>

namespace fathom {
namespace {

constexpr int DT = 1024;      // dedupe threads
constexpr int GT = 256;       // gather threads
constexpr int GROWS = 64;     // unique rows per gather CTA
constexpr int AW = 32;        // attend warps
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

__device__ __forceinline__ float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// The online softmax of one warp over its picks, DU at a time (shared by attend_kernel and the two
// in-place kernels, so all three sum in the same order and give the same bits).
struct WarpSoftmax {
  float m = -INFINITY, l = 0.0f, a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
  __device__ __forceinline__ void add(const float4& qv, const bool (&ok)[8], const uint2 (&kw)[8],
                                      const uint2 (&vw)[8], float scale) {
    float sc[8];
#pragma unroll
    for (int u = 0; u < 8; ++u)
      sc[u] = qv.x * bf16lo(kw[u].x) + qv.y * bf16hi(kw[u].x) + qv.z * bf16lo(kw[u].y) + qv.w * bf16hi(kw[u].y);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
      for (int u = 0; u < 8; ++u) sc[u] += __shfl_xor_sync(0xffffffffu, sc[u], o);
    }
    float mx = m;
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      sc[u] = ok[u] ? sc[u] * scale : -INFINITY;
      mx = fmaxf(mx, sc[u]);
    }
    if (mx == -INFINITY) return;  // nothing owned yet
    const float corr = m == -INFINITY ? 0.0f : expf(m - mx);
    l *= corr;
    a0 *= corr;
    a1 *= corr;
    a2 *= corr;
    a3 *= corr;
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const float pr = sc[u] == -INFINITY ? 0.0f : expf(sc[u] - mx);
      l += pr;
      a0 = fmaf(pr, bf16lo(vw[u].x), a0);
      a1 = fmaf(pr, bf16hi(vw[u].x), a1);
      a2 = fmaf(pr, bf16lo(vw[u].y), a2);
      a3 = fmaf(pr, bf16hi(vw[u].y), a3);
    }
    m = mx;
  }
};
constexpr int DU = 8;   // rows in flight per warp

// Merges the AW warp states of a CTA and writes the (batch, query head) output or partial.
__device__ __forceinline__ void attend_finish(const WarpSoftmax& ws, int64_t bhg, float* s_m, float* s_l,
                                              float (*s_acc)[D], float* __restrict__ out_f32,
                                              uint16_t* __restrict__ out_bf16, float* __restrict__ out_packed) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (lane == 0) {
    s_m[warp] = ws.m;
    s_l[warp] = ws.l;
  }
  s_acc[warp][lane * 4 + 0] = ws.a0;
  s_acc[warp][lane * 4 + 1] = ws.a1;
  s_acc[warp][lane * 4 + 2] = ws.a2;
  s_acc[warp][lane * 4 + 3] = ws.a3;
  __syncthreads();
  if (tid < D) {
    float Mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < AW; ++w) Mx = fmaxf(Mx, s_m[w]);
    float L = 0.0f, O = 0.0f;
#pragma unroll
    for (int w = 0; w < AW; ++w) {
      const float e = s_m[w] == -INFINITY ? 0.0f : expf(s_m[w] - Mx);
      L = fmaf(s_l[w], e, L);
      O = fmaf(s_acc[w][tid], e, O);
    }
    if (out_packed) {
      float* pk = out_packed + bhg * (D + 2);
      pk[tid] = O;
      if (tid == 0) {
        pk[D] = Mx;
        pk[D + 1] = L;
      }
    } else {
      const float o = O / L;
      if (out_f32) out_f32[bhg * D + tid] = o;
      if (out_bf16) out_bf16[bhg * D + tid] = __bfloat16_as_ushort(__float2bfloat16_rn(o));
    }
  }
}

// Host-resident rows, after dedupe + gather: one CTA of AW warps per (batch, query head); warp w owns
// picks [w*PW, w*PW + PW), PW = ceil(k / AW).  Per 32 picks the warp loads their staging slots with
// one coalesced load, then reads the staged K and V rows DU picks at a time (8 bytes per lane of each
// 256-byte row).  out_packed != NULL: partial form, [BH*G][130] = (sum_r e^(s_r - m) V_r, m, l).
__global__ void __launch_bounds__(AW * 32) attend_kernel(const float* __restrict__ q, int G, int64_t k, int64_t M,
                                                         const int32_t* __restrict__ slot,
                                                         const uint16_t* __restrict__ kstage,
                                                         const uint16_t* __restrict__ vstage,
                                                         float* __restrict__ out_f32, uint16_t* __restrict__ out_bf16,
                                                         float* __restrict__ out_packed) {
  __shared__ float s_m[AW], s_l[AW];
  __shared__ float s_acc[AW][D];
  const int64_t bhg = blockIdx.x;
  const int64_t bh = bhg / G, g = bhg % G;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float4 qv = *reinterpret_cast<const float4*>(q + bhg * D + lane * 4);
  const int32_t* sl = slot + bh * M + g * k;
  const uint16_t* kb = kstage + bh * M * D + lane * 4;
  const uint16_t* vb = vstage + bh * M * D + lane * 4;
  const float scale = rsqrtf((float)D);
  const int64_t PW = (k + AW - 1) / AW;
  const int64_t p0 = (int64_t)warp * PW;
  const int64_t p1 = p0 + PW < k ? p0 + PW : k;
  WarpSoftmax ws;
  for (int64_t c0 = p0; c0 < p1; c0 += 32) {   // uniform per warp
    const int32_t mine = c0 + lane < p1 ? sl[c0 + lane] : -1;
    const int nc = (int)(p1 - c0 < 32 ? p1 - c0 : 32);
    for (int s0 = 0; s0 < nc; s0 += DU) {
      bool ok[DU];
      uint2 kw[DU], vw[DU];
#pragma unroll
      for (int u = 0; u < DU; ++u) {
        int32_t r = __shfl_sync(0xffffffffu, mine, (s0 + u) & 31);
        if (s0 + u >= nc) r = -1;
        ok[u] = r >= 0;
        kw[u] = ok[u] ? *reinterpret_cast<const uint2*>(kb + (int64_t)r * D) : make_uint2(0, 0);
        vw[u] = ok[u] ? *reinterpret_cast<const uint2*>(vb + (int64_t)r * D) : make_uint2(0, 0);
      }
      ws.add(qv, ok, kw, vw, scale);
    }
  }
  attend_finish(ws, bhg, s_m, s_l, s_acc, out_f32, out_bf16, out_packed);
}

// Device-resident rows (HBM), many query heads: no dedupe and no staging.  The layout and summation
// order of attend_kernel, with each pick's K and V rows read in place by index (rows repeated across the
// query heads of a KV head are L2 hits).  A pick outside [idx_lo, idx_hi) or beyond the readable
// rows (n_host rows of the source, then recent_cap rows of the recent buffer) is skipped.
__global__ void __launch_bounds__(AW * 32) attend_direct_kernel(const float* __restrict__ q, int G, int64_t k,
                                                                const int64_t* __restrict__ idx, int64_t idx_lo,
                                                                int64_t idx_hi, const uint16_t* __restrict__ ksrc,
                                                                const uint16_t* __restrict__ vsrc, int64_t cap,
                                                                int64_t row_stride, int64_t n_host,
                                                                const uint16_t* __restrict__ krec,
                                                                const uint16_t* __restrict__ vrec, int64_t recent_cap,
                                                                float* __restrict__ out_f32,
                                                                uint16_t* __restrict__ out_bf16,
                                                                float* __restrict__ out_packed) {
  __shared__ float s_m[AW], s_l[AW];
  __shared__ float s_acc[AW][D];
  const int64_t bhg = blockIdx.x;
  const int64_t bh = bhg / G;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float4 qv = *reinterpret_cast<const float4*>(q + bhg * D + lane * 4);
  const int64_t* ib = idx + bhg * k;
  const float scale = rsqrtf((float)D);
  const int64_t PW = (k + AW - 1) / AW;
  const int64_t p0 = (int64_t)warp * PW;
  const int64_t p1 = p0 + PW < k ? p0 + PW : k;
  WarpSoftmax ws;
  for (int64_t c0 = p0; c0 < p1; c0 += 32) {   // uniform per warp
    // this lane's pick of the chunk: its row (< 2^32 - 1, checked by the launcher), or -1 when not owned
    int32_t rel = -1;
    if (c0 + lane < p1) {
      const int64_t t = ib[c0 + lane];
      if (t >= idx_lo && t < idx_hi && t - idx_lo < n_host + recent_cap) rel = (int32_t)(uint32_t)(t - idx_lo);
    }
    const int nc = (int)(p1 - c0 < 32 ? p1 - c0 : 32);
    for (int s0 = 0; s0 < nc; s0 += DU) {
      bool ok[DU];
      uint2 kw[DU], vw[DU];
#pragma unroll
      for (int u = 0; u < DU; ++u) {
        int32_t rr = __shfl_sync(0xffffffffu, rel, (s0 + u) & 31);
        if (s0 + u >= nc) rr = -1;
        ok[u] = rr != -1;
        kw[u] = make_uint2(0, 0);
        vw[u] = make_uint2(0, 0);
        if (ok[u]) {
          const int64_t r = (int64_t)(uint32_t)rr;
          const uint16_t* kr = r < n_host ? ksrc + (bh * cap + r) * row_stride : krec + (bh * recent_cap + r - n_host) * D;
          const uint16_t* vr = r < n_host ? vsrc + (bh * cap + r) * row_stride : vrec + (bh * recent_cap + r - n_host) * D;
          kw[u] = *reinterpret_cast<const uint2*>(kr + lane * 4);
          vw[u] = *reinterpret_cast<const uint2*>(vr + lane * 4);
        }
      }
      ws.add(qv, ok, kw, vw, scale);
    }
  }
  attend_finish(ws, bhg, s_m, s_l, s_acc, out_f32, out_bf16, out_packed);
}

// Device-resident rows (HBM), few query heads (fewer than SMs): the pick layout and summation order
// of attend_kernel, spread over a cluster of CS CTAs of AW / CS warps each: global warp w (CTA w / 8,
// warp w % 8) owns picks [w*PW, w*PW + PW), PW = ceil(k / AW), and reads each pick's K and V rows in
// place by index (rows repeated across the query heads of a KV head are L2 hits).  The cluster's
// first CTA merges the AW warp states through distributed shared memory in global warp order, so the
// result has the bits of attend_kernel.  A pick outside [idx_lo, idx_hi) or beyond the readable rows
// (n_host rows of the source, then recent_cap rows of the recent buffer) is skipped.
constexpr int CS = 4;            // CTAs per (batch, query head)
constexpr int CW = AW / CS;      // warps per CTA
__global__ void __launch_bounds__(CW * 32, 1) attend_direct_cluster_kernel(const float* __restrict__ q, int G, int64_t k,
                                                                const int64_t* __restrict__ idx, int64_t idx_lo,
                                                                int64_t idx_hi, const uint16_t* __restrict__ ksrc,
                                                                const uint16_t* __restrict__ vsrc, int64_t cap,
                                                                int64_t row_stride, int64_t n_host,
                                                                const uint16_t* __restrict__ krec,
                                                                const uint16_t* __restrict__ vrec, int64_t recent_cap,
                                                                float* __restrict__ out_f32,
                                                                uint16_t* __restrict__ out_bf16,
                                                                float* __restrict__ out_packed) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  __shared__ float s_m[CW], s_l[CW];
  __shared__ float s_acc[CW][D];
  const unsigned crank = cluster.block_rank();
  const int64_t bhg = blockIdx.x / CS;
  const int64_t bh = bhg / G;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gw = (int)crank * CW + warp;   // global warp of the (batch, query head)
  const float4 qv = *reinterpret_cast<const float4*>(q + bhg * D + lane * 4);
  const int64_t* ib = idx + bhg * k;
  const float scale = rsqrtf((float)D);
  const int64_t PW = (k + AW - 1) / AW;
  const int64_t p0 = (int64_t)gw * PW;
  const int64_t p1 = p0 + PW < k ? p0 + PW : k;
  WarpSoftmax ws;
  for (int64_t c0 = p0; c0 < p1; c0 += 32) {   // uniform per warp
    // this lane's pick of the chunk: its row (< 2^32 - 1, checked by the launcher), or -1 when not owned
    int32_t rel = -1;
    if (c0 + lane < p1) {
      const int64_t t = ib[c0 + lane];
      if (t >= idx_lo && t < idx_hi && t - idx_lo < n_host + recent_cap) rel = (int32_t)(uint32_t)(t - idx_lo);
    }
    const int nc = (int)(p1 - c0 < 32 ? p1 - c0 : 32);
    for (int s0 = 0; s0 < nc; s0 += DU) {
      bool ok[DU];
      uint2 kw[DU], vw[DU];
#pragma unroll
      for (int u = 0; u < DU; ++u) {
        int32_t rr = __shfl_sync(0xffffffffu, rel, (s0 + u) & 31);
        if (s0 + u >= nc) rr = -1;
        ok[u] = rr != -1;
        kw[u] = make_uint2(0, 0);
        vw[u] = make_uint2(0, 0);
        if (ok[u]) {
          const int64_t r = (int64_t)(uint32_t)rr;
          const uint16_t* kr = r < n_host ? ksrc + (bh * cap + r) * row_stride : krec + (bh * recent_cap + r - n_host) * D;
          const uint16_t* vr = r < n_host ? vsrc + (bh * cap + r) * row_stride : vrec + (bh * recent_cap + r - n_host) * D;
          kw[u] = *reinterpret_cast<const uint2*>(kr + lane * 4);
          vw[u] = *reinterpret_cast<const uint2*>(vr + lane * 4);
        }
      }
      ws.add(qv, ok, kw, vw, scale);
    }
  }
  if (lane == 0) {
    s_m[warp] = ws.m;
    s_l[warp] = ws.l;
  }
  s_acc[warp][lane * 4 + 0] = ws.a0;
  s_acc[warp][lane * 4 + 1] = ws.a1;
  s_acc[warp][lane * 4 + 2] = ws.a2;
  s_acc[warp][lane * 4 + 3] = ws.a3;
  cluster.sync();   // every CTA's warp states are written
  if (crank == 0 && tid < D) {
    float Mx = -INFINITY;
    for (int w = 0; w < AW; ++w) Mx = fmaxf(Mx, *cluster.map_shared_rank(&s_m[w % CW], w / CW));
    float L = 0.0f, O = 0.0f;
    for (int w = 0; w < AW; ++w) {
      const float mw = *cluster.map_shared_rank(&s_m[w % CW], w / CW);
      const float e = mw == -INFINITY ? 0.0f : expf(mw - Mx);
      L = fmaf(*cluster.map_shared_rank(&s_l[w % CW], w / CW), e, L);
      O = fmaf(*cluster.map_shared_rank(&s_acc[w % CW][tid], w / CW), e, O);
    }
    if (out_packed) {
      float* pk = out_packed + bhg * (D + 2);
      pk[tid] = O;
      if (tid == 0) {
        pk[D] = Mx;
        pk[D + 1] = L;
      }
    } else {
      const float o = O / L;
      if (out_f32) out_f32[bhg * D + tid] = o;
      if (out_bf16) out_bf16[bhg * D + tid] = __bfloat16_as_ushort(__float2bfloat16_rn(o));
    }
  }
  cluster.sync();   // the first CTA has read the others' shared memory
}

// out = sum_p o_p e^(m_p - M) / sum_p l_p e^(m_p - M), M = max_p m_p: log-sum-exp merge of the
// partial attention of P context shards.  One CTA of 128 threads per (batch, query head).
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
    const float w = m == -INFINITY ? 0.0f : expf(m - M);
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
    if (BH * G >= (int64_t)sm_count()) {   // enough CTAs of 32 warps to fill the GPU
      attend_direct_kernel<<<(unsigned)(BH * G), AW * 32, 0, st>>>(q, G, k, idx, idx_lo, idx_hi, K_src, V_src, cap,
                                                                   kv_row_stride, n_host, K_recent, V_recent,
                                                                   recent_cap, out_f32, out_bf16, out_packed);
      return check_launch("decode_attention");
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(BH * G * CS));
    cfg.blockDim = dim3(CW * 32);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = CS;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, attend_direct_cluster_kernel, q, G, k, idx, idx_lo, idx_hi, K_src, V_src,
                                             cap, kv_row_stride, n_host, K_recent, V_recent, recent_cap, out_f32,
                                             out_bf16, out_packed);
    if (e != cudaSuccess) return set_error(FATHOM_ERR_CUDA, "decode_attention: launch: %s", cudaGetErrorString(e));
    return check_launch("decode_attention");
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
  attend_kernel<<<(unsigned)(BH * G), AW * 32, 0, st>>>(q, G, k, M, w.slot, w.kstage, w.vstage, out_f32, out_bf16,
                                                         out_packed);
  return check_launch("decode_attention");
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
