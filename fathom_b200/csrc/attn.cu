// Zero-copy K/V row gather and decode attention over the selected rows
// (scripts/B_e2e_offload_v2.py:73-83 gather_rows, :226-244 offload_attn tail;
//  HBM twin scripts/B_kernel_bench.py:26-31 gather_attn).
//
// decode attention, two launches:
//   1 dedupe_gather  one CTA per (batch, kv-head): bitonic sort of the G*k selected indices,
//                    unique ranks by a block scan, slot map (query head, pick) -> unique row, and
//                    a gather of each unique K and V row ONCE from its source (mapped host memory
//                    or the device-resident recent buffer) into a device staging area; 16 B per
//                    lane, 16 lanes per 256-byte row, several rows in flight per thread.
//   2 attend         one CTA per (batch, query head): q.K^T / sqrt(128) over its k picks from the
//                    staging area, max-subtracted softmax and the weighted sum of V, fp32 math.
#include "common.cuh"

namespace fathom {
namespace {

constexpr int DT = 1024;    // dedupe_gather threads
constexpr int AT = 256;     // attend threads
constexpr int MAX_M = 16384;  // G*k per (batch, kv-head) handled by one CTA

size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

struct DecodeWs {
  int32_t* slot;       // [BH][M]
  int64_t* uniq;       // [BH][M] unique indices of each row, ascending
  uint16_t* kstage;    // [BH][M][128] bf16
  uint16_t* vstage;    // [BH][M][128] bf16
};

size_t decode_ws_bytes(int64_t BH, int64_t M) {
  return align256(BH * M * sizeof(int32_t)) + align256(BH * M * sizeof(int64_t)) +
         2 * align256(BH * M * D * sizeof(uint16_t));
}

DecodeWs carve(void* base, int64_t BH, int64_t M) {
  char* p = static_cast<char*>(base);
  DecodeWs w;
  w.slot = reinterpret_cast<int32_t*>(p);
  p += align256(BH * M * sizeof(int32_t));
  w.uniq = reinterpret_cast<int64_t*>(p);
  p += align256(BH * M * sizeof(int64_t));
  w.kstage = reinterpret_cast<uint16_t*>(p);
  p += align256(BH * M * D * sizeof(uint16_t));
  w.vstage = reinterpret_cast<uint16_t*>(p);
  return w;
}

__device__ void bitonic_asc(uint64_t* s, int P) {
  for (int k = 2; k <= P; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < P; i += blockDim.x) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const uint64_t a = s[i], b = s[ixj];
          const bool asc = (i & k) == 0;
          if (asc ? (a > b) : (a < b)) {
            s[i] = b;
            s[ixj] = a;
          }
        }
      }
      __syncthreads();
    }
  }
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

constexpr int POS_BITS = 24;  // position of a pick within G*k (< 2^24); index in the upper 40 bits

__global__ void __launch_bounds__(DT) dedupe_gather_kernel(const int64_t* __restrict__ idx, int64_t M,
                                                           const uint4* __restrict__ ksrc, const uint4* __restrict__ vsrc,
                                                           int64_t cap, int64_t n_host, const uint4* __restrict__ krec,
                                                           const uint4* __restrict__ vrec, int64_t recent_cap,
                                                           int32_t* __restrict__ slot, int64_t* __restrict__ uniq,
                                                           uint4* __restrict__ kstage,
                                                           uint4* __restrict__ vstage) {
  extern __shared__ uint64_t s_sort[];  // P entries
  __shared__ uint32_t s_warp[33];
  const int64_t bh = blockIdx.x;
  int P = 1;
  while (P < M) P <<= 1;
  const int64_t* ib = idx + bh * M;
  for (int i = threadIdx.x; i < P; i += blockDim.x)
    s_sort[i] = i < M ? ((uint64_t)ib[i] << POS_BITS) | (uint64_t)i : ~0ull;
  __syncthreads();
  bitonic_asc(s_sort, P);

  // slot map (pick position -> unique rank) and the unique index list, from the sorted picks
  int32_t* sl = slot + bh * M;
  int64_t* ul = uniq + bh * M;
  uint32_t base = 0;
  for (int64_t c0 = 0; c0 < M; c0 += blockDim.x) {
    const int64_t i = c0 + threadIdx.x;
    uint64_t v = 0;
    bool first = false;
    if (i < M) {
      v = s_sort[i];
      first = i == 0 || (v >> POS_BITS) != (s_sort[i - 1] >> POS_BITS);
    }
    uint32_t tot;
    const uint32_t ex = block_exclusive_scan(first ? 1u : 0u, s_warp, &tot);
    if (i < M) {
      sl[v & ((1ull << POS_BITS) - 1)] = (int32_t)(base + ex - (first ? 0u : 1u));
      if (first) ul[base + ex] = (int64_t)(v >> POS_BITS);
    }
    base += tot;
  }
  __syncthreads();  // makes the unique list (global) visible to the whole CTA
  const int64_t U = base;
  // gather: 16 lanes x 16 B per 256-byte row; K and V
  constexpr int LPR = D * 2 / 16;  // uint4 per row = 16
  const int sub = threadIdx.x % LPR;
  const int rows_per_iter = blockDim.x / LPR;
  uint4* ks = kstage + bh * M * LPR;
  uint4* vs = vstage + bh * M * LPR;
  constexpr int UNROLL = 4;
  for (int64_t r0 = threadIdx.x / LPR; r0 < U; r0 += (int64_t)rows_per_iter * UNROLL) {
    uint4 kv[UNROLL], vv[UNROLL];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      const int64_t r = r0 + (int64_t)u * rows_per_iter;
      if (r < U) {
        const int64_t t = ul[r];
        const uint4* kp;
        const uint4* vp;
        if (t < n_host) {
          kp = ksrc + (bh * cap + t) * LPR;
          vp = vsrc + (bh * cap + t) * LPR;
        } else {
          kp = krec + (bh * recent_cap + (t - n_host)) * LPR;
          vp = vrec + (bh * recent_cap + (t - n_host)) * LPR;
        }
        kv[u] = kp[sub];
        vv[u] = vp[sub];
      }
    }
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      const int64_t r = r0 + (int64_t)u * rows_per_iter;
      if (r < U) {
        ks[r * LPR + sub] = kv[u];
        vs[r * LPR + sub] = vv[u];
      }
    }
  }
}

__device__ __forceinline__ float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

__global__ void __launch_bounds__(AT) attend_kernel(const float* __restrict__ q, int G, int64_t k, int64_t M,
                                                    const int32_t* __restrict__ slot, const uint16_t* __restrict__ kstage,
                                                    const uint16_t* __restrict__ vstage, float* __restrict__ out_f32,
                                                    uint16_t* __restrict__ out_bf16) {
  extern __shared__ float s_p[];  // k probabilities
  __shared__ float s_q[D];
  __shared__ float s_red[AT / 32];
  __shared__ float s_acc[2][D];
  const int64_t bhg = blockIdx.x;
  const int64_t bh = bhg / G, g = bhg % G;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid < D) s_q[tid] = q[bhg * D + tid];
  __syncthreads();
  const int32_t* sl = slot + bh * M + g * k;
  const uint16_t* kb = kstage + bh * M * D;
  const uint16_t* vb = vstage + bh * M * D;
  const float scale = rsqrtf((float)D);
  // scores: one warp per pick, 4 dims per lane
  float qv[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) qv[i] = s_q[lane * 4 + i];
  float mloc = -INFINITY;
  for (int64_t r = warp; r < k; r += AT / 32) {
    const uint2 w = *reinterpret_cast<const uint2*>(kb + (int64_t)sl[r] * D + lane * 4);
    float d = qv[0] * bf16lo(w.x) + qv[1] * bf16hi(w.x) + qv[2] * bf16lo(w.y) + qv[3] * bf16hi(w.y);
    d = warp_sum(d) * scale;
    if (lane == 0) s_p[r] = d;
    mloc = fmaxf(mloc, d);
  }
  if (lane == 0) s_red[warp] = mloc;
  __syncthreads();
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < AT / 32; ++i) m = fmaxf(m, s_red[i]);
  __syncthreads();
  float sloc = 0.0f;
  for (int64_t r = tid; r < k; r += AT) {
    const float e = expf(s_p[r] - m);
    s_p[r] = e;
    sloc += e;
  }
  sloc = warp_sum(sloc);
  if (lane == 0) s_red[warp] = sloc;
  __syncthreads();
  float ssum = 0.0f;
#pragma unroll
  for (int i = 0; i < AT / 32; ++i) ssum += s_red[i];
  // weighted V: thread -> (dimension, parity of the pick)
  const int dim = tid & (D - 1), par = tid >> 7;
  float acc = 0.0f;
  for (int64_t r = par; r < k; r += 2) {
    const uint16_t v = vb[(int64_t)sl[r] * D + dim];
    acc = fmaf(s_p[r], __uint_as_float((uint32_t)v << 16), acc);
  }
  s_acc[par][dim] = acc;
  __syncthreads();
  if (tid < D) {
    const float o = (s_acc[0][tid] + s_acc[1][tid]) / ssum;
    if (out_f32) out_f32[bhg * D + tid] = o;
    if (out_bf16) out_bf16[bhg * D + tid] = __bfloat16_as_ushort(__float2bfloat16_rn(o));
  }
}

__global__ void gather_rows_kernel(const uint4* __restrict__ src, int64_t cap, const int32_t* __restrict__ idx,
                                   int64_t R, int lpr, uint4* __restrict__ dst) {
  const int64_t bh = blockIdx.y;
  const int rows_per_cta = blockDim.x / lpr;
  const int64_t r = (int64_t)blockIdx.x * rows_per_cta + threadIdx.x / lpr;
  const int sub = threadIdx.x % lpr;
  if (r >= R || threadIdx.x >= rows_per_cta * lpr) return;
  const int32_t t = idx[bh * R + r];
  if (t < 0) return;
  dst[(bh * R + r) * lpr + sub] = src[(bh * cap + t) * lpr + sub];
}

}  // namespace
}  // namespace fathom

using namespace fathom;

extern "C" size_t fathom_decode_workspace_bytes(int64_t BH, int G, int64_t k) {
  if (BH <= 0 || G <= 0 || k <= 0) return 0;
  return decode_ws_bytes(BH, (int64_t)G * k);
}

extern "C" int fathom_decode_attention(const float* q, int64_t BH, int G, const int64_t* idx, int64_t k,
                                       const uint16_t* K_src, const uint16_t* V_src, int64_t cap, int64_t n_host,
                                       const uint16_t* K_recent, const uint16_t* V_recent, int64_t recent_cap,
                                       float* out_f32, uint16_t* out_bf16, void* workspace, size_t workspace_bytes,
                                       void* stream) {
  FATHOM_REQUIRE(q && idx && K_src && V_src && workspace, FATHOM_ERR_NULL, "decode_attention: NULL pointer");
  FATHOM_REQUIRE(out_f32 || out_bf16, FATHOM_ERR_NULL, "decode_attention: no output");
  FATHOM_REQUIRE(BH >= 1 && G >= 1 && k >= 1 && n_host >= 0 && n_host <= cap, FATHOM_ERR_SHAPE,
                 "decode_attention: bad shape");
  const int64_t M = (int64_t)G * k;
  FATHOM_REQUIRE(M <= MAX_M, FATHOM_ERR_UNSUPPORTED, "decode_attention: G*k=%lld exceeds %d", (long long)M, MAX_M);
  FATHOM_REQUIRE(recent_cap == 0 || (K_recent && V_recent), FATHOM_ERR_NULL,
                 "decode_attention: recent buffers missing");
  FATHOM_REQUIRE(workspace_bytes >= decode_ws_bytes(BH, M) && (reinterpret_cast<uintptr_t>(workspace) & 255) == 0,
                 FATHOM_ERR_WORKSPACE, "decode_attention: workspace needs %zu bytes, 256-byte aligned",
                 decode_ws_bytes(BH, M));
  FATHOM_REQUIRE((reinterpret_cast<uintptr_t>(K_src) & 15) == 0 && (reinterpret_cast<uintptr_t>(V_src) & 15) == 0,
                 FATHOM_ERR_SHAPE, "decode_attention: K/V sources must be 16-byte aligned");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  DecodeWs w = carve(workspace, BH, M);
  int P = 1;
  while (P < M) P <<= 1;
  const size_t smem = (size_t)P * sizeof(uint64_t);
  cudaFuncSetAttribute(dedupe_gather_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  dedupe_gather_kernel<<<(unsigned)BH, DT, smem, st>>>(
      idx, M, reinterpret_cast<const uint4*>(K_src), reinterpret_cast<const uint4*>(V_src), cap, n_host,
      reinterpret_cast<const uint4*>(K_recent), reinterpret_cast<const uint4*>(V_recent), recent_cap, w.slot, w.uniq,
      reinterpret_cast<uint4*>(w.kstage), reinterpret_cast<uint4*>(w.vstage));
  const size_t smem2 = (size_t)k * sizeof(float);
  FATHOM_REQUIRE(smem2 <= 160 * 1024, FATHOM_ERR_UNSUPPORTED, "decode_attention: k too large");
  cudaFuncSetAttribute(attend_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem2);
  attend_kernel<<<(unsigned)(BH * G), AT, smem2, st>>>(q, G, k, M, w.slot, w.kstage, w.vstage, out_f32, out_bf16);
  return check_launch("decode_attention");
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
