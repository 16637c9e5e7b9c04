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
                                                           int64_t idx_lo, int64_t idx_hi,
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
      const int64_t t = (int64_t)(v >> POS_BITS);
      const bool owned = t >= idx_lo && t < idx_hi;
      sl[v & ((1ull << POS_BITS) - 1)] = owned ? (int32_t)(base + ex - (first ? 0u : 1u)) : -1;
      if (first) ul[base + ex] = owned ? t - idx_lo : -1;
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
      const int64_t t = r < U ? ul[r] : -1;
      if (t >= 0) {
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
      if (r < U && ul[r] >= 0) {
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
                                                    uint16_t* __restrict__ out_bf16, float* __restrict__ out_ml) {
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
    const int32_t sr = sl[r];
    float d = -INFINITY;
    if (sr >= 0) {  // slot -1: the pick is owned by another context shard
      const uint2 w = *reinterpret_cast<const uint2*>(kb + (int64_t)sr * D + lane * 4);
      d = qv[0] * bf16lo(w.x) + qv[1] * bf16hi(w.x) + qv[2] * bf16lo(w.y) + qv[3] * bf16hi(w.y);
      d = warp_sum(d) * scale;
    }
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
    const float e = s_p[r] == -INFINITY ? 0.0f : expf(s_p[r] - m);
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
    const int32_t sr = sl[r];
    if (sr >= 0) {
      const uint16_t v = vb[(int64_t)sr * D + dim];
      acc = fmaf(s_p[r], __uint_as_float((uint32_t)v << 16), acc);
    }
  }
  s_acc[par][dim] = acc;
  __syncthreads();
  if (tid < D) {
    const float un = s_acc[0][tid] + s_acc[1][tid];
    if (out_ml) {  // partial: unnormalised sum, with (max, sum of exp) beside it
      out_f32[bhg * D + tid] = un;
      if (tid == 0) {
        out_ml[bhg * 2] = m;
        out_ml[bhg * 2 + 1] = ssum;
      }
    } else {
      const float o = un / ssum;
      if (out_f32) out_f32[bhg * D + tid] = o;
      if (out_bf16) out_bf16[bhg * D + tid] = __bfloat16_as_ushort(__float2bfloat16_rn(o));
    }
  }
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

__global__ void pack_partial_kernel(const float* __restrict__ o, const float* __restrict__ ml, int64_t rows,
                                    float* __restrict__ packed) {
  const int64_t row = blockIdx.x;
  const int t = threadIdx.x;
  packed[row * (D + 2) + t] = o[row * D + t];
  if (t < 2) packed[row * (D + 2) + D + t] = ml[row * 2 + t];
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


int run_decode(const float* q, int64_t BH, int G, const int64_t* idx, int64_t k, const uint16_t* K_src,
               const uint16_t* V_src, int64_t cap, int64_t n_host, const uint16_t* K_recent, const uint16_t* V_recent,
               int64_t recent_cap, int64_t idx_lo, int64_t idx_hi, float* out_f32, uint16_t* out_bf16,
               float* out_ml, void* workspace, size_t workspace_bytes, cudaStream_t st) {
  FATHOM_REQUIRE(q && idx && K_src && V_src && workspace, FATHOM_ERR_NULL, "decode_attention: NULL pointer");
  FATHOM_REQUIRE(out_f32 || out_bf16, FATHOM_ERR_NULL, "decode_attention: no output");
  FATHOM_REQUIRE(BH >= 1 && G >= 1 && k >= 1 && n_host >= 0 && n_host <= cap && idx_lo <= idx_hi, FATHOM_ERR_SHAPE,
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
  DecodeWs w = carve(workspace, BH, M);
  int P = 1;
  while (P < M) P <<= 1;
  const size_t smem = (size_t)P * sizeof(uint64_t);
  cudaFuncSetAttribute(dedupe_gather_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  dedupe_gather_kernel<<<(unsigned)BH, DT, smem, st>>>(
      idx, M, idx_lo, idx_hi, reinterpret_cast<const uint4*>(K_src), reinterpret_cast<const uint4*>(V_src), cap,
      n_host, reinterpret_cast<const uint4*>(K_recent), reinterpret_cast<const uint4*>(V_recent), recent_cap, w.slot,
      w.uniq, reinterpret_cast<uint4*>(w.kstage), reinterpret_cast<uint4*>(w.vstage));
  const size_t smem2 = (size_t)k * sizeof(float);
  FATHOM_REQUIRE(smem2 <= 160 * 1024, FATHOM_ERR_UNSUPPORTED, "decode_attention: k too large");
  cudaFuncSetAttribute(attend_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem2);
  attend_kernel<<<(unsigned)(BH * G), AT, smem2, st>>>(q, G, k, M, w.slot, w.kstage, w.vstage, out_f32, out_bf16,
                                                       out_ml);
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
                                       const uint16_t* K_src, const uint16_t* V_src, int64_t cap, int64_t n_host,
                                       const uint16_t* K_recent, const uint16_t* V_recent, int64_t recent_cap,
                                       float* out_f32, uint16_t* out_bf16, void* workspace, size_t workspace_bytes,
                                       void* stream) {
  return run_decode(q, BH, G, idx, k, K_src, V_src, cap, n_host, K_recent, V_recent, recent_cap, 0, INT64_MAX,
                    out_f32, out_bf16, nullptr, workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int fathom_decode_attention_partial(const float* q, int64_t BH, int G, const int64_t* idx, int64_t k,
                                               const uint16_t* K_src, const uint16_t* V_src, int64_t cap,
                                               int64_t idx_lo, int64_t idx_hi, float* out_packed, void* workspace,
                                               size_t workspace_bytes, void* stream) {
  FATHOM_REQUIRE(out_packed, FATHOM_ERR_NULL, "decode_attention_partial: NULL output");
  FATHOM_REQUIRE(idx_hi - idx_lo <= cap, FATHOM_ERR_SHAPE, "decode_attention_partial: owned range exceeds cap");
  const size_t need = decode_ws_bytes(BH, (int64_t)G * k);
  const size_t extra = align256((size_t)BH * G * (D + 2) * sizeof(float));
  FATHOM_REQUIRE(workspace_bytes >= need + extra, FATHOM_ERR_WORKSPACE,
                 "decode_attention_partial: workspace needs %zu bytes", need + extra);
  float* o = reinterpret_cast<float*>(static_cast<char*>(workspace) + need);
  float* ml = o + (size_t)BH * G * D;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int r = run_decode(q, BH, G, idx, k, K_src, V_src, cap, idx_hi - idx_lo, nullptr, nullptr, 0, idx_lo, idx_hi, o,
                     nullptr, ml, workspace, need, st);
  if (r != FATHOM_OK) return r;
  pack_partial_kernel<<<(unsigned)(BH * G), D, 0, st>>>(o, ml, BH * G, out_packed);
  return check_launch("decode_attention_partial");
}

extern "C" size_t fathom_decode_partial_workspace_bytes(int64_t BH, int G, int64_t k) {
  if (BH <= 0 || G <= 0 || k <= 0) return 0;
  return decode_ws_bytes(BH, (int64_t)G * k) + align256((size_t)BH * G * (D + 2) * sizeof(float));
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
