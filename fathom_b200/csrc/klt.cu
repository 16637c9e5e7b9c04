// KLT-rotated store ("planesK"): the bit-plane store over the keys rotated into a per-head
// Karhunen-Loeve basis, the basis rule for models without QK-norm (scripts/R_ruler.py:4, 63-64,
// 82-84; basis from scripts/R_agent.py:59-63 or scripts/sketch.py:44-52).
//
//   store:  Kr[bh, tok, e] = sum_d (K[bh, tok, d] - mu[bh, d]) * Vt[bh, d, e]   (fp32; pad tokens 0)
//           then the 4-bit block quantiser + plane packer of quant_common.cuh over Kr
//   query:  qr[bh, g, e]   = sum_d q[bh, g, d] * Vt[bh, d, e]
//           gains[bh, e]   = sum_g (qr[bh, g, e]^2 * lam[bh, e])    (g ascending, no contraction)
//
// The scan is the plain plane-prefix scan over (qr, plan(gains, budget)); it gives q.(K - mu),
// i.e. the scores up to the per-query constant q.mu, exactly as the reference's planesK scorer.
//
// Store build: one CTA (256 threads) per (block range, kv-head row) keeps the row's 128 x 128 basis
// in shared memory (64 KB, loaded once) and walks its 64-token blocks: stage (K - mu) of the block,
// a 64 x 128 x 128 fp32 product on the CUDA cores (each thread 4 tokens x 8 channels, d ascending
// with one FMA per term), then the shared quantiser epilogue on the rotated tile.  The product stays
// on the CUDA cores because the codes are floor(x / s) of fp32 values: a tensor-core product in a
// narrower type would move values across code boundaries.
#include "quant_common.cuh"

namespace fathom {
namespace {

constexpr int KT = 256;         // threads per CTA of the store build
constexpr int XS = QS;          // row stride of the staged (K - mu) tile: 16-byte aligned rows

struct KltSmem {
  float vt[D][D];                       // basis Vt[d][e]
  union {
    float x[BLK][XS];                   // (K - mu) of the block, token-major
    float tile[BLK][QS];                // rotated block, as quantise_tile reads it
  } u;
  float mu[D];
  float half_amax[2][D];
  __align__(16) uint8_t code[BLK][D];
};

template <typename T>
__global__ void __launch_bounds__(KT, 2) klt_quantise_pack_kernel(
    const T* __restrict__ K, int64_t n, int64_t k_stride_bh, const float* __restrict__ mu,
    const float* __restrict__ Vt, int64_t nblk, int64_t nsb, int64_t sub, int amax_f16, uint8_t* __restrict__ code,
    void* __restrict__ scales_blk, int scales_blk_f32, uint32_t* __restrict__ planes32,
    uint16_t* __restrict__ scales_k, float* __restrict__ rot_out) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  KltSmem& S = *reinterpret_cast<KltSmem*>(smem_raw);
  const int64_t bh = blockIdx.y;
  const int tid = threadIdx.x;
  {
    const float4* src = reinterpret_cast<const float4*>(Vt + bh * D * D);
    float4* dst = reinterpret_cast<float4*>(&S.vt[0][0]);
    for (int e = tid; e < D * D / 4; e += KT) dst[e] = __ldg(src + e);
    if (tid < D) S.mu[tid] = __ldg(mu + bh * D + tid);
  }
  const int64_t total_blk = planes32 ? nsb * sub : nblk;
  const int tx = tid & 15, ty = tid >> 4;      // channels 4tx..4tx+3 and 64+4tx..; tokens 4ty..4ty+3
  const T* Kb = K + bh * k_stride_bh;
  for (int64_t blk = blockIdx.x; blk < total_blk; blk += gridDim.x) {
    const bool real_blk = blk < nblk;
    const int64_t tok0 = blk * BLK;
    __syncthreads();                           // basis loaded / previous block's epilogue done
    for (int e = tid; e < BLK * D; e += KT) {
      const int r = e >> 7, c = e & (D - 1);
      const int64_t tok = tok0 + r;
      // pad tokens rotate to 0: the reference rotates the n real keys and pads the result
      S.u.x[r][c] = (real_blk && tok < n) ? __fsub_rn(load_elem<T>(Kb + tok * D + c), S.mu[c]) : 0.0f;
    }
    __syncthreads();

    float acc[4][8];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;
#pragma unroll 2
    for (int d0 = 0; d0 < D; d0 += 4) {
      float4 xv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) xv[i] = *reinterpret_cast<const float4*>(&S.u.x[ty * 4 + i][d0]);
#pragma unroll
      for (int dd = 0; dd < 4; ++dd) {
        const float4 va = *reinterpret_cast<const float4*>(&S.vt[d0 + dd][tx * 4]);
        const float4 vb = *reinterpret_cast<const float4*>(&S.vt[d0 + dd][64 + tx * 4]);
        const float v[8] = {va.x, va.y, va.z, va.w, vb.x, vb.y, vb.z, vb.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float xi = dd == 0 ? xv[i].x : dd == 1 ? xv[i].y : dd == 2 ? xv[i].z : xv[i].w;
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(xi, v[j], acc[i][j]);
        }
      }
    }
    __syncthreads();                           // every thread is done reading x: the tile aliases it
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = ty * 4 + i;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        S.u.tile[r][tx * 4 + j] = acc[i][j];
        S.u.tile[r][64 + tx * 4 + j] = acc[i][4 + j];
      }
      if (rot_out && real_blk && tok0 + r < n) {
        float4* o = reinterpret_cast<float4*>(rot_out + (bh * n + tok0 + r) * D);
        o[tx] = make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
        o[16 + tx] = make_float4(acc[i][4], acc[i][5], acc[i][6], acc[i][7]);
      }
    }
    __syncthreads();
    quantise_tile(S.u.tile, S.half_amax, S.code, bh, blk, n, nblk, nsb, sub, amax_f16, code, scales_blk,
                  scales_blk_f32, planes32, scales_k);
  }
}

// Query side, latency-bound (a few KB per row): CTA (row, 32 rotated channels) of QW warps; warp w
// sums input channels 16w .. 16w+15 for lane e (its 16 basis loads issued together), then warp 0
// adds the QW partial sums in warp order and forms the gains.
constexpr int QW = 8;
constexpr int QD = D / QW;      // input channels per warp

template <int G>
__global__ void __launch_bounds__(QW * 32) klt_query_kernel(const float* __restrict__ q, const float* __restrict__ Vt,
                                                            const float* __restrict__ lam, float* __restrict__ qr,
                                                            float* __restrict__ gains) {
  __shared__ float s_q[G][D];
  __shared__ float s_part[QW][G][32];
  const int64_t bh = blockIdx.x;
  const int e0 = blockIdx.y * 32;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  for (int i = tid; i < G * D; i += QW * 32) s_q[i / D][i % D] = __ldg(q + bh * G * D + i);
  const float* V = Vt + bh * D * D + (int64_t)(w * QD) * D + e0 + lane;
  float v[QD];
#pragma unroll
  for (int k = 0; k < QD; ++k) v[k] = __ldg(V + k * D);
  __syncthreads();
  float acc[G];
#pragma unroll
  for (int g = 0; g < G; ++g) acc[g] = 0.0f;
#pragma unroll
  for (int k = 0; k < QD; ++k)
#pragma unroll
    for (int g = 0; g < G; ++g) acc[g] = fmaf(s_q[g][w * QD + k], v[k], acc[g]);
#pragma unroll
  for (int g = 0; g < G; ++g) s_part[w][g][lane] = acc[g];
  __syncthreads();
  if (w != 0) return;
  const int e = e0 + lane;
  const float l = gains ? __ldg(lam + bh * D + e) : 0.0f;
  float gs = 0.0f;
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float s = s_part[0][g][lane];
#pragma unroll
    for (int ww = 1; ww < QW; ++ww) s = __fadd_rn(s, s_part[ww][g][lane]);
    qr[(bh * G + g) * D + e] = s;
    gs = __fadd_rn(gs, __fmul_rn(__fmul_rn(s, s), l));
  }
  if (gains) gains[bh * D + e] = gs;
}

int device_sms() {
  int dev = 0, v = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
  return v > 0 ? v : 148;
}

template <typename T>
int launch_klt_pack(const T* K, int64_t BH, int64_t n, int64_t k_stride_bh, const float* mu, const float* Vt,
                    int64_t nblk, int64_t nsb, int64_t sub, int amax_f16, uint8_t* code, void* scales_blk,
                    int scales_blk_f32, uint32_t* p32, uint16_t* scales_k, float* rot_out, cudaStream_t st) {
  const size_t smem = sizeof(KltSmem);
  cudaError_t e = cudaFuncSetAttribute(klt_quantise_pack_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return set_error(FATHOM_ERR_CUDA, "klt_quantise_pack: %s", cudaGetErrorString(e));
  const int64_t total_blk = p32 ? nsb * sub : nblk;
  // two resident CTAs per SM; each CTA loads its row's basis once and walks blocks with a stride
  const int64_t want = cdiv(2 * (int64_t)device_sms(), BH);
  const int64_t gx = total_blk < want ? total_blk : want;
  klt_quantise_pack_kernel<T><<<dim3((unsigned)gx, (unsigned)BH), KT, smem, st>>>(
      K, n, k_stride_bh, mu, Vt, nblk, nsb, sub, amax_f16, code, scales_blk, scales_blk_f32, p32, scales_k, rot_out);
  return check_launch("klt_quantise_pack");
}

}  // namespace
}  // namespace fathom

using namespace fathom;

extern "C" int fathom_klt_quantise_pack(const void* K, int k_dtype, int64_t BH, int64_t n, int64_t k_stride_bh,
                                        const float* mu, const float* Vt, int64_t sub, int amax_f16, uint8_t* code,
                                        void* scales_blk, int scales_blk_f32, uint64_t* planes_k, uint16_t* scales_k,
                                        float* rot_out, void* stream) {
  FATHOM_REQUIRE(K && mu && Vt, FATHOM_ERR_NULL, "klt_quantise_pack: K, mu and Vt must be given");
  FATHOM_REQUIRE(BH >= 1 && BH <= 65535 && n >= 1 && sub >= 1, FATHOM_ERR_SHAPE,
                 "klt_quantise_pack: need 1 <= BH <= 65535, n >= 1, sub >= 1 (BH=%lld n=%lld sub=%lld)",
                 (long long)BH, (long long)n, (long long)sub);
  FATHOM_REQUIRE(k_stride_bh >= n * D, FATHOM_ERR_SHAPE, "klt_quantise_pack: k_stride_bh < n*128");
  FATHOM_REQUIRE((planes_k == nullptr) == (scales_k == nullptr), FATHOM_ERR_NULL,
                 "klt_quantise_pack: planes_k and scales_k must both be given or both be NULL");
  FATHOM_REQUIRE((reinterpret_cast<uintptr_t>(Vt) & 15) == 0 && (rot_out == nullptr ||
                 (reinterpret_cast<uintptr_t>(rot_out) & 15) == 0), FATHOM_ERR_SHAPE,
                 "klt_quantise_pack: Vt and rot_out must be 16-byte aligned");
  const int64_t nblk = cdiv(n, BLK);
  const int64_t nsb = cdiv(nblk, sub);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  uint32_t* p32 = reinterpret_cast<uint32_t*>(planes_k);
  switch (k_dtype) {
    case FATHOM_DTYPE_F32:
      return launch_klt_pack(static_cast<const float*>(K), BH, n, k_stride_bh, mu, Vt, nblk, nsb, sub, amax_f16, code,
                             scales_blk, scales_blk_f32, p32, scales_k, rot_out, st);
    case FATHOM_DTYPE_BF16:
      return launch_klt_pack(static_cast<const __nv_bfloat16*>(K), BH, n, k_stride_bh, mu, Vt, nblk, nsb, sub,
                             amax_f16, code, scales_blk, scales_blk_f32, p32, scales_k, rot_out, st);
    case FATHOM_DTYPE_F16:
      return launch_klt_pack(static_cast<const __half*>(K), BH, n, k_stride_bh, mu, Vt, nblk, nsb, sub, amax_f16,
                             code, scales_blk, scales_blk_f32, p32, scales_k, rot_out, st);
    default:
      return set_error(FATHOM_ERR_UNSUPPORTED, "klt_quantise_pack: unknown k_dtype %d", k_dtype);
  }
}

extern "C" int fathom_klt_query(const float* q, int64_t BH, int G, const float* Vt, const float* lam, float* qr,
                                float* gains, void* stream) {
  FATHOM_REQUIRE(q && Vt && qr, FATHOM_ERR_NULL, "klt_query: q, Vt and qr must be given");
  FATHOM_REQUIRE(gains == nullptr || lam != nullptr, FATHOM_ERR_NULL, "klt_query: gains need lam");
  FATHOM_REQUIRE(BH >= 1 && BH <= 0x7fffffffLL, FATHOM_ERR_SHAPE, "klt_query: bad BH");
  FATHOM_REQUIRE(G >= 1 && G <= 8, FATHOM_ERR_UNSUPPORTED, "klt_query: G must be in 1..8 (got %d)", G);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
#define FATHOM_KLTQ(GG) \
  case GG:              \
    klt_query_kernel<GG><<<dim3((unsigned)BH, D / 32), QW * 32, 0, st>>>(q, Vt, lam, qr, gains); \
    break;
  switch (G) {
    FATHOM_KLTQ(1)
    FATHOM_KLTQ(2)
    FATHOM_KLTQ(3)
    FATHOM_KLTQ(4)
    FATHOM_KLTQ(5)
    FATHOM_KLTQ(6)
    FATHOM_KLTQ(7)
    FATHOM_KLTQ(8)
  }
#undef FATHOM_KLTQ
  return check_launch("klt_query");
}
