// Plane-prefix key scan (PlaneStore.scan / scan_planes_cls_kernel, kernels/bitplane.py:275-338).
//
//   score[bh, g, tok] = sum_j q[bh, g, j] * s_j(blk) * (c_t(tok, j) + 1/2 - 2^(t-1)) / 2^(t-1)
//
// over the channels j of depth t = t_j >= 1, where c_t = code >> (4 - t) is read from the first
// t bit planes only.  Rewriting the dequantiser with f = 1 + c_t / 2^t (a float whose top t
// mantissa bits ARE the t plane bits, assembled with shifts and ORs and no conversion):
//
//   value_t = s * (2 f + 2^-t - 3)   =>   score = sum_j (2 q_j s_j) f_j  +  sum_j q_j s_j (2^-t - 3)
//
// so each (token, channel) costs t shift+or pairs and one FMA per query head.
//
// Work split: a warp owns a group of consecutive 64-token blocks of one (batch, kv-head) row;
// each lane owns TPL tokens of one 32-bit plane half-word: TPL = 32 (16 blocks per warp), 16 (8
// blocks) or 8 (4 blocks).  The launch picks the largest TPL that still gives every SM enough
// warps (small problems such as 128k tokens x 8 heads need the finer split; G > 4 never uses 32,
// to bound registers).  For a (channel, plane) the warp's words are 128 (64, 32) consecutive
// bytes in both the HBM order (sub = 16) and the host run order (sub = nblk).  Every lane keeps
// G x TPL fp32 accumulators in registers; the query tile and the channel list sit in shared memory.
//
// Memory parallelism: the channel list is cut into batches of about WB plane words.  One lane per
// half-word copies the words (and the 4-byte word holding the block scale) of the next batch into
// shared memory with cp.async while the warp computes the current batch from the other buffer, so
// a warp keeps a whole batch in flight instead of one channel.  Lanes sharing a half-word read the
// copy after cp.async.wait_group and a warp barrier; a second warp barrier guards buffer reuse.
#include "select_common.cuh"

#include <stdlib.h>

namespace fathom {
namespace {

constexpr int WARPS = 4;
constexpr int WB = 32;            // a batch holds the channels whose first word slot falls in [b*WB, (b+1)*WB)
constexpr int WBUF = WB + 3;      // ... so its words span at most WB + 3 slots
constexpr int CB = WB;            // and at most WB channels (each has >= 1 word)
template <int TPL>
constexpr int stage_u32() { return (WBUF + CB) * (32 * TPL / 32); }  // one buffer of one warp: (WBUF+CB) x half-words
constexpr int MAXB = D * NPLANES / WB + 2;   // batch boundaries

__device__ __forceinline__ void cp_async4(uint32_t* smem_dst, const void* gsrc) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(d), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

template <int G, int TPL, int C>
__device__ __forceinline__ void tokens(float (&acc)[G][TPL], const uint32_t (&w)[4], const float (&W)[G]) {
#pragma unroll
  for (int k = 0; k < TPL; ++k) {
    uint32_t bits = 0x3F800000u;
#pragma unroll
    for (int p = 0; p < C; ++p) {
      const int sh = 22 - p - k;
      const uint32_t m = sh >= 0 ? (w[p] << sh) : (w[p] >> (-sh));
      bits |= m & (1u << (22 - p));
    }
    const float f = __uint_as_float(bits);
#pragma unroll
    for (int g = 0; g < G; ++g) acc[g][k] = fmaf(W[g], f, acc[g][k]);
  }
}

template <int TPL, int G>
constexpr int min_blocks() { return TPL == 32 ? 2 : TPL == 16 ? (G > 4 ? 2 : 3) : (G > 4 ? 3 : 5); }

template <int G, int TPL>
__global__ void __launch_bounds__(WARPS * 32, (min_blocks<TPL, G>()))
    scan_kernel(const float* __restrict__ q, const int32_t* __restrict__ cls, const int32_t* __restrict__ clsn,
                int bmax, const uint32_t* __restrict__ planes32, const uint16_t* __restrict__ scales, int64_t n,
                int64_t nblk, int64_t nsb, int64_t sub, int64_t blk_begin, int64_t blk_end, int64_t grp_begin,
                float* __restrict__ out) {
  constexpr int LPW = 32 / TPL;          // lanes sharing a plane half-word
  constexpr int NHW = 32 / LPW;          // half-words per warp
  constexpr int BPW = NHW / 2;           // blocks per warp
  constexpr int STAGE_U32 = stage_u32<TPL>();
  extern __shared__ uint32_t s_stage[];  // [WARPS][2][STAGE_U32]
  __shared__ float s_q[G][D];
  __shared__ int s_ch[D], s_t[D], s_slot[D];
  __shared__ int s_bstart[MAXB + 1];
  __shared__ int s_nb;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t bh = blockIdx.y;
  for (int e = tid; e < G * D; e += blockDim.x) s_q[e / D][e % D] = q[bh * G * D + e];
  // one round of global loads: the query tile above, and here every thread's column of the four
  // class lists plus the class counts; then the flat channel list in class order (depth 1, 2, 3, 4).
  // Entry i of class c sits at flat index cstart[c] + i and word slot cword[c] + c * i; its batch
  // is slot / WB.
  int cnt4[NPLANES];
  int ch4[NPLANES];
#pragma unroll
  for (int c = 0; c < NPLANES; ++c) {
    int v = c < bmax ? clsn[bh * bmax + c] : 0;
    cnt4[c] = v < 0 ? 0 : (v > D ? D : v);             // memory safety for foreign plans
    ch4[c] = (c < bmax && tid < D) ? cls[(bh * bmax + c) * D + tid] : 0;
  }
  int cstart[NPLANES + 1], cword[NPLANES];
  {
    int st = 0, wd = 0;
#pragma unroll
    for (int c = 0; c < NPLANES; ++c) {
      cstart[c] = st;
      cword[c] = wd;
      st += cnt4[c];
      wd += (c + 1) * cnt4[c];
    }
    cstart[NPLANES] = st;
  }
  const int total = cstart[NPLANES];
  if (tid == 0) s_nb = 0;
  __syncthreads();   // s_nb reset before any thread closes the last batch below
#pragma unroll
  for (int c = 0; c < NPLANES; ++c) {
    const int i = tid;
    if (i < cnt4[c]) {
      const int m = cstart[c] + i;
      const int t = c + 1;
      const int slot = cword[c] + t * i;
      s_ch[m] = ch4[c] & (D - 1);                      // channel ids are 0..127
      s_t[m] = t;
      const int b = slot / WB;
      s_slot[m] = slot - b * WB;
      // the previous flat entry's batch (entry i-1 of this class, or the last of an earlier class)
      int prev = -1;
      if (m > 0) {
        int pc = c, pi = i - 1;
        while (pi < 0) {
          --pc;
          pi = cnt4[pc] - 1;
        }
        prev = (cword[pc] + (pc + 1) * pi) / WB;
      }
      if (b != prev) s_bstart[b] = m;
      if (m == total - 1) {  // the last channel closes the last batch
        s_nb = b + 1;
        s_bstart[b + 1] = m + 1;
      }
    }
  }
  __syncthreads();

  const int64_t grp = grp_begin + (int64_t)blockIdx.x * WARPS + warp;
  const int64_t wblk0 = grp * BPW;
  const int64_t lo = blk_begin > wblk0 ? blk_begin : wblk0;
  const int64_t hi_lim = blk_end < nblk ? blk_end : nblk;
  const bool warp_live = !(lo >= hi_lim || wblk0 + BPW <= blk_begin);  // some block of the warp in range

  const int hw = lane / LPW;                 // this lane's half-word within the warp
  const int64_t blk = wblk0 + (hw >> 1);
  const int64_t half = hw & 1;
  const int bitoff = (lane % LPW) * TPL;
  const bool issuer = (lane % LPW) == 0;
  const bool active = warp_live && blk >= blk_begin && blk < hi_lim;
  const int64_t bsafe = active ? blk : lo;
  const int64_t sb = bsafe / sub, s_in = bsafe - sb * sub;
  const uint32_t* pbase = planes32 + ((bh * nsb + sb) * D * NPLANES * sub + s_in) * 2 + half;
  const int64_t plane_stride32 = sub * 2;
  const int64_t chan_stride32 = NPLANES * sub * 2;
  const int64_t sc_elem0 = (bh * nsb + sb) * D * sub + s_in;   // scale element of channel 0

  uint32_t* stage = s_stage + warp * 2 * STAGE_U32;
  const int nbatch = warp_live ? s_nb : 0;

  auto issue = [&](int b) {
    uint32_t* wbuf = stage + (b & 1) * STAGE_U32;
    uint32_t* sbuf = wbuf + WBUF * NHW;
    if (active && issuer) {
      for (int i = s_bstart[b]; i < s_bstart[b + 1]; ++i) {
        const int ch = s_ch[i], t = s_t[i], slot = s_slot[i];
        const uint32_t* gp = pbase + ch * chan_stride32;
        for (int p = 0; p < t; ++p) cp_async4(&wbuf[(slot + p) * NHW + hw], gp + p * plane_stride32);
        const int64_t e = sc_elem0 + (int64_t)ch * sub;            // the aligned 4-byte word holding it
        cp_async4(&sbuf[(i - s_bstart[b]) * NHW + hw], scales + (e & ~(int64_t)1));
      }
    }
    cp_async_commit();
  };

  float acc[G][TPL];
  float cst[G];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    cst[g] = 0.0f;
#pragma unroll
    for (int k = 0; k < TPL; ++k) acc[g][k] = 0.0f;
  }

  if (nbatch > 0) issue(0);
  for (int b = 0; b < nbatch; ++b) {
    if (LPW > 1) __syncwarp();             // every lane is done with the buffer issue(b + 1) refills
    if (b + 1 < nbatch) {
      issue(b + 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    if (LPW > 1) __syncwarp();             // the issuers' copies are visible to the whole warp
    const uint32_t* wbuf = stage + (b & 1) * STAGE_U32;
    const uint32_t* sbuf = wbuf + WBUF * NHW;
    for (int i = s_bstart[b]; i < s_bstart[b + 1]; ++i) {
      const int ch = s_ch[i], t = s_t[i], slot = s_slot[i];
      const int64_t e = sc_elem0 + (int64_t)ch * sub;
      const uint32_t sw = sbuf[(i - s_bstart[b]) * NHW + hw];
      const float sc = active ? __half2float(__ushort_as_half((uint16_t)(sw >> ((e & 1) * 16)))) : 0.0f;
      uint32_t w[4];
#pragma unroll
      for (int p = 0; p < 4; ++p) w[p] = (p < t && active) ? (wbuf[(slot + p) * NHW + hw] >> bitoff) : 0u;
      float W[G];
      const float KC = __uint_as_float(0x3F800000u - ((uint32_t)t << 23)) - 3.0f;   // 2^-t - 3
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float qs = s_q[g][ch] * sc;
        W[g] = 2.0f * qs;
        cst[g] = fmaf(qs, KC, cst[g]);
      }
      switch (t) {
        case 1: tokens<G, TPL, 1>(acc, w, W); break;
        case 2: tokens<G, TPL, 2>(acc, w, W); break;
        case 3: tokens<G, TPL, 3>(acc, w, W); break;
        default: tokens<G, TPL, 4>(acc, w, W); break;
      }
    }
  }
  // Epilogue, one query head at a time: the warp's scores go through its (now idle) staging area, so
  // the global stores are fully coalesced (512 contiguous bytes per warp instruction).
  // Lane l owns warp tokens l*TPL .. l*TPL+TPL-1; float4 slot j of lane l's row is stored at
  // j ^ swz(l), which keeps both the row writes and the token-order reads free of bank conflicts.
  constexpr int R = TPL / 4;                       // float4 per lane row
  constexpr int ROWS_PER_128B = 8 / R;
  float* s_sc = reinterpret_cast<float*>(stage);   // 32 * TPL floats
  const int64_t wtok0 = wblk0 * BLK;               // first token of the warp
  const int64_t tok_lo = (warp_live ? lo : 0) * BLK;
  const int64_t tok_hi = warp_live ? (hi_lim * BLK < n ? hi_lim * BLK : n) : 0;   // valid tokens: [tok_lo, tok_hi)
  auto swz = [](int row) { return (row / ROWS_PER_128B) & (R - 1); };
  const bool vec_ok = (n % 4 == 0) && ((reinterpret_cast<uintptr_t>(out) & 15) == 0);
#pragma unroll
  for (int g = 0; g < G; ++g) {
    __syncwarp();
#pragma unroll
    for (int j = 0; j < R; ++j)
      reinterpret_cast<float4*>(s_sc)[lane * R + (j ^ swz(lane))] =
          make_float4(acc[g][4 * j] + cst[g], acc[g][4 * j + 1] + cst[g], acc[g][4 * j + 2] + cst[g],
                      acc[g][4 * j + 3] + cst[g]);
    __syncwarp();
    if (warp_live) {
      float* o = out + (bh * G + g) * n;
      // coalesced stores: iteration it covers warp tokens it*128 .. it*128+127, 4 per lane
#pragma unroll 1
      for (int it = 0; it < TPL / 4; ++it) {
        const int t = it * 128 + 4 * lane;
        const int row = t / TPL, j = (t % TPL) / 4;
        const float4 v = reinterpret_cast<const float4*>(s_sc)[row * R + (j ^ swz(row))];
        const int64_t tg = wtok0 + t;
        if (vec_ok && tg >= tok_lo && tg + 4 <= tok_hi) {
          *reinterpret_cast<float4*>(o + tg) = v;
        } else {
          const float e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int u = 0; u < 4; ++u)
            if (tg + u >= tok_lo && tg + u < tok_hi) o[tg + u] = e[u];
        }
      }
    }
  }
}

template <int G, int TPL>
int launch_scan(const float* q, int64_t BH, int64_t n, int64_t nblk, int64_t nsb, int64_t sub, const int32_t* cls,
                const int32_t* clsn, int bmax, const uint32_t* planes32, const uint16_t* scales, int64_t b0, int64_t b1,
                float* out, cudaStream_t st) {
  constexpr int BPW = TPL / 2;
  const int64_t g0 = b0 / BPW, g1 = cdiv(b1, BPW);
  const int64_t grid_x = cdiv(g1 - g0, WARPS);
  FATHOM_REQUIRE(grid_x <= 0x7fffffffLL && BH <= 65535, FATHOM_ERR_SHAPE, "scan: grid too large");
  const size_t smem = (size_t)WARPS * 2 * stage_u32<TPL>() * sizeof(uint32_t);
  cudaFuncSetAttribute(scan_kernel<G, TPL>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  dim3 grid((unsigned)grid_x, (unsigned)BH);
  scan_kernel<G, TPL><<<grid, WARPS * 32, smem, st>>>(q, cls, clsn, bmax, planes32, scales, n, nblk, nsb, sub, b0, b1,
                                                      g0, out);
  return check_launch("scan");
}

}  // namespace
}  // namespace fathom

using namespace fathom;

namespace fathom {
namespace {
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

int scan_dispatch(const float* q, int64_t BH, int G, int64_t n, int64_t sub, const int32_t* cls, const int32_t* clsn,
                  int bmax, const uint64_t* planes_k, const uint16_t* scales_k, int64_t blk_begin, int64_t blk_end,
                  float* scores, cudaStream_t st) {
  FATHOM_REQUIRE(q && cls && clsn && planes_k && scales_k && scores, FATHOM_ERR_NULL, "scan: NULL pointer");
  FATHOM_REQUIRE(BH >= 1 && BH <= 65535 && n >= 1 && sub >= 1, FATHOM_ERR_SHAPE, "scan: bad shape (BH=%lld n=%lld)",
                 (long long)BH, (long long)n);
  FATHOM_REQUIRE(G >= 1 && G <= 8, FATHOM_ERR_UNSUPPORTED, "scan: G must be in 1..8 (got %d)", G);
  FATHOM_REQUIRE(bmax >= 1 && bmax <= NPLANES, FATHOM_ERR_SHAPE, "scan: bmax must be in 1..4");
  FATHOM_REQUIRE((reinterpret_cast<uintptr_t>(planes_k) & 7) == 0 && (reinterpret_cast<uintptr_t>(scales_k) & 3) == 0,
                 FATHOM_ERR_SHAPE, "scan: planes must be 8-byte and scales 4-byte aligned");
  const int64_t nblk = cdiv(n, BLK), nsb = cdiv(nblk, sub);
  FATHOM_REQUIRE(blk_begin >= 0 && blk_begin <= blk_end && blk_end <= nblk, FATHOM_ERR_SHAPE,
                 "scan: block range [%lld, %lld) outside [0, %lld]", (long long)blk_begin, (long long)blk_end,
                 (long long)nblk);
  if (blk_begin == blk_end) return FATHOM_OK;
  const uint32_t* p32 = reinterpret_cast<const uint32_t*>(planes_k);
  // tokens per lane: 32 for G <= 4 (16 for G > 4, to bound registers); a split 4x finer only when the
  // coarse one would leave most SMs without a warp
  const int64_t range = blk_end - blk_begin;
  auto warps_for = [&](int tpl) { return BH * cdiv(range, tpl / 2); };
  int tpl = G <= 4 ? 32 : 16;
  if (warps_for(tpl) < (int64_t)sm_count()) tpl = 8;
  if (const char* env = getenv("FATHOM_SCAN_TPL")) {  // tuning override: 8, 16 or 32
    const int v = atoi(env);
    if (v == 8 || v == 16 || (v == 32 && G <= 4)) tpl = v;
  }
#define FATHOM_SCAN_LAUNCH(GG, TT) \
  return launch_scan<GG, TT>(q, BH, n, nblk, nsb, sub, cls, clsn, bmax, p32, scales_k, blk_begin, blk_end, scores, st);
#define FATHOM_SCAN_CASE4(GG)                    \
  case GG:                                       \
    if (tpl == 32) { FATHOM_SCAN_LAUNCH(GG, 32) } \
    if (tpl == 16) { FATHOM_SCAN_LAUNCH(GG, 16) } \
    FATHOM_SCAN_LAUNCH(GG, 8)
#define FATHOM_SCAN_CASE8(GG)                    \
  case GG:                                       \
    if (tpl == 16) { FATHOM_SCAN_LAUNCH(GG, 16) } \
    FATHOM_SCAN_LAUNCH(GG, 8)
  switch (G) {
    FATHOM_SCAN_CASE4(1)
    FATHOM_SCAN_CASE4(2)
    FATHOM_SCAN_CASE4(3)
    FATHOM_SCAN_CASE4(4)
    FATHOM_SCAN_CASE8(5)
    FATHOM_SCAN_CASE8(6)
    FATHOM_SCAN_CASE8(7)
    FATHOM_SCAN_CASE8(8)
  }
#undef FATHOM_SCAN_CASE4
#undef FATHOM_SCAN_CASE8
#undef FATHOM_SCAN_LAUNCH
  return set_error(FATHOM_ERR_UNSUPPORTED, "scan: G=%d", G);
}
}  // namespace
}  // namespace fathom

extern "C" int fathom_scan(const float* q, int64_t BH, int G, int64_t n, int64_t sub, const int32_t* cls,
                           const int32_t* clsn, int bmax, const uint64_t* planes_k, const uint16_t* scales_k,
                           int64_t blk_begin, int64_t blk_end, float* scores, void* stream) {
  return scan_dispatch(q, BH, G, n, sub, cls, clsn, bmax, planes_k, scales_k, blk_begin, blk_end, scores,
                       reinterpret_cast<cudaStream_t>(stream));
}

extern "C" size_t fathom_scan_select_workspace_bytes(int64_t BH, int G, int64_t n, int64_t kk) {
  (void)n;
  (void)kk;
  return BH > 0 && G > 0 ? selectk::ws_bytes(BH * G) : 0;
}

extern "C" int fathom_scan_select(const float* q, int64_t BH, int G, int64_t n, int64_t sub, const int32_t* cls,
                                  const int32_t* clsn, int bmax, const uint64_t* planes_k, const uint16_t* scales_k,
                                  int64_t kk, int64_t mask_lo, int64_t mask_hi, int64_t index_offset,
                                  int64_t append_sink, int64_t append_local, float* scores, int64_t* out_idx,
                                  int64_t out_stride, float* out_scores, void* workspace, size_t workspace_bytes,
                                  void* scan_done_event, void* stream) {
  const int64_t rows = BH * G;
  FATHOM_REQUIRE(out_idx && workspace, FATHOM_ERR_NULL, "scan_select: NULL pointer");
  FATHOM_REQUIRE(kk >= 1 && kk <= selectk::MAX_KK && kk <= n && n <= 0xffffffffLL, FATHOM_ERR_SHAPE,
                 "scan_select: kk=%lld outside 1..min(4096, n=%lld)", (long long)kk, (long long)n);
  FATHOM_REQUIRE(append_sink >= 0 && append_local >= 0 && out_stride >= kk + append_sink + append_local,
                 FATHOM_ERR_SHAPE, "scan_select: bad output stride");
  FATHOM_REQUIRE(workspace_bytes >= selectk::ws_bytes(rows) && (reinterpret_cast<uintptr_t>(workspace) & 255) == 0,
                 FATHOM_ERR_WORKSPACE, "scan_select: workspace needs %zu bytes, 256-byte aligned",
                 selectk::ws_bytes(rows));
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int64_t nblk = cdiv(n, BLK);
  int r = scan_dispatch(q, BH, G, n, sub, cls, clsn, bmax, planes_k, scales_k, 0, nblk, scores, st);
  if (r != FATHOM_OK) return r;
  if (scan_done_event) {
    const cudaError_t e = cudaEventRecord(reinterpret_cast<cudaEvent_t>(scan_done_event), st);
    if (e != cudaSuccess) return set_error(FATHOM_ERR_CUDA, "scan_select: event record: %s", cudaGetErrorString(e));
  }
  return selectk::launch_select(scores, rows, n, n, kk, mask_lo, mask_hi, index_offset, out_idx, out_stride,
                                out_scores, append_sink, append_local, workspace, workspace_bytes, st);
}
