// Chan4 comparator store and scan: the reference's baseline for SparQ / Double-Sparsity / Loki
// style channel subsets (Chan4Store, pack_chan4, channel_list, scan_chan4_kernel;
// kernels/bitplane.py:67-74, 128-132, 175-198, 342-355).
//
// Store: chan_k [BH][nsb][128][SUB][8] int32 -- for a (channel, block) 8 words, nibble k of word m
// holding the 4-bit code of token 8m+k of the block; scales_k [BH][nsb][128][SUB] fp16 as in the
// bit-plane store.  A scan reads, for every listed channel, the full 4-bit codes of each block:
// 32 + 2 bytes per (block, channel).
//
//   score[bh, g, tok] = sum_{i < nact} q[g, ch_i] * s_{ch_i}(blk) / 8 * (c(tok, ch_i) - 7.5)
//
// with c - 7.5 formed exactly as 16 f - 23.5 from f = 1 + c/16 (the nibble placed in the top mantissa
// bits of 1.0f, no integer conversion), then one FMA per query head: the product (c - 7.5) * (q s / 8)
// as the reference forms it, so an infinite block scale gives the reference's +-inf, not inf - inf.
//
// Work split: a warp owns 4 consecutive blocks of one (batch, kv-head) row; lane l reads word l % 8
// of block l / 8 (8 tokens), so the warp's 32 words of a channel are one 128-byte line when the 4
// blocks share a superblock.  CTA = 4 warps; the query tile and the channel list sit in shared
// memory; 4 channels' words are loaded before their math.
#include "common.cuh"

namespace fathom {
namespace {

constexpr int CW = 4;           // warps per CTA
constexpr int CBPW = 4;         // blocks per warp
constexpr int CU = 4;           // channels in flight

// one thread per output word
__global__ void pack_chan4_kernel(const uint8_t* __restrict__ code, int64_t n, int64_t nsb, int64_t sub,
                                  int64_t words_per_bh, int32_t* __restrict__ chan_k) {
  const int64_t bh = blockIdx.y;
  for (int64_t w = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; w < words_per_bh; w += (int64_t)gridDim.x * blockDim.x) {
    // w enumerates (token group of 8, channel) with the channel fastest: coalesced code reads
    const int64_t ch = w % D;
    const int64_t grp = w / D;                    // global 8-token group = ((sb*sub + s) * 8 + m)
    const int64_t m = grp % 8;
    const int64_t blk = grp / 8;
    const int64_t sb = blk / sub, s = blk % sub;
    uint32_t word = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int64_t tok = blk * BLK + m * 8 + k;
      const uint32_t c = tok < n ? code[(bh * n + tok) * D + ch] : 0u;
      word |= (c & 15u) << (4 * k);
    }
    chan_k[((((bh * nsb + sb) * D + ch) * sub + s) * 8) + m] = (int32_t)word;
  }
}

// one warp per (batch, kv-head): active channels ascending, then the inactive ones ascending
__global__ void channel_list_kernel(const uint8_t* __restrict__ active, int64_t BH, int32_t* __restrict__ act,
                                    int32_t* __restrict__ nact) {
  const int64_t bh = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (bh >= BH) return;
  const int lane = threadIdx.x & 31;
  uint32_t n_on = 0;
  for (int pass = 0; pass < 2; ++pass) {        // pass 0: active, pass 1: inactive
    uint32_t base = pass == 0 ? 0u : n_on;
    for (int c0 = 0; c0 < D; c0 += 32) {
      const int ch = c0 + lane;
      const bool on = active[bh * D + ch] != 0;
      const bool take = pass == 0 ? on : !on;
      const uint32_t m = __ballot_sync(0xffffffffu, take);
      if (take) act[bh * D + base + __popc(m & ((1u << lane) - 1))] = ch;
      base += __popc(m);
    }
    if (pass == 0) n_on = base;
  }
  if (lane == 0) nact[bh] = (int32_t)n_on;
}

template <int G>
__global__ void __launch_bounds__(CW * 32) scan_chan4_kernel(const float* __restrict__ q, const int32_t* __restrict__ act,
                                                             const int32_t* __restrict__ nact_bh,
                                                             const int32_t* __restrict__ chan_k,
                                                             const uint16_t* __restrict__ scales, int64_t n, int64_t nsb,
                                                             int64_t sub, int64_t blk_begin, int64_t blk_end,
                                                             float* __restrict__ out) {
  __shared__ float s_q[G][D];
  __shared__ int s_ch[D];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t bh = blockIdx.y;
  for (int e = tid; e < G * D; e += blockDim.x) s_q[e / D][e % D] = q[bh * G * D + e];
  int nact = nact_bh[bh];
  nact = nact < 0 ? 0 : (nact > D ? D : nact);   // memory safety for foreign lists
  for (int i = tid; i < nact; i += blockDim.x) s_ch[i] = act[bh * D + i] & (D - 1);
  __syncthreads();

  const int64_t blk = blk_begin + ((int64_t)blockIdx.x * CW + warp) * CBPW + lane / 8;
  const int m = lane % 8;
  const bool live = blk < blk_end;
  const int64_t bsafe = live ? blk : blk_begin;
  const int64_t sb = bsafe / sub, s = bsafe - sb * sub;
  const int32_t* wbase = chan_k + ((bh * nsb + sb) * D * sub + s) * 8 + m;   // + ch * sub * 8
  const uint16_t* sbase = scales + (bh * nsb + sb) * D * sub + s;             // + ch * sub

  float acc[G][8];
#pragma unroll
  for (int g = 0; g < G; ++g) {
#pragma unroll
    for (int k = 0; k < 8; ++k) acc[g][k] = 0.0f;
  }
  for (int i0 = 0; i0 < nact; i0 += CU) {
    uint32_t w[CU];
    float sc[CU];
#pragma unroll
    for (int u = 0; u < CU; ++u) {
      const int i = i0 + u;
      const int ch = i < nact ? s_ch[i] : 0;
      w[u] = (i < nact && live) ? (uint32_t)__ldg(wbase + (int64_t)ch * sub * 8) : 0u;
      sc[u] = (i < nact && live) ? __half2float(__ushort_as_half(__ldg(sbase + (int64_t)ch * sub))) : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < CU; ++u) {
      const int i = i0 + u;
      if (i >= nact) break;
      const int ch = s_ch[i];
      float W[G];
#pragma unroll
      for (int g = 0; g < G; ++g) W[g] = s_q[g][ch] * sc[u] * 0.125f;   // q * s / 8
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float f = __uint_as_float(0x3F800000u | (((w[u] >> (4 * k)) & 15u) << 19));   // 1 + c/16
        const float v = fmaf(16.0f, f, -23.5f);                                             // c - 7.5, exact
#pragma unroll
        for (int g = 0; g < G; ++g) acc[g][k] = fmaf(W[g], v, acc[g][k]);
      }
    }
  }
  if (!live) return;
  const int64_t tok0 = blk * BLK + m * 8;
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float* o = out + (bh * G + g) * n + tok0;
#pragma unroll
    for (int k = 0; k < 8; ++k)
      if (tok0 + k < n) o[k] = acc[g][k];
  }
}

}  // namespace
}  // namespace fathom

using namespace fathom;

extern "C" int fathom_pack_chan4(const uint8_t* code, int64_t BH, int64_t n, int64_t sub, int32_t* chan_k, void* stream) {
  FATHOM_REQUIRE(code && chan_k, FATHOM_ERR_NULL, "pack_chan4: NULL pointer");
  FATHOM_REQUIRE(BH >= 1 && BH <= 65535 && n >= 1 && sub >= 1, FATHOM_ERR_SHAPE, "pack_chan4: bad shape");
  const int64_t nsb = cdiv(cdiv(n, BLK), sub);
  const int64_t words = nsb * sub * 8 * D;    // per (batch, kv-head): every block of every superblock
  const int64_t grid_x = cdiv(words, 256) < 4096 ? cdiv(words, 256) : 4096;
  pack_chan4_kernel<<<dim3((unsigned)grid_x, (unsigned)BH), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      code, n, nsb, sub, words, chan_k);
  return check_launch("pack_chan4");
}

extern "C" int fathom_channel_list(const uint8_t* active, int64_t BH, int32_t* act, int32_t* nact, void* stream) {
  FATHOM_REQUIRE(active && act && nact, FATHOM_ERR_NULL, "channel_list: NULL pointer");
  FATHOM_REQUIRE(BH >= 1 && cdiv(BH, 4) <= 0x7fffffffLL, FATHOM_ERR_SHAPE, "channel_list: bad BH");
  channel_list_kernel<<<(unsigned)cdiv(BH, 4), 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(active, BH, act, nact);
  return check_launch("channel_list");
}

extern "C" int fathom_scan_chan4(const float* q, int64_t BH, int G, int64_t n, int64_t sub, const int32_t* act,
                                 const int32_t* nact, const int32_t* chan_k, const uint16_t* scales_k,
                                 int64_t blk_begin, int64_t blk_end, float* scores, void* stream) {
  FATHOM_REQUIRE(q && act && nact && chan_k && scales_k && scores, FATHOM_ERR_NULL, "scan_chan4: NULL pointer");
  FATHOM_REQUIRE(BH >= 1 && BH <= 65535 && n >= 1 && sub >= 1, FATHOM_ERR_SHAPE, "scan_chan4: bad shape");
  FATHOM_REQUIRE(G >= 1 && G <= 8, FATHOM_ERR_UNSUPPORTED, "scan_chan4: G must be in 1..8 (got %d)", G);
  const int64_t nblk = cdiv(n, BLK), nsb = cdiv(nblk, sub);
  FATHOM_REQUIRE(blk_begin >= 0 && blk_begin <= blk_end && blk_end <= nblk, FATHOM_ERR_SHAPE,
                 "scan_chan4: block range [%lld, %lld) outside [0, %lld]", (long long)blk_begin, (long long)blk_end,
                 (long long)nblk);
  if (blk_begin == blk_end) return FATHOM_OK;
  const int64_t grid_x = cdiv(blk_end - blk_begin, (int64_t)CW * CBPW);
  FATHOM_REQUIRE(grid_x <= 0x7fffffffLL, FATHOM_ERR_SHAPE, "scan_chan4: grid too large");
  dim3 grid((unsigned)grid_x, (unsigned)BH);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
#define FATHOM_CHAN4(GG)                                                                                            \
  case GG:                                                                                                          \
    scan_chan4_kernel<GG><<<grid, CW * 32, 0, st>>>(q, act, nact, chan_k, scales_k, n, nsb, sub, blk_begin, blk_end, \
                                                    scores);                                                        \
    break;
  switch (G) {
    FATHOM_CHAN4(1)
    FATHOM_CHAN4(2)
    FATHOM_CHAN4(3)
    FATHOM_CHAN4(4)
    FATHOM_CHAN4(5)
    FATHOM_CHAN4(6)
    FATHOM_CHAN4(7)
    FATHOM_CHAN4(8)
  }
#undef FATHOM_CHAN4
  return check_launch("scan_chan4");
}
