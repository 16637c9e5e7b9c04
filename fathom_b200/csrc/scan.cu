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
// Memory parallelism: the channel list is cut into batches of about WB plane words.  The CTA copies
// the plane words of the next batch into shared memory while it computes the current batch from
// the other buffer, so a whole batch stays in flight.  Three copy modes, picked by the launch from
// the superblock order:
//   BULK  (sub a multiple of the CTA tile, e.g. the host run order): the whole tile of a (channel,
//         plane) is one contiguous run of tile_blocks * 8 bytes, and of a channel's scales one of
//         tile_blocks * 2 bytes; one warp issues one cp.async.bulk per run, completing on a
//         per-buffer mbarrier.  Over the host link these reach ~51 GB/s.
//   VEC16 (sub even and below the tile, the HBM order): the CTA copies 16-byte chunks (2 blocks)
//         with cp.async; fastest from HBM, but only ~36 GB/s from host memory.
//   LANE4 (anything else): one lane per half-word copies 4 bytes with cp.async (~47 GB/s host).
// Outside BULK, block scales are 4-byte copies of the aligned word holding each lane's scale.
// Block barriers order the copies against their readers and guard buffer reuse.  Every mbarrier
// wait is bounded: a wait that gives up counts in a device counter the host reads back
// (fathom_wait_timeouts), the CTA stops issuing, waits (bounded again) for its copies in flight and
// writes NaN scores.
#include "select_common.cuh"

#include <stdlib.h>
#include <string.h>

#include <mutex>

namespace fathom {
namespace {

constexpr int WARPS = 4;
constexpr int WB = 32;            // a batch holds the channels whose first word slot falls in [b*WB, (b+1)*WB)
constexpr int WBUF = WB + 3;      // ... so its words span at most WB + 3 slots
constexpr int CB = WB;            // and at most WB channels (each has >= 1 word)
template <int TPL>
constexpr int stage_u32() { return (WBUF + CB) * WARPS * TPL; }   // one CTA buffer: (WBUF+CB) rows x tile half-words
constexpr int MAXB = D * NPLANES / WB + 2;   // batch boundaries
enum CopyMode : int { COPY_LANE4 = 0, COPY_VEC16 = 1, COPY_BULK = 2 };
constexpr unsigned long long WAIT_LIMIT_NS = 2000000000ull;   // 2 s per mbarrier wait

__device__ unsigned long long g_wait_timeouts = 0;   // bounded waits that gave up (host-readable)

__device__ __forceinline__ void cp_async4(uint32_t* smem_dst, const void* gsrc) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(d), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async16(uint32_t* smem_dst, const void* gsrc) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(d), "l"(gsrc) : "memory");
}
// L2 eviction policies (createpolicy) and the accesses that take them: the phase kernel streams its
// plane words (read once: evict first) and keeps its scores, which the selection reads back (evict last).
__device__ __forceinline__ uint64_t l2_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;\n" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;\n" : "=l"(p));
  return p;
}
__device__ __forceinline__ void cp_async16_hint(uint32_t* smem_dst, const void* gsrc, uint64_t pol) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
  asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;\n" ::"r"(d), "l"(gsrc), "l"(pol)
               : "memory");
}
__device__ __forceinline__ void st_float4_hint(float* p, const float4& v, uint64_t pol) {
  asm volatile("st.global.L2::cache_hint.v4.f32 [%0], {%1, %2, %3, %4}, %5;\n" ::"l"(p), "f"(v.x), "f"(v.y),
               "f"(v.z), "f"(v.w), "l"(pol)
               : "memory");
}
__device__ __forceinline__ void mbar_init(uint64_t* mb) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(mb));
  asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(a) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* mb, uint32_t bytes) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(mb));
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(a), "r"(bytes) : "memory");
}
// global -> this CTA's shared memory, no multicast; 16-byte aligned addresses, size a multiple of 16
__device__ __forceinline__ void bulk_g2s(uint32_t* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* mb) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(mb));
  asm volatile("cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(d),
               "l"(gsrc), "r"(bytes), "r"(a)
               : "memory");
}
__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Waits until the phase with this parity completes; false after WAIT_LIMIT_NS.
__device__ __forceinline__ bool mbar_wait(uint64_t* mb, uint32_t parity) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(mb));
  uint32_t done = 0;
  const unsigned long long t0 = global_ns();
  while (true) {
    asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }\n"
                 : "=r"(done)
                 : "r"(a), "r"(parity)
                 : "memory");
    if (done) return true;
    if (global_ns() - t0 > WAIT_LIMIT_NS) return false;
  }
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

template <int G, int TPL, bool BULK>
__global__ void __launch_bounds__(WARPS * 32, (min_blocks<TPL, G>()))
    scan_kernel(const float* __restrict__ q, const int32_t* __restrict__ cls, const int32_t* __restrict__ clsn,
                int bmax, const uint32_t* __restrict__ planes32, const uint16_t* __restrict__ scales, int64_t n,
                int64_t nblk, int64_t nsb, int64_t sub, int64_t blk_begin, int64_t blk_end, int64_t grp_begin,
                int mode, float* __restrict__ out, uint32_t* __restrict__ gkey, int64_t ng) {
  // BULK instances run the bulk copies; the others run mode COPY_VEC16 or COPY_LANE4
  constexpr int LPW = 32 / TPL;          // lanes sharing a plane half-word
  constexpr int NHW = 32 / LPW;          // half-words per warp
  constexpr int BPW = NHW / 2;           // blocks per warp
  constexpr int TW = WARPS * NHW;        // half-words of the CTA tile (WARPS * BPW blocks)
  constexpr int CPP = TW / 4;            // 16-byte chunks per (channel, plane) of the tile
  constexpr int STAGE_U32 = (WBUF + CB) * TW;   // one buffer: WBUF word rows, then CB scale rows
  constexpr int TILE_BLOCKS = WARPS * BPW;
  constexpr uint32_t ROW_BYTES = TILE_BLOCKS * 8;     // one (channel, plane) run of the tile
  constexpr uint32_t SROW_BYTES = TILE_BLOCKS * 2;    // one channel's scales of the tile
  extern __shared__ __align__(16) uint32_t s_stage[];  // [2][STAGE_U32]
  __shared__ float s_q2[G][D];                 // 2 q of channel j
  __shared__ float s_qk[G][D];                 // q of channel j times 2^-t_j - 3
  __shared__ int s_ch[D], s_t[D], s_slot[D];
  __shared__ uint16_t s_pair[D * NPLANES];     // word position -> channel | plane << 8
  __shared__ int s_bstart[MAXB + 1], s_wstart[MAXB + 1];
  __shared__ int s_nb;
  __shared__ __align__(8) uint64_t s_mbar[2];   // BULK: one per stage buffer

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t bh = blockIdx.y;
  // one round of global loads: every thread's column of the four class lists plus the class counts;
  // then the flat channel list in class order (depth 1, 2, 3, 4) and the per-channel head tables.
  // Entry i of class c sits at flat index cstart[c] + i and word position cword[c] + c * i; its batch
  // is position / WB; s_pair maps every word position to its (channel, plane).
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
  if (tid == 0) {
    s_nb = 0;
    if constexpr (BULK) {
      mbar_init(&s_mbar[0]);
      mbar_init(&s_mbar[1]);
      asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");   // visible to the bulk copies
    }
  }
  __syncthreads();   // s_nb reset before any thread closes the last batch below
#pragma unroll
  for (int c = 0; c < NPLANES; ++c) {
    const int i = tid;
    if (i < cnt4[c]) {
      const int m = cstart[c] + i;
      const int t = c + 1;
      const int slot = cword[c] + t * i;
      const int ch = ch4[c] & (D - 1);                 // channel ids are 0..127
      s_ch[m] = ch;
      s_t[m] = t;
      for (int p = 0; p < t; ++p) s_pair[slot + p] = (uint16_t)(ch | (p << 8));
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
      if (b != prev) {
        s_bstart[b] = m;
        s_wstart[b] = slot;
      }
      if (m == total - 1) {  // the last channel closes the last batch
        s_nb = b + 1;
        s_bstart[b + 1] = m + 1;
        s_wstart[b + 1] = slot + t;
      }
      const float KC = __uint_as_float(0x3F800000u - ((uint32_t)t << 23)) - 3.0f;   // 2^-t - 3
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float qv = q[(bh * G + g) * D + ch];
        s_q2[g][ch] = 2.0f * qv;
        s_qk[g][ch] = qv * KC;
      }
    }
  }
  __syncthreads();

  const int64_t grp = grp_begin + (int64_t)blockIdx.x * WARPS + warp;
  const int64_t wblk0 = grp * BPW;
  const int64_t tile_blk0 = (grp_begin + (int64_t)blockIdx.x * WARPS) * BPW;
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
  const int col = warp * NHW + hw;           // this lane's column in the CTA stage rows
  const int64_t store_blocks = nsb * sub;    // blocks the store holds (pads included)
  const int nbatch = s_nb;                   // uniform over the CTA (barriers below)
  // this thread's 16-byte chunk of the tile: blocks tile_blk0 + 2 * chunk and the next one, which
  // share a superblock because sub is even whenever the 16-byte path is taken
  constexpr int PSTEP = WARPS * 32 / CPP;
  const int chunk = tid % CPP, chunk_row = tid / CPP;
  const int64_t cblk = tile_blk0 + 2 * chunk;
  const bool chunk_ok = cblk < store_blocks;
  const int64_t csb = chunk_ok ? cblk / sub : 0;
  const uint32_t* chunk_src = planes32 + ((bh * nsb + csb) * D * NPLANES * sub + (cblk - csb * sub)) * 2;
  const int64_t pstride32 = sub * 2;         // 32-bit words between consecutive (channel, plane) rows
  // BULK: the tile lies inside one superblock (sub is a multiple of TILE_BLOCKS and tiles start on
  // multiples of it), so its runs start at these two addresses plus a channel / plane offset
  const int64_t tsb = tile_blk0 / sub;
  const uint32_t* tile_planes = planes32 + ((bh * nsb + tsb) * D * NPLANES * sub + (tile_blk0 - tsb * sub)) * 2;
  const uint16_t* tile_scales = scales + (bh * nsb + tsb) * D * sub + (tile_blk0 - tsb * sub);
  const int tblk = warp * BPW + (hw >> 1);   // this lane's block within the tile

  auto issue = [&](int b) {
    uint32_t* wbuf = s_stage + (b & 1) * STAGE_U32;
    uint32_t* sbuf = wbuf + WBUF * TW;
    if constexpr (BULK) {
      if (warp == 0) {
        const int w0 = s_wstart[b], w1 = s_wstart[b + 1], c0 = s_bstart[b], c1 = s_bstart[b + 1];
        uint64_t* mb = &s_mbar[b & 1];
        if (lane == 0) mbar_expect_tx(mb, (uint32_t)(w1 - w0) * ROW_BYTES + (uint32_t)(c1 - c0) * SROW_BYTES);
        __syncwarp();
        for (int pos = w0 + lane; pos < w1; pos += 32) {
          const int pc = s_pair[pos];
          bulk_g2s(wbuf + (pos - b * WB) * TW, tile_planes + ((pc & 0xFF) * NPLANES + (pc >> 8)) * pstride32, ROW_BYTES,
                   mb);
        }
        for (int i = c0 + lane; i < c1; i += 32) bulk_g2s(sbuf + (i - c0) * TW, tile_scales + s_ch[i] * sub, SROW_BYTES, mb);
      }
      return;
    }
    if (mode == COPY_VEC16) {
      // plane words: the CTA copies each (channel, plane) of its tile in 16-byte chunks (2 blocks);
      // thread tid always copies chunk tid % CPP, of every PSTEP-th word position of the batch
      if (chunk_ok) {
        const int w1 = s_wstart[b + 1];
        for (int pos = s_wstart[b] + chunk_row; pos < w1; pos += PSTEP) {
          const int pc = s_pair[pos];
          cp_async16(&wbuf[(pos - b * WB) * TW + 4 * chunk], chunk_src + ((pc & 0xFF) * NPLANES + (pc >> 8)) * pstride32);
        }
      }
    } else if (active && issuer) {
      for (int i = s_bstart[b]; i < s_bstart[b + 1]; ++i) {
        const int ch = s_ch[i], t = s_t[i], slot = s_slot[i];
        const uint32_t* gp = pbase + ch * chan_stride32;
        for (int p = 0; p < t; ++p) cp_async4(&wbuf[(slot + p) * TW + col], gp + p * plane_stride32);
      }
    }
    if (active && issuer) {  // block scales: the aligned 4-byte word holding this lane's scale
      for (int i = s_bstart[b]; i < s_bstart[b + 1]; ++i) {
        const int64_t e = sc_elem0 + (int64_t)s_ch[i] * sub;
        cp_async4(&sbuf[(i - s_bstart[b]) * TW + col], scales + (e & ~(int64_t)1));
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

  bool stalled = false;                    // this thread gave up on an mbarrier wait
  int issued = 0;                          // batches issued so far (uniform)
  if (nbatch > 0) {
    issue(0);
    issued = 1;
  }
  for (int b = 0; b < nbatch; ++b) {
    // every thread is done with the buffer issue(b + 1) refills; a stall anywhere stops the CTA
    if (__syncthreads_or(stalled)) break;
    if (b + 1 < nbatch) {
      issue(b + 1);
      issued = b + 2;
    }
    if constexpr (BULK) {
      if (!mbar_wait(&s_mbar[b & 1], (b >> 1) & 1)) {
        stalled = true;
        atomicAdd(&g_wait_timeouts, 1ull);
        continue;
      }
    } else {
      if (b + 1 < nbatch) cp_async_wait<1>();
      else cp_async_wait<0>();
      __syncthreads();                     // every thread's copies of batch b are visible to the CTA
    }
    const uint32_t* wbuf = s_stage + (b & 1) * STAGE_U32;
    const uint32_t* sbuf = wbuf + WBUF * TW;
    for (int i = s_bstart[b]; i < s_bstart[b + 1]; ++i) {
      const int ch = s_ch[i], t = s_t[i], slot = s_slot[i];
      float sc;
      if constexpr (BULK) {
        sc = __half2float(__ushort_as_half(reinterpret_cast<const uint16_t*>(sbuf + (i - s_bstart[b]) * TW)[tblk]));
      } else {
        const int64_t e = sc_elem0 + (int64_t)ch * sub;
        const uint32_t sw = sbuf[(i - s_bstart[b]) * TW + col];
        sc = __half2float(__ushort_as_half((uint16_t)(sw >> ((e & 1) * 16))));
      }
      sc = active ? sc : 0.0f;
      uint32_t w[4];
#pragma unroll
      for (int p = 0; p < 4; ++p) w[p] = (p < t && active) ? (wbuf[(slot + p) * TW + col] >> bitoff) : 0u;
      float W[G];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        W[g] = s_q2[g][ch] * sc;
        cst[g] = fmaf(sc, s_qk[g][ch], cst[g]);
      }
      switch (t) {
        case 1: tokens<G, TPL, 1>(acc, w, W); break;
        case 2: tokens<G, TPL, 2>(acc, w, W); break;
        case 3: tokens<G, TPL, 3>(acc, w, W); break;
        default: tokens<G, TPL, 4>(acc, w, W); break;
      }
    }
  }
  // the stage is reused for the epilogue below; after a stall, first wait (bounded) for the copies
  // still in flight: the last batch issued into each buffer
  if (__syncthreads_or(stalled)) {
    if constexpr (BULK)
      for (int b = issued - 2 < 0 ? 0 : issued - 2; b < issued; ++b) mbar_wait(&s_mbar[b & 1], (b >> 1) & 1);
    __syncthreads();
#pragma unroll
    for (int g = 0; g < G; ++g) cst[g] = __int_as_float(0x7fc00000);   // NaN scores flag the failed tiles
  }

  // Epilogue, one query head at a time: the warp's scores go through its slice of the stage, so
  // the global stores are fully coalesced (512 contiguous bytes per warp instruction).
  // Lane l owns warp tokens l*TPL .. l*TPL+TPL-1; float4 slot j of lane l's row is stored at
  // j ^ swz(l), which keeps both the row writes and the token-order reads free of bank conflicts.
  constexpr int R = TPL / 4;                       // float4 per lane row
  constexpr int ROWS_PER_128B = 8 / R;
  float* s_sc = reinterpret_cast<float*>(s_stage) + warp * 32 * TPL;   // 32 * TPL floats per warp
  const int64_t wtok0 = wblk0 * BLK;               // first token of the warp
  const int64_t tok_lo = (warp_live ? lo : 0) * BLK;
  const int64_t tok_hi = warp_live ? (hi_lim * BLK < n ? hi_lim * BLK : n) : 0;   // valid tokens: [tok_lo, tok_hi)
  auto swz = [](int row) { return (row / ROWS_PER_128B) & (R - 1); };
  const bool vec_ok = (n % 4 == 0) && ((reinterpret_cast<uintptr_t>(out) & 15) == 0);
  // group keys for the selection (gkey != NULL): the largest key of each GROUP-token group, from the
  // same floats the stores below write; a group spans GL lanes
  constexpr int GL = selectk::GROUP / TPL;
  const int64_t ltok0 = wtok0 + (int64_t)lane * TPL;   // this lane's first token
#pragma unroll
  for (int g = 0; g < G; ++g) {
    __syncwarp();
    uint32_t gm = 0;
#pragma unroll
    for (int j = 0; j < R; ++j) {
      const float4 v = make_float4(acc[g][4 * j] + cst[g], acc[g][4 * j + 1] + cst[g], acc[g][4 * j + 2] + cst[g],
                                   acc[g][4 * j + 3] + cst[g]);
      reinterpret_cast<float4*>(s_sc)[lane * R + (j ^ swz(lane))] = v;
      if (gkey) {
        const float e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int64_t t = ltok0 + 4 * j + u;
          if (t >= tok_lo && t < tok_hi) gm = max(gm, f2key(e[u]));
        }
      }
    }
    if (gkey) {
#pragma unroll
      for (int o = 1; o < GL; o <<= 1) gm = max(gm, __shfl_xor_sync(0xffffffffu, gm, o));
      const int64_t grp = ltok0 / selectk::GROUP;
      if (lane % GL == 0 && ltok0 >= tok_lo && ltok0 < tok_hi) gkey[(bh * G + g) * ng + grp] = gm;
    }
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
                float* out, uint32_t* gkey, cudaStream_t st) {
  constexpr int BPW = TPL / 2;
  constexpr int TILE_BLOCKS = WARPS * BPW;
  const int64_t g0 = b0 / TILE_BLOCKS * WARPS, g1 = cdiv(b1, BPW);   // tiles start on multiples of TILE_BLOCKS
  const int64_t grid_x = cdiv(g1 - g0, WARPS);
  FATHOM_REQUIRE(grid_x <= 0x7fffffffLL && BH <= 65535, FATHOM_ERR_SHAPE, "scan: grid too large");
  const size_t smem = (size_t)2 * stage_u32<TPL>() * sizeof(uint32_t);
  // BULK needs each tile inside one superblock and 16-byte aligned runs; VEC16 needs every 2-block
  // pair contiguous and 16-byte aligned
  const bool a16 = (reinterpret_cast<uintptr_t>(planes32) & 15) == 0;
  const bool bulk_ok = a16 && (reinterpret_cast<uintptr_t>(scales) & 15) == 0 && sub % TILE_BLOCKS == 0;
  const bool vec16_ok = a16 && sub % 2 == 0;
  int mode = bulk_ok ? COPY_BULK : (vec16_ok && sub < TILE_BLOCKS) ? COPY_VEC16 : COPY_LANE4;
  if (const char* env = getenv("FATHOM_SCAN_COPY")) {   // tuning override: bulk, 16 or 4 (when the layout allows)
    if (!strcmp(env, "4")) mode = COPY_LANE4;
    else if (!strcmp(env, "16") && vec16_ok) mode = COPY_VEC16;
    else if (!strcmp(env, "bulk") && bulk_ok) mode = COPY_BULK;
  }
  auto kernel = mode == COPY_BULK ? scan_kernel<G, TPL, true> : scan_kernel<G, TPL, false>;
  cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  dim3 grid((unsigned)grid_x, (unsigned)BH);
  kernel<<<grid, WARPS * 32, smem, st>>>(q, cls, clsn, bmax, planes32, scales, n, nblk, nsb, sub, b0, b1, g0, mode, out,
                                         gkey, selectk::n_groups(n));
  return check_launch("scan");
}

}  // namespace
}  // namespace fathom

#include "scan_phase.cuh"

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

// Resident CTAs of a kernel on the current device, cached per (device, kernel).
template <typename K>
int resident_ctas(K kernel, int threads, size_t smem) {
  struct Entry {
    const void* fn;
    int dev;
    int ctas;
  };
  static Entry cache[256];
  static int used = 0;
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) dev = 0;
  const void* fn = reinterpret_cast<const void*>(kernel);
  for (int i = 0; i < used; ++i)
    if (cache[i].fn == fn && cache[i].dev == dev) return cache[i].ctas;
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem) != cudaSuccess || per_sm < 1) {
    cudaGetLastError();
    per_sm = 1;
  }
  const int ctas = per_sm * sm_count();
  if (used < 256) cache[used++] = Entry{fn, dev, ctas};
  return ctas;
}

template <int G, int P>
int launch_phase_scan(const float* q, int64_t BH, int64_t n, int64_t nblk, int64_t nsb, int64_t sub, const int32_t* cls,
                      const int32_t* clsn, int bmax, const uint32_t* planes32, const uint16_t* scales, int64_t b0,
                      int64_t b1, float* out, uint32_t* gkey, cudaStream_t st) {
  using Ge = ph::Geo<P>;
  const int64_t tile_lo = b0 / Ge::BPT, tile_hi = cdiv(b1, Ge::BPT);
  const int64_t ntiles = tile_hi - tile_lo;
  const size_t smem = (size_t)ph::WARPS * ph::NSTAGE * Ge::STAGE_U32 * sizeof(uint32_t);
  // With group keys the selection follows and reads candidate scores back: when the launch's scores
  // exceed half of L2 they are stored with an evict-last policy and the one-touch plane words loaded
  // with evict-first (config 3, 117 MB of scores per layer: step 6.44 -> 6.24 ms); smaller score sets
  // stay in L2 anyway and the plain instance is faster.
  const bool keep = gkey && (double)BH * G * n * sizeof(float) > 64.0 * 1024 * 1024;
  auto kernel = gkey ? (keep ? ph::phase_scan_kernel<G, P, true, true> : ph::phase_scan_kernel<G, P, true, false>)
                     : ph::phase_scan_kernel<G, P, false, false>;
  cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  // tiles per warp: one while the grid fills fewer than ~3 waves of resident CTAs, more (up to 8) to
  // spread each CTA's plan set-up (query and plan tables) over more tiles once it fills many waves
  // (config 3 per layer: 2 tiles per warp, 6% faster than 1; batched launches: 8)
  const int64_t ctas1 = BH * cdiv(ntiles, ph::WARPS);
  const int64_t resident = resident_ctas(kernel, ph::WARPS * 32, smem);
  int64_t tpw = ctas1 / (3 * resident);
  tpw = tpw < 1 ? 1 : (tpw > 8 ? 8 : tpw);
  if (const char* env = getenv("FATHOM_SCAN_TPW")) {    // tuning override
    const int v = atoi(env);
    if (v >= 1 && v <= 64) tpw = v;
  }
  const int64_t grid_x = cdiv(ntiles, ph::WARPS * tpw);
  FATHOM_REQUIRE(grid_x <= 0x7fffffffLL && BH <= 65535, FATHOM_ERR_SHAPE, "scan: grid too large");
  dim3 grid((unsigned)grid_x, (unsigned)BH);
  kernel<<<grid, ph::WARPS * 32, smem, st>>>(q, cls, clsn, bmax, planes32, scales, (int)n, (int)nsb, (int)sub, (int)b0,
                                             (int)b1, (int)tile_lo, (int)tile_hi, out, gkey,
                                             (int)selectk::n_groups(n));
  return check_launch("scan");
}

// The phase-interleaved kernel takes stores in device memory whose superblock order keeps a warp tile
// and its 8-block scale group inside one superblock row; mapped host memory keeps the bulk-copy
// kernel, whose long runs suit the host link.
bool phase_scan_applies(const uint64_t* planes_k, const uint16_t* scales_k, int64_t sub, int64_t nsb, int G,
                        int64_t n) {
  if (const char* env = getenv("FATHOM_SCAN_KERNEL"))    // tuning override: "classic" keeps scan_kernel
    if (!strcmp(env, "classic")) return false;
  if (sub % 8 != 0 || (reinterpret_cast<uintptr_t>(planes_k) & 15) || (reinterpret_cast<uintptr_t>(scales_k) & 15))
    return false;
  // the kernel's offsets within one row are 32-bit: the row's planes (1024 words per block) and its
  // G score rows must stay below 2^31 elements
  if (nsb * sub * 1024 >= (int64_t(1) << 31) || (int64_t)G * n >= (int64_t(1) << 31)) return false;
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, planes_k) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

int scan_dispatch(const float* q, int64_t BH, int G, int64_t n, int64_t sub, const int32_t* cls, const int32_t* clsn,
                  int bmax, const uint64_t* planes_k, const uint16_t* scales_k, int64_t blk_begin, int64_t blk_end,
                  float* scores, uint32_t* gkey, cudaStream_t st) {
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
  if (phase_scan_applies(planes_k, scales_k, sub, nsb, G, n)) {
    // two phases (16 tokens) per lane unless one phase per lane still fits the grid in one wave of
    // resident warps (16 per SM).  Config 1, one layer per launch (8 rows, 2048 warps at P = 2): 14.2
    // against 17.8 us per layer for P = 1.  G > 6 at P = 2 spills ~100 bytes per thread and still beats
    // P = 1 (config 3 batched: 53.0 against 59.6 us per layer)
    const int64_t range = blk_end - blk_begin;
    const bool small = BH * cdiv(range, 4) <= (int64_t)sm_count() * 16;
    int P = small ? 1 : 2;
    if (const char* env = getenv("FATHOM_SCAN_P")) {       // tuning override: 1 or 2
      const int v = atoi(env);
      if (v == 1 || v == 2) P = v;
    }
#define FATHOM_PH(GG, PP) \
  return launch_phase_scan<GG, PP>(q, BH, n, nblk, nsb, sub, cls, clsn, bmax, p32, scales_k, blk_begin, blk_end, scores, \
                                   gkey, st);
    switch (G) {
      case 1: if (P == 2) { FATHOM_PH(1, 2) } FATHOM_PH(1, 1)
      case 2: if (P == 2) { FATHOM_PH(2, 2) } FATHOM_PH(2, 1)
      case 3: if (P == 2) { FATHOM_PH(3, 2) } FATHOM_PH(3, 1)
      case 4: if (P == 2) { FATHOM_PH(4, 2) } FATHOM_PH(4, 1)
      case 5: if (P == 2) { FATHOM_PH(5, 2) } FATHOM_PH(5, 1)
      case 6: if (P == 2) { FATHOM_PH(6, 2) } FATHOM_PH(6, 1)
      case 7: if (P == 2) { FATHOM_PH(7, 2) } FATHOM_PH(7, 1)
      case 8: if (P == 2) { FATHOM_PH(8, 2) } FATHOM_PH(8, 1)
    }
#undef FATHOM_PH
  }
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
  return launch_scan<GG, TT>(q, BH, n, nblk, nsb, sub, cls, clsn, bmax, p32, scales_k, blk_begin, blk_end, scores, gkey, \
                             st);
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
  return scan_dispatch(q, BH, G, n, sub, cls, clsn, bmax, planes_k, scales_k, blk_begin, blk_end, scores, nullptr,
                       reinterpret_cast<cudaStream_t>(stream));
}

extern "C" size_t fathom_scan_select_workspace_bytes(int64_t BH, int G, int64_t n, int64_t kk) {
  (void)kk;
  return BH > 0 && G > 0 && n > 0 ? selectk::select_ws_bytes(BH * G, n) : 0;
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
  FATHOM_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 255) == 0, FATHOM_ERR_WORKSPACE,
                 "scan_select: workspace must be 256-byte aligned");
  // the group-key selection takes its keys from the scan's epilogue
  const bool gkeys = selectk::group_select_applies(rows, n, kk, mask_lo, mask_hi, workspace_bytes);
  FATHOM_REQUIRE(gkeys || workspace_bytes >= selectk::ws_bytes(rows), FATHOM_ERR_WORKSPACE,
                 "scan_select: workspace needs %zu bytes (got %zu)", selectk::select_ws_bytes(rows, n), workspace_bytes);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int64_t nblk = cdiv(n, BLK);
  int r = scan_dispatch(q, BH, G, n, sub, cls, clsn, bmax, planes_k, scales_k, 0, nblk, scores,
                        gkeys ? static_cast<uint32_t*>(workspace) : nullptr, st);
  if (r != FATHOM_OK) return r;
  if (scan_done_event) {
    const cudaError_t e = cudaEventRecord(reinterpret_cast<cudaEvent_t>(scan_done_event), st);
    if (e != cudaSuccess) return set_error(FATHOM_ERR_CUDA, "scan_select: event record: %s", cudaGetErrorString(e));
  }
  return selectk::launch_select(scores, rows, n, n, kk, mask_lo, mask_hi, index_offset, out_idx, out_stride,
                                out_scores, append_sink, append_local, workspace, workspace_bytes, gkeys, st);
}

extern "C" int fathom_wait_timeouts(unsigned long long* count, int reset) {
  unsigned long long v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_wait_timeouts, sizeof(v));
  if (e == cudaSuccess && reset) {
    const unsigned long long zero = 0;
    e = cudaMemcpyToSymbol(g_wait_timeouts, &zero, sizeof(zero));
  }
  if (e != cudaSuccess) return set_error(FATHOM_ERR_CUDA, "wait_timeouts: %s", cudaGetErrorString(e));
  if (count) *count = v;
  return FATHOM_OK;
}
