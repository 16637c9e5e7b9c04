// Plane-prefix scan for stores in device memory: the phase-interleaved kernel.
// Included by scan.cu, whose copy helpers and batch constants it shares.
//
// Same scores as scan_kernel, bit for bit: per (token, channel of depth t) the same f = 1 + c_t / 2^t,
// the same W_g = (2 q_g) * s and fma(W_g, f, acc) in the same channel order, and the same constant
// term cst_g = fma(s, q_g * (2^-t - 3), cst_g).  What changes is how f is formed and how the work is
// issued:
//
// Phases.  A 32-token plane half-word holds token k at bit k.  Phase r (0..3) is the 8 tokens
// k = 4m + r.  Rotating each of the t plane words of a channel so that plane p of token 4m + r lands
// on bit 4m + 6 - p, and merging the t rotated words with bit-select masks, gives one word z whose
// bits 4m+3..4m+6 hold token (4m + r)'s t-bit code (plane 0 highest; bits of planes >= t are masked
// off).  Two masks then give E (even m) and O (odd m) with one byte per token: 0x80 | code << 3.  A
// byte permute (prmt) drops byte j of E or O into bits 16..23 of 0x3F000000, which is exactly the
// float 1 + c_t / 2^t.  Per phase word that is 2t + 2 logic ops plus one prmt per token, against 2t
// ops per token when f is assembled token by token.
//
// Paired FMAs.  The accumulators of one query head for two tokens share a 64-bit register pair and
// take one fma.rn.f32x2 with {f_a, f_b} (each half written by its own byte permute) and the head's
// weight duplicated {W_g, W_g}, formed once per channel.  The halves are independent fma.rn
// operations, so the sums are those of scan_kernel.  (Measured against pairing two heads of one token,
// which copies f into both halves of a pair per token and gives an odd G a scalar head: 8.69 against
// 9.04 us per layer on config 1 batched, 53.0 against 55.2 on config 3.)
//
// Work split.  A lane owns P phases (P = 2: 16 tokens; P = 1: 8 tokens, for grids under one wave) of
// one half-word; a warp tile is 4P blocks of one (batch, kv-head) row.  Warps run independently: each
// streams its tiles'
// channel batches through NSTAGE shared-memory stages of its own with 16-byte cp.async copies (a lane
// per 16 bytes of the tile's (channel, plane) rows and 16-byte scale groups), one commit group per
// batch, so the main loop has no block-wide barrier.  The epilogue stages each head's scores in the
// warp's stage and stores 512 contiguous bytes per instruction; the group keys of the selection come
// from the same floats.
//
// Requirements (checked by the launcher): planes and scales 16-byte aligned, sub a multiple of 8 (a
// tile and its 8-block scale group lie inside one superblock row), device memory.
namespace fathom {
namespace {
namespace ph {

constexpr int WARPS = 4;
constexpr int NSTAGE = 3;

template <int P>
struct Geo {
  static constexpr int LPH = 4 / P;                // lanes per 32-token half-word
  static constexpr int HPW = 32 / LPH;             // half-words of a warp tile = 32-bit words of a stage row
  static constexpr int BPT = HPW / 2;              // 64-token blocks of a warp tile (4P)
  static constexpr int TPL = 8 * P;                // tokens per lane
  static constexpr int CPR = BPT * 8 / 16;         // 16-byte chunks of one (channel, plane) row of the tile
  static constexpr int SROW_U32 = 4;               // one channel's scale row: the aligned 8-block group, 16 bytes
  static constexpr int STAGE_U32 = WBUF * HPW + CB * SROW_U32;
  static constexpr int TILE_TOK = BPT * BLK;
  static constexpr int EPI_STRIDE = 36;            // staged scores: 32 tokens of a half-word + 4 pad words
};

__device__ __forceinline__ uint32_t rotl(uint32_t w, uint32_t a) { return __funnelshift_l(w, w, a); }
__device__ __forceinline__ uint32_t sel(uint32_t m, uint32_t a, uint32_t b) { return (a & m) | (b & ~m); }

// bits of plane p sit at positions = 6 - p (mod 4) of each nibble of z
__host__ __device__ constexpr uint32_t plane_mask(int p) { return 0x11111111u << ((6 - p) & 3); }
// of each byte of E / O, keep the bits of planes 0..t-1 (bit 6 - p)
__host__ __device__ constexpr uint32_t depth_mask(int t) {
  return (t == 1 ? 0x40u : t == 2 ? 0x60u : t == 3 ? 0x70u : 0x78u) * 0x01010101u;
}

// E and O of one phase r: amt[p + OFF] = 6 - p - r, the left rotation taking plane p of token 4m + r
// from bit 4m + r to bit 4m + 6 - p (mod 32; rotations keep bit positions mod 4, so the nibble of
// m = 7, which crosses bit 31, stays consistent with the plane masks)
template <int T, int OFF, int NA>
__device__ __forceinline__ void phase_words(const uint32_t (&w)[T], const uint32_t (&amt)[NA], uint32_t& E, uint32_t& O) {
  uint32_t z = rotl(w[T - 1], amt[T - 1 + OFF]);
#pragma unroll
  for (int p = T - 2; p >= 0; --p) z = sel(plane_mask(p), rotl(w[p], amt[p + OFF]), z);
  E = (z & depth_mask(T)) | 0x80808080u;
  O = (__funnelshift_r(z, z, 4) & depth_mask(T)) | 0x80808080u;   // a rotation: token 28 + r wraps past bit 31
}

// Byte j of E / O moved to bits 16..23 of zero: the float f * 2^-126 (exponent field 1 from the byte's
// 0x80, mantissa the code bits), exact.  Taking the other bytes from the zero register leaves the
// permute without a constant operand.  The weights carry 2^63 (F_SCALE) and the epilogue multiplies the
// sums by 2^63 (exact, power-of-two scaling while every product and sum stays normal), so the scores
// are those of f itself.
__device__ __forceinline__ uint32_t fbits(uint32_t X, int j) {
  return __byte_perm(X, 0u, 0x4044u | ((uint32_t)j << 8));
}
constexpr float F_SCALE = 9223372036854775808.0f;   // 2^63: weights are 2q * 2^63
constexpr float F_UNSCALE = 9223372036854775808.0f; // sums times 2^63 restore f's scale (2^-126 * 2^63 * 2^63)

// Accumulators of one lane, TPL tokens x G heads: r[g * TPL / 2 + pr] holds head g of the lane's token
// slots 2pr, 2pr + 1 (see token_of), so one fma.rn.f32x2 takes {f_a, f_b} of two tokens (two byte
// permutes straight into the register pair) and the head's weight duplicated, {W_g, W_g}.
template <int G, int P>
struct Acc {
  static constexpr int TPL = 8 * P;
  float2 r[G * TPL / 2];
  __device__ __forceinline__ void zero() {
#pragma unroll
    for (int i = 0; i < G * TPL / 2; ++i) r[i] = make_float2(0.f, 0.f);
  }
  __device__ __forceinline__ float get(int g, int k) const {
    const float2 v = r[g * (TPL / 2) + (k >> 1)];
    return (k & 1) ? v.y : v.x;
  }
};

// The lane's token of slot k within its half-word: pair k >> 1, half k & 1.
template <int P>
__device__ __forceinline__ int token_of(int k, int r0) {
  if constexpr (P == 1) return 8 * (k >> 1) + 4 * (k & 1) + r0;   // E / O byte j = k >> 1
  else return 4 * (k >> 1) + r0 + (k & 1);                         // phases r0, r0 + 1 of nibble m = k >> 1
}

// One channel of depth T for one lane: P phase words, then per token pair G paired FMAs
// {W_g, W_g} x {f_a, f_b}.
template <int T, int P, int G>
__device__ __forceinline__ void channel(Acc<G, P>& acc, const uint32_t (&w)[T], const uint32_t (&amt)[P + 3],
                                        const float2 (&Wd)[G]) {
  constexpr int TPL = 8 * P;
  uint32_t X[2][2];   // [phase][E, O]
  phase_words<T, 0>(w, amt, X[0][0], X[0][1]);
  if constexpr (P == 2) phase_words<T, 1>(w, amt, X[1][0], X[1][1]);
#pragma unroll
  for (int pr = 0; pr < TPL / 2; ++pr) {
    uint32_t xa, xb;
    int j;
    if constexpr (P == 1) {
      xa = X[0][0];
      xb = X[0][1];
      j = pr;
    } else {
      xa = X[0][pr & 1];
      xb = X[1][pr & 1];
      j = pr >> 1;
    }
    const float2 f2 = make_float2(__uint_as_float(fbits(xa, j)), __uint_as_float(fbits(xb, j)));
#pragma unroll
    for (int g = 0; g < G; ++g) acc.r[g * (TPL / 2) + pr] = __ffma2_rn(Wd[g], f2, acc.r[g * (TPL / 2) + pr]);
  }
}

template <int G, int P, bool GK, bool KEEP>
__global__ void __launch_bounds__(WARPS * 32, (P == 2 && G > 4 ? 3 : 4))
    phase_scan_kernel(const float* __restrict__ q, const int32_t* __restrict__ cls, const int32_t* __restrict__ clsn,
                      int bmax, const uint32_t* __restrict__ planes32, const uint16_t* __restrict__ scales, int n,
                      int nsb, int sub, int blk_begin, int blk_end, int tile_lo, int tile_hi, float* __restrict__ out,
                      uint32_t* __restrict__ gkey, int ng) {
  // Offsets within one (batch, kv-head) row are 32-bit (the launcher keeps a row's store under 2^31
  // words); the row's base pointers are formed once.
  using Ge = Geo<P>;
  constexpr int G2 = (G + 1) / 2;
  constexpr int TPL = Ge::TPL;
  extern __shared__ __align__(16) uint32_t s_stage[];   // [WARPS][NSTAGE][STAGE_U32]
  __shared__ float4 s_qt[D][G2];                        // flat entry i, g = 2k: {2q_g S, 2q_g+1 S, q_g KC_t, q_g+1 KC_t}
  __shared__ int s_ch[D], s_slot[D];
  __shared__ int s_roff[D * NPLANES];                  // word offset of each (channel, plane) row of a slot
  __shared__ int s_bstart[MAXB + 1], s_wstart[MAXB + 1];
  __shared__ int s_nb, s_cstart[NPLANES + 1];
  __shared__ float s_q[G][D];                           // the row's queries, staged beside the plan lists

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int bh = blockIdx.y;
  // ---- the row's channel list in class order, its copy batches and the per-entry head tables.  The
  // queries are loaded with the plan lists (thread = channel), not after them, so the set-up waits on
  // one round of global loads.
  static_assert(WARPS * 32 == D, "one thread per channel in the set-up");
  int cnt4[NPLANES], ch4[NPLANES];
  float qrow[G];
#pragma unroll
  for (int g = 0; g < G; ++g) qrow[g] = q[(bh * G + g) * D + tid];
#pragma unroll
  for (int c = 0; c < NPLANES; ++c) {
    const int v = c < bmax ? clsn[bh * bmax + c] : 0;
    cnt4[c] = v < 0 ? 0 : (v > D ? D : v);               // memory safety for foreign plans
    ch4[c] = (c < bmax && tid < D) ? cls[(bh * bmax + c) * D + tid] : 0;
  }
#pragma unroll
  for (int g = 0; g < G; ++g) s_q[g][tid] = qrow[g];
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
#pragma unroll
    for (int c = 0; c <= NPLANES; ++c) s_cstart[c] = cstart[c];
  }
  __syncthreads();
#pragma unroll
  for (int c = 0; c < NPLANES; ++c) {
    const int i = tid;
    if (i < cnt4[c]) {
      const int m = cstart[c] + i;
      const int t = c + 1;
      const int slot = cword[c] + t * i;
      const int ch = ch4[c] & (D - 1);
      s_ch[m] = ch;
      for (int p = 0; p < t; ++p) s_roff[slot + p] = (ch * NPLANES + p) * (sub * 2);
      const int b = slot / WB;
      s_slot[m] = slot - b * WB;
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
      if (m == total - 1) {
        s_nb = b + 1;
        s_bstart[b + 1] = m + 1;
        s_wstart[b + 1] = slot + t;
      }
      const float KC = __uint_as_float(0x3F800000u - ((uint32_t)t << 23)) - 3.0f;   // 2^-t - 3
      float qv[G];
#pragma unroll
      for (int g = 0; g < G; ++g) qv[g] = s_q[g][ch];
#pragma unroll
      for (int k = 0; k < G2; ++k) {
        const float a = 2.0f * qv[2 * k] * F_SCALE, b2 = 2 * k + 1 < G ? 2.0f * qv[2 * k + 1] * F_SCALE : 0.0f;
        s_qt[m][k] = make_float4(a, b2, qv[2 * k] * KC, 2 * k + 1 < G ? qv[2 * k + 1] * KC : 0.0f);
      }
    }
  }
  __syncthreads();
  const int nb = s_nb;

  // ---- this warp's tiles and lane geometry
  const int gw = blockIdx.x * WARPS + warp;
  const int wstride = gridDim.x * WARPS;
  const int ntw = tile_hi - tile_lo > gw ? (tile_hi - tile_lo - gw + wstride - 1) / wstride : 0;
  if (ntw == 0) return;                                   // no barrier follows: warps are independent from here
  const int hw = lane / Ge::LPH;                          // half-word of the tile
  const int r0 = (lane % Ge::LPH) * P;                    // first phase of the lane
  uint32_t amt[P + 3];                                    // rotations: phase r0 + d, plane p uses amt[p + d]
#pragma unroll
  for (int k = 0; k < P + 3; ++k) amt[k] = (uint32_t)(6 - k - r0);
  uint32_t* my_stage = s_stage + (size_t)warp * NSTAGE * Ge::STAGE_U32;
  const uint32_t* planes_row = planes32 + (int64_t)bh * nsb * (D * NPLANES * 2) * sub;
  const uint16_t* scales_row = scales + (int64_t)bh * nsb * D * sub;
  // items = (tile k of this warp, batch b) in order; 32-bit counters, advanced incrementally
  const int items = ntw * nb;

  auto tile_of = [&](int k) { return tile_lo + gw + k * wstride; };
  // copies of item (k, b) into stage stg: 16-byte chunks, lane e of every 32
  // the tile's plane and scale rows, formed once per tile (the items of a tile are issued in a row)
  int rows_k = -1;
  const uint32_t* rows = planes_row;
  const uint16_t* srow = scales_row;
  auto issue = [&](int k, int b, int stg) {
    if (k != rows_k) {
      const int tb0 = tile_of(k) * Ge::BPT;
      const int sb = tb0 / sub, s_in = tb0 - sb * sub;
      rows = planes_row + (sb * (D * NPLANES) * sub + s_in) * 2;
      srow = scales_row + sb * D * sub + (s_in & ~7);
      rows_k = k;
    }
    uint32_t* st = my_stage + stg * Ge::STAGE_U32;
    const int w0 = s_wstart[b], w1 = s_wstart[b + 1], c0 = s_bstart[b], c1 = s_bstart[b + 1];
    const int nrc = (w1 - w0) * Ge::CPR;
    const int nch = nrc + (c1 - c0);
    for (int e = lane; e < nch; e += 32) {
      if (e < nrc) {
        const int pos = w0 + e / Ge::CPR, part = e % Ge::CPR;
        if constexpr (KEEP)   // plane words are read once: evict them first
          cp_async16_hint(st + (pos - b * WB) * Ge::HPW + 4 * part, rows + s_roff[pos] + 4 * part, l2_evict_first());
        else
          cp_async16(st + (pos - b * WB) * Ge::HPW + 4 * part, rows + s_roff[pos] + 4 * part);
      } else {
        const int i = c0 + (e - nrc);
        cp_async16(st + WBUF * Ge::HPW + (i - c0) * Ge::SROW_U32, srow + s_ch[i] * sub);
      }
    }
  };

  Acc<G, P> acc;
  float2 cst[G2];
  auto reset = [&]() {
    acc.zero();
#pragma unroll
    for (int k = 0; k < G2; ++k) cst[k] = make_float2(0.f, 0.f);
  };
  reset();

  // Epilogue of one tile: scores = acc + cst per head, staged in `st` (the stage just consumed) and
  // stored with 16-byte stores; group keys from the same floats.
  auto epilogue = [&](int tile, uint32_t* st) {
    const int tb0 = tile * Ge::BPT;
    const int tok0 = tb0 * BLK;                               // first token of the tile
    const int lo_blk = blk_begin > tb0 ? blk_begin : tb0;
    const int hi_blk = blk_end < tb0 + Ge::BPT ? blk_end : tb0 + Ge::BPT;
    // valid tokens of the tile, relative to its first token: [lo, hi)
    const int lo = (lo_blk - tb0) * BLK;
    const int hi = (hi_blk * BLK < n ? hi_blk * BLK : n) - tok0;
    float* s_sc = reinterpret_cast<float*>(st);
    const bool vec_ok = (n % 4 == 0) && ((reinterpret_cast<uintptr_t>(out) & 15) == 0);
    const bool full = lo == 0 && hi == Ge::TILE_TOK;          // every token of the tile is written
    const int hwt = hw * 32;                                  // this lane's half-word, relative to the tile
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float c = (g & 1) ? cst[g >> 1].y : cst[g >> 1].x;
      uint32_t gm = 0;
      __syncwarp();
      if constexpr (P == 2 && !GK) {
        // slots 2m, 2m + 1 are the adjacent tokens 4m + r0, 4m + r0 + 1 (r0 even): one paired FMA and one
        // 8-byte store per accumulator pair
        const float2 cc = make_float2(c, c), us = make_float2(F_UNSCALE, F_UNSCALE);
#pragma unroll
        for (int m = 0; m < TPL / 2; ++m) {
          const float2 v = __ffma2_rn(acc.r[g * (TPL / 2) + m], us, cc);   // = (sum of W f) + cst, one rounding
          const int l = 4 * m + r0;
          *reinterpret_cast<float2*>(s_sc + hw * Ge::EPI_STRIDE + l) = v;
          if constexpr (GK) {
            if (full || (hwt + l >= lo && hwt + l < hi)) gm = max(gm, f2key(v.x));
            if (full || (hwt + l + 1 >= lo && hwt + l + 1 < hi)) gm = max(gm, f2key(v.y));
          }
        }
      } else {
#pragma unroll
        for (int k = 0; k < TPL; ++k) {
          const float v = fmaf(acc.get(g, k), F_UNSCALE, c);   // = (sum of W f) + cst, one rounding
          const int l = token_of<P>(k, r0);
          s_sc[hw * Ge::EPI_STRIDE + l] = v;
          if constexpr (GK) {
            if (full || (hwt + l >= lo && hwt + l < hi)) gm = max(gm, f2key(v));
          }
        }
      }
      if constexpr (GK) {
#pragma unroll
        for (int o = 1; o < Ge::LPH; o <<= 1) gm = max(gm, __shfl_xor_sync(0xffffffffu, gm, o));
        if (lane % Ge::LPH == 0 && hwt >= lo && hwt < hi) gkey[((int64_t)bh * G + g) * ng + (tok0 + hwt) / 32] = gm;
      }
      __syncwarp();
      float* o = out + ((int64_t)bh * G + g) * n + tok0;
#pragma unroll
      for (int it = 0; it < Ge::TILE_TOK / 128; ++it) {       // 128 tokens per warp instruction
        const int T = it * 128 + 4 * lane;
        const float4 v = *reinterpret_cast<const float4*>(s_sc + (T >> 5) * Ge::EPI_STRIDE + (T & 31));
        if (vec_ok && (full || (T >= lo && T + 4 <= hi))) {
          if constexpr (KEEP) st_float4_hint(o + T, v, l2_evict_last());   // the selection reads them back
          else *reinterpret_cast<float4*>(o + T) = v;
        } else {
          const float e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int u = 0; u < 4; ++u)
            if (T + u >= lo && T + u < hi) o[T + u] = e[u];
        }
      }
    }
    __syncwarp();
  };

  if (nb == 0) {                                              // no active channel: every score is 0
    for (int kk = 0; kk < ntw; ++kk) epilogue(tile_of(kk), my_stage);
    return;
  }
  const int sidx0 = hw >> 1;                                  // the lane's block within the tile
  int issued = 0, kp = 0, bp = 0, sp = 0;                     // producer: next item (kp, bp) into stage sp
  auto issue_next = [&]() {
    if (issued < items) {
      issue(kp, bp, sp);
      ++issued;
      if (++bp == nb) {
        bp = 0;
        ++kp;
      }
      if (++sp == NSTAGE) sp = 0;
    }
    cp_async_commit();                                        // one group per item slot, empty past the end
  };
  for (int j = 0; j < NSTAGE - 1; ++j) issue_next();
  int k = 0, b = 0, sc = 0;                                   // consumer: item (k, b) in stage sc
  for (int it = 0; it < items; ++it) {
    __syncwarp();                                             // every lane is done with the stage refilled next
    issue_next();
    cp_async_wait<NSTAGE - 1>();                              // this lane's copies of item it have landed
    __syncwarp();                                             // ... and every lane's
    const int tile = tile_of(k);
    const uint32_t* st = my_stage + sc * Ge::STAGE_U32;
    const uint16_t* srow16 = reinterpret_cast<const uint16_t*>(st + WBUF * Ge::HPW);
    const int sidx = ((tile * Ge::BPT) & 7) + sidx0;         // block within the aligned 8-block scale group
    const int c0 = s_bstart[b], c1 = s_bstart[b + 1];
#pragma unroll
    for (int c = 0; c < NPLANES; ++c) {
      const int i0 = c0 > s_cstart[c] ? c0 : s_cstart[c];
      const int i1 = c1 < s_cstart[c + 1] ? c1 : s_cstart[c + 1];
      if (i0 >= i1) continue;
      // consecutive channels of one class in one batch: scale rows SROW_U32 words apart, plane words
      // t = c + 1 rows apart, head tables one entry apart
      const uint16_t* sp = srow16 + (i0 - c0) * (Ge::SROW_U32 * 2) + sidx;
      const uint32_t* wr = st + s_slot[i0] * Ge::HPW + hw;
      const float4* qt = &s_qt[i0][0];
#pragma unroll 1
      for (int i = i0; i < i1; ++i, sp += Ge::SROW_U32 * 2, wr += (c + 1) * Ge::HPW, qt += G2) {
        const float s = __half2float(__ushort_as_half(*sp));
        const float2 ss = make_float2(s, s);
        float2 Wd[G];
#pragma unroll
        for (int k2 = 0; k2 < G2; ++k2) {
          const float4 v = qt[k2];
          const float2 wp = __fmul2_rn(make_float2(v.x, v.y), ss);   // {W_2k2, W_2k2+1}
          Wd[2 * k2] = make_float2(wp.x, wp.x);
          if (2 * k2 + 1 < G) Wd[2 * k2 + 1] = make_float2(wp.y, wp.y);
          cst[k2] = __ffma2_rn(ss, make_float2(v.z, v.w), cst[k2]);
        }
        if (c == 0) {
          uint32_t w[1] = {wr[0]};
          channel<1, P, G>(acc, w, amt, Wd);
        } else if (c == 1) {
          uint32_t w[2] = {wr[0], wr[Ge::HPW]};
          channel<2, P, G>(acc, w, amt, Wd);
        } else if (c == 2) {
          uint32_t w[3] = {wr[0], wr[Ge::HPW], wr[2 * Ge::HPW]};
          channel<3, P, G>(acc, w, amt, Wd);
        } else {
          uint32_t w[4] = {wr[0], wr[Ge::HPW], wr[2 * Ge::HPW], wr[3 * Ge::HPW]};
          channel<4, P, G>(acc, w, amt, Wd);
        }
      }
    }
    if (b == nb - 1) {
      epilogue(tile, my_stage + sc * Ge::STAGE_U32);
      reset();
    }
    if (++b == nb) {
      b = 0;
      ++k;
    }
    if (++sc == NSTAGE) sc = 0;
  }
  cp_async_wait<0>();                                         // only empty groups remain; leave none behind
}

}  // namespace ph
}  // namespace
}  // namespace fathom
