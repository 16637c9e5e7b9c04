// Copy-index staging of a host-resident store into device memory (gather_runs_kernel and the chunked
// copy of stream_planes, scripts/B_e2e_offload_v2.py:62-71, 118-133).
//
// The store in pinned mapped host memory keeps the run order (SUB = nblk): the nblk plane words of one
// (kv-head, channel, plane) are one contiguous run, and so are the nblk fp16 block scales of one
// (kv-head, channel).  Staging copies, for a range of blocks [b0, b1), the first t planes of every
// channel of depth t >= 1 and its scales into a device buffer of the same layout, at the same offsets;
// the plane-prefix scan then reads that range from device memory.  Inactive channels and planes
// below the plan's depth are not copied, so a staged range moves exactly the bytes of bytes_planes.
//
// Both kernels are SM-issued copies: 16-byte loads of the mapped host memory (four in flight per thread)
// and 16-byte stores to device memory.  Source and destination share their offsets, so they share their
// alignment modulo 16 bytes; a run's unaligned head and tail go byte by byte.
#include "common.cuh"

namespace fathom {
namespace {

constexpr int CT = 256;   // threads per copy CTA
constexpr int UNR = 4;    // 16-byte loads in flight per thread

// Copies nbytes from s to d with the CTA's threads; (s - d) is a multiple of 16.
__device__ __forceinline__ void cta_copy(const uint8_t* __restrict__ s, uint8_t* __restrict__ d, int64_t nbytes) {
  if (nbytes <= 0) return;
  const int tid = threadIdx.x;
  int64_t head = (16 - (int64_t)(reinterpret_cast<uintptr_t>(s) & 15)) & 15;
  if (head > nbytes) head = nbytes;
  if (tid < head) d[tid] = s[tid];
  const int64_t nvec = (nbytes - head) >> 4;
  const uint4* vs = reinterpret_cast<const uint4*>(s + head);
  uint4* vd = reinterpret_cast<uint4*>(d + head);
  int64_t i = tid;
  for (; i + (UNR - 1) * CT < nvec; i += UNR * CT) {
    uint4 v[UNR];
#pragma unroll
    for (int u = 0; u < UNR; ++u) v[u] = vs[i + u * CT];
#pragma unroll
    for (int u = 0; u < UNR; ++u) vd[i + u * CT] = v[u];
  }
  for (; i < nvec; i += CT) vd[i] = vs[i];
  const int64_t done = head + (nvec << 4);
  if (tid < nbytes - done) d[done + tid] = s[done + tid];
}

// Run r (int32 words [off[r], off[r] + len[r])) of src copied into dst at the same offsets, words
// [c0, c0 + ch) of it per CTA row y; runs r >= nrun[0], zero lengths and negative offsets are skipped.
__global__ void __launch_bounds__(CT) gather_runs_kernel(const uint32_t* __restrict__ src, uint32_t* __restrict__ dst,
                                                         const int32_t* __restrict__ off,
                                                         const int32_t* __restrict__ len,
                                                         const int32_t* __restrict__ nrun, int64_t ch) {
  const int64_t r = blockIdx.x;
  if (r >= (int64_t)*nrun || off[r] < 0) return;
  const int64_t ln = len[r];
  const int64_t c0 = (int64_t)blockIdx.y * ch;
  if (ln <= c0) return;
  const int64_t c1 = c0 + ch < ln ? c0 + ch : ln;
  const int64_t o = (int64_t)off[r] + c0;
  cta_copy(reinterpret_cast<const uint8_t*>(src + o), reinterpret_cast<uint8_t*>(dst + o), (c1 - c0) * 4);
}

// CTA (channel, kv-head): the first t planes of blocks [b0, b1) and their scales, t = depth[bh][ch]
// (clamped to 4); nothing for t = 0.
__global__ void __launch_bounds__(CT) stage_planes_kernel(const uint64_t* __restrict__ planes_src,
                                                          const uint16_t* __restrict__ scales_src,
                                                          const int8_t* __restrict__ depth, int64_t nblk, int64_t b0,
                                                          int64_t b1, uint64_t* __restrict__ planes_dst,
                                                          uint16_t* __restrict__ scales_dst) {
  const int64_t slot = (int64_t)blockIdx.y * D + blockIdx.x;   // (bh, channel)
  int t = depth[slot];
  if (t <= 0) return;
  if (t > NPLANES) t = NPLANES;
  const int64_t nb = b1 - b0;
  for (int p = 0; p < t; ++p) {
    const int64_t o = (slot * NPLANES + p) * nblk + b0;
    cta_copy(reinterpret_cast<const uint8_t*>(planes_src + o), reinterpret_cast<uint8_t*>(planes_dst + o), nb * 8);
  }
  const int64_t o = slot * nblk + b0;
  cta_copy(reinterpret_cast<const uint8_t*>(scales_src + o), reinterpret_cast<uint8_t*>(scales_dst + o), nb * 2);
}

bool same_alignment(const void* a, const void* b) {
  return ((reinterpret_cast<uintptr_t>(a) ^ reinterpret_cast<uintptr_t>(b)) & 15) == 0;
}

}  // namespace
}  // namespace fathom

using namespace fathom;

extern "C" int fathom_gather_runs(const uint32_t* src, uint32_t* dst, const int32_t* off, const int32_t* len,
                                  const int32_t* nrun, int64_t R, int64_t max_len, int64_t ch, void* stream) {
  FATHOM_REQUIRE(src && dst && off && len && nrun, FATHOM_ERR_NULL, "gather_runs: NULL pointer");
  FATHOM_REQUIRE(R >= 0 && R <= 0x7fffffffLL && max_len >= 0 && ch >= 1, FATHOM_ERR_SHAPE,
                 "gather_runs: bad shape (R=%lld max_len=%lld CH=%lld)", (long long)R, (long long)max_len,
                 (long long)ch);
  FATHOM_REQUIRE(same_alignment(src, dst), FATHOM_ERR_SHAPE,
                 "gather_runs: src and dst must have the same alignment modulo 16 bytes");
  if (R == 0 || max_len == 0) return FATHOM_OK;
  const int64_t gy = cdiv(max_len, ch);
  FATHOM_REQUIRE(gy <= 65535, FATHOM_ERR_SHAPE, "gather_runs: max_len / CH = %lld chunks exceeds 65535",
                 (long long)gy);
  gather_runs_kernel<<<dim3((unsigned)R, (unsigned)gy), CT, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      src, dst, off, len, nrun, ch);
  return check_launch("gather_runs");
}

extern "C" int fathom_stage_planes(const uint64_t* planes_src, const uint16_t* scales_src, const int8_t* t, int64_t BH,
                                   int64_t nblk, int64_t b0, int64_t b1, uint64_t* planes_dst, uint16_t* scales_dst,
                                   void* stream) {
  FATHOM_REQUIRE(planes_src && scales_src && t && planes_dst && scales_dst, FATHOM_ERR_NULL,
                 "stage_planes: NULL pointer");
  FATHOM_REQUIRE(BH >= 1 && BH <= 65535 && nblk >= 1 && b0 >= 0 && b0 <= b1 && b1 <= nblk, FATHOM_ERR_SHAPE,
                 "stage_planes: bad shape (BH=%lld nblk=%lld blocks [%lld, %lld))", (long long)BH, (long long)nblk,
                 (long long)b0, (long long)b1);
  FATHOM_REQUIRE(same_alignment(planes_src, planes_dst) && same_alignment(scales_src, scales_dst), FATHOM_ERR_SHAPE,
                 "stage_planes: source and staging must have the same alignment modulo 16 bytes");
  if (b0 == b1) return FATHOM_OK;
  stage_planes_kernel<<<dim3(D, (unsigned)BH), CT, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      planes_src, scales_src, t, nblk, b0, b1, planes_dst, scales_dst);
  return check_launch("stage_planes");
}
