/*
 * fathom_b200 -- C ABI of the B200 (sm_100a) key-scan library.
 *
 * Every entry point takes plain device pointers (or device aliases of pinned,
 * mapped host memory), sizes, and a CUDA stream passed as `void*`
 * (a cudaStream_t; NULL = the legacy default stream).  Work is enqueued on that
 * stream and the call returns without synchronising.  Every function returns
 * FATHOM_OK (0) or a negative status; fathom_last_error() then holds a message
 * for the calling thread.  No function allocates device memory except
 * fathom_host_alloc_mapped; scratch space is a caller-provided workspace whose
 * size the matching *_workspace_bytes() function returns.
 *
 * Store layout ("superblock order", reference kernels/bitplane.py:7-11, 60-65):
 *   planes_k [BH][nsb][128][4][sub]  uint64   bit i of word (bh,sb,j,p,s) is bit p
 *                                             (p = 0 = MSB) of the 4-bit code of token
 *                                             64*(sb*sub+s)+i, channel j
 *   scales_k [BH][nsb][128][sub]     fp16     absmax of block sb*sub+s, channel j
 *   nsb = ceil(nblk / sub), nblk = ceil(n / 64); pad blocks hold zero words/scales.
 * sub = 16 is the HBM order; sub = nblk is the host "copy-index" order in which
 * every (bh, channel, plane) is one contiguous run (scripts/B_e2e_offload_v2.py:267);
 * sub = 1 is the logical order of pack_planes (kernels/bitplane.py:44-50).
 */
#ifndef FATHOM_B200_H
#define FATHOM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  FATHOM_OK = 0,
  FATHOM_ERR_NULL = -1,        /* a required pointer is NULL */
  FATHOM_ERR_SHAPE = -2,       /* a size / shape / range argument is invalid */
  FATHOM_ERR_UNSUPPORTED = -3, /* valid request outside what this build implements */
  FATHOM_ERR_CUDA = -4,        /* a CUDA runtime call or a kernel launch failed */
  FATHOM_ERR_WORKSPACE = -5    /* caller workspace too small or misaligned */
};

enum { FATHOM_DTYPE_F32 = 0, FATHOM_DTYPE_BF16 = 1, FATHOM_DTYPE_F16 = 2 };

/* Message of the last failing call on this thread ("" if none). */
const char* fathom_last_error(void);
/* ABI version of this library (bumped on any signature change). */
int fathom_abi_version(void);

/* ---------------------------------------------------------------- store build */

/* Quantise keys to 4-bit codes and pack them into bit planes in one pass.
 * Replaces quantise_u4 + pack_planes + to_superblocks (kernels/bitplane.py:23-32,
 * 44-50, 60-65) as used by PlaneStore.__init__ (kernels/bitplane.py:312-316).
 *   K          [BH][n][128] rows of k_dtype; row bh starts at K + bh*k_stride_bh elements
 *   amax_f16   1: the block absmax is rounded to fp16 before the codes are computed
 *              (scale_dtype=float16, the default); 0: fp32 absmax (scale_dtype=float32)
 * Outputs (each may be NULL):
 *   code       [BH][n][128] uint8 codes in [0, 16)
 *   scales_blk [BH][nblk][128] absmax, fp32 if scales_blk_f32 else fp16
 *   planes_k / scales_k   the store in superblock order `sub` (see above); pad
 *              blocks up to nsb*sub are written with zeros. */
int fathom_quantise_pack(const void* K, int k_dtype, int64_t BH, int64_t n, int64_t k_stride_bh,
                         int64_t sub, int amax_f16, uint8_t* code, void* scales_blk, int scales_blk_f32,
                         uint64_t* planes_k, uint16_t* scales_k, void* stream);

/* Codes [BH][n][128] uint8 -> planes in superblock order `sub` (sub = 1: pack_planes,
 * kernels/bitplane.py:44-50).  Pad tokens and pad blocks are zero. */
int fathom_pack_codes(const uint8_t* code, int64_t BH, int64_t n, int64_t sub, uint64_t* planes_k, void* stream);

/* Planes in superblock order `sub` -> codes [BH][n][128] uint8 (unpack_planes,
 * kernels/bitplane.py:52-58, with sub = 1). */
int fathom_unpack_planes(const uint64_t* planes_k, int64_t BH, int64_t n, int64_t sub, uint8_t* code, void* stream);

/* Re-order a store between superblock orders (to_superblocks, kernels/bitplane.py:60-65,
 * is sub_src = 1 -> sub_dst = SUB).  Either pair of pointers may be NULL. */
int fathom_relayout(const uint64_t* planes_src, const uint16_t* scales_src, int64_t BH, int64_t nblk, int64_t sub_src,
                    uint64_t* planes_dst, uint16_t* scales_dst, int64_t sub_dst, void* stream);

/* ---------------------------------------------------------------- dense reference helpers */

/* dequant_planes (kernels/bitplane.py:34-42): out [rows][n][128] fp32 = the top-t planes of the
 * codes dequantised, ((c >> (4-t)) + 0.5 - 2^(t-1)) * s / 2^(t-1) in that fp32 order, 0 where t = 0.
 *   code [rows][n][128] uint8; scales [rows][ceil(n/64)][128] block absmax, fp32 if scales_f32 else fp16;
 *   t int32 depths, [128] shared by every row (t_stride_row = 0) or [rows][128] (t_stride_row = 128);
 *   depths above 4 are read as 4. */
int fathom_dequant_planes(const uint8_t* code, const void* scales, int scales_f32, int64_t rows, int64_t n,
                          const int32_t* t, int64_t t_stride_row, float* out, void* stream);

/* scan_planes_reference (kernels/bitplane.py:357-363): scores [BH][G][n] = q [BH][G][128] times the
 * dequant_planes values of code [BH][n][128] (16-byte aligned) with per-row depths t [BH][128] int32,
 * summed over channels in ascending order.  G in 1..8. */
int fathom_scan_planes_reference(const float* q, int64_t BH, int G, int64_t n, const uint8_t* code,
                                 const void* scales, int scales_f32, const int32_t* t, float* scores, void* stream);

/* scan_chan4_reference (kernels/bitplane.py:365-370): as fathom_scan_planes_reference with every
 * channel at depth 4, each value multiplied by its channel's active flag (active [BH][128], 0/1 bytes). */
int fathom_scan_chan4_reference(const float* q, int64_t BH, int G, int64_t n, const uint8_t* code,
                                const void* scales, int scales_f32, const uint8_t* active, float* scores,
                                void* stream);

/* ---------------------------------------------------------------- plan */

/* Per-(batch, kv-head) reverse water-filling plan (plan_kernel + make_plan,
 * kernels/bitplane.py:83-116; depths equal make_plan_torch, :118-126).
 *   g [BH][128] fp32 gains; budget [BH] fp32 bits per token.
 *   t [BH][128] int8; pairs [BH][128*bmax], npairs [BH]; act [BH][128], nact [BH];
 *   cls [BH][bmax][128], clsn [BH][bmax] (int32).  List tails are zero-filled.
 *   bmax in 1..4; iters >= 0. */
int fathom_make_plan(const float* g, const float* budget, int64_t BH, int bmax, int iters, int8_t* t, int32_t* pairs,
                     int32_t* npairs, int32_t* act, int32_t* nact, int32_t* cls, int32_t* clsn, void* stream);

/* ---------------------------------------------------------------- scan */

/* Plane-prefix scan (PlaneStore.scan -> scan_planes_cls_kernel, kernels/bitplane.py:319-338,
 * 275-307): scores[bh][g][tok] = sum_j q[bh][g][j] * value_{t_j}(tok, j) over the channels
 * of the depth-class lists, reading only the first t_j planes of channel j.
 *   q [BH][G][128] fp32, G in 1..8; cls/clsn from fathom_make_plan (stride bmax);
 *   planes_k/scales_k in order `sub`, device memory or a mapped host alias;
 *   tokens of blocks [blk_begin, blk_end) are written to scores [BH][G][n]; others untouched.
 *   Channel ids are taken modulo 128 and class counts clamped to 0..128 (plans from
 *   fathom_make_plan always satisfy both). */
int fathom_scan(const float* q, int64_t BH, int G, int64_t n, int64_t sub, const int32_t* cls, const int32_t* clsn,
                int bmax, const uint64_t* planes_k, const uint16_t* scales_k, int64_t blk_begin, int64_t blk_end,
                float* scores, void* stream);

/* Diagnostic, no reference counterpart: the number of bounded device waits that gave up on the
 * current device since the last reset (the scan's bulk-copy mbarrier waits, 2 s each).  A wait
 * that gives up makes its tile's scores NaN; 0 in normal operation.  Synchronises the device.
 *   count may be NULL; reset != 0 zeroes the counter after reading it. */
int fathom_wait_timeouts(unsigned long long* count, int reset);

/* Workspace bytes of fathom_scan_select: enough for either selection path (below). */
size_t fathom_scan_select_workspace_bytes(int64_t BH, int G, int64_t n, int64_t kk);

/* PlaneStore.scan followed by sink_local_topk-style selection in one call (kernels/bitplane.py:319-338,
 * 372-378), all on the stream.  Writes scores [BH][G][n] (all blocks) and, per row r = bh*G+g, the
 * top-kk of tokens in [mask_lo, mask_hi) plus index_offset to out_idx [r][out_stride] in (score desc,
 * index asc) order, followed by 0..append_sink-1 and n-append_local..n-1; the selected scores to
 * out_scores [r][kk] if not NULL.  sink_local_topk(k, sink, local) is kk = k-sink-local, mask
 * [sink, n-local), offset 0, append (sink, local), out_stride k.  When the row has at least 1.5*kk
 * fully unmasked 32-token groups, the scan also writes each group's largest score key to the
 * workspace and one selection kernel per row works from those (group-key path); otherwise the
 * histogram / collect / finalize passes run.  The workspace must hold the chosen path's buffers;
 * fathom_scan_select_workspace_bytes() covers both.  scan_done_event (a cudaEvent_t, may be NULL)
 * is recorded on the stream right after the scan kernel, to time the scan alone. */
int fathom_scan_select(const float* q, int64_t BH, int G, int64_t n, int64_t sub, const int32_t* cls,
                       const int32_t* clsn, int bmax, const uint64_t* planes_k, const uint16_t* scales_k, int64_t kk,
                       int64_t mask_lo, int64_t mask_hi, int64_t index_offset, int64_t append_sink,
                       int64_t append_local, float* scores, int64_t* out_idx, int64_t out_stride, float* out_scores,
                       void* workspace, size_t workspace_bytes, void* scan_done_event, void* stream);

/* ---------------------------------------------------------------- Chan4 comparator */

/* pack_chan4 (kernels/bitplane.py:67-74): codes [BH][n][128] uint8 -> chan_k [BH][nsb][128][sub][8]
 * int32, nibble k of word m of block s = the code of token 64*(sb*sub+s) + 8*m + k (pad tokens 0). */
int fathom_pack_chan4(const uint8_t* code, int64_t BH, int64_t n, int64_t sub, int32_t* chan_k, void* stream);

/* channel_list (kernels/bitplane.py:128-132): active [BH][128] (0/1 bytes) -> act [BH][128] int32
 * (active channels ascending, then the inactive ones ascending) and nact [BH] int32. */
int fathom_channel_list(const uint8_t* active, int64_t BH, int32_t* act, int32_t* nact, void* stream);

/* Chan4Store.scan -> scan_chan4_kernel (kernels/bitplane.py:342-352, 175-198): scores[bh][g][tok] =
 * sum over the first nact[bh] channels of act of q[bh][g][ch] * (c - 7.5) * s / 8, reading the full
 * 4-bit codes (32 + 2 bytes per block and channel).  q [BH][G][128] fp32, G in 1..8; chan_k from
 * fathom_pack_chan4 and scales_k [BH][nsb][128][sub] fp16 in order `sub`; tokens of blocks
 * [blk_begin, blk_end) are written to scores [BH][G][n], others untouched.  Channel ids are taken
 * modulo 128 and nact clamped to 0..128. */
int fathom_scan_chan4(const float* q, int64_t BH, int G, int64_t n, int64_t sub, const int32_t* act,
                      const int32_t* nact, const int32_t* chan_k, const uint16_t* scales_k, int64_t blk_begin,
                      int64_t blk_end, float* scores, void* stream);

/* ---------------------------------------------------------------- KLT-rotated store (planesK) */

/* The planesK store build (scripts/R_ruler.py:63-64: codes_u4 of einsum(Kp - mu, Vt)): the keys
 * rotated into a per-head basis, Kr[bh][tok][e] = sum_d (K[bh][tok][d] - mu[bh][d]) * Vt[bh][d][e] in
 * fp32 (pad tokens 0), then the same quantiser and store as fathom_quantise_pack, with the same
 * arguments.  mu [BH][128] and Vt [BH][128][128] fp32 (Vt 16-byte aligned); rot_out, if given,
 * receives Kr [BH][n][128] fp32 (16-byte aligned).  amax_f16 = 0 gives the reference planesK codes
 * (codes_u4: fp32 block absmax); the stored scales_k are fp16 either way. */
int fathom_klt_quantise_pack(const void* K, int k_dtype, int64_t BH, int64_t n, int64_t k_stride_bh,
                             const float* mu, const float* Vt, int64_t sub, int amax_f16, uint8_t* code,
                             void* scales_blk, int scales_blk_f32, uint64_t* planes_k, uint16_t* scales_k,
                             float* rot_out, void* stream);

/* The planesK query side (scripts/R_ruler.py:82-84): qr[bh][g][e] = sum_d q[bh][g][d] * Vt[bh][d][e]
 * and, if gains is given, gains[bh][e] = sum_g qr[bh][g][e]^2 * lam[bh][e] (the water-filling gains of
 * fathom_make_plan).  q [BH][G][128], lam [BH][128], qr [BH][G][128], gains [BH][128] fp32; G in 1..8. */
int fathom_klt_query(const float* q, int64_t BH, int G, const float* Vt, const float* lam, float* qr, float* gains,
                     void* stream);

/* ---------------------------------------------------------------- selection */

/* Workspace bytes fathom_select_topk / fathom_sink_local_topk need for `rows` rows of n scores:
 * enough for either selection path (the group-key path, taken when a row has at least 1.5*kk fully
 * unmasked 32-token groups and the workspace holds rows * ceil(n/32) keys; else the histogram path). */
size_t fathom_select_workspace_bytes(int64_t rows, int64_t n, int64_t kk);

/* Top-kk of each row of scores [rows][n] (row r at scores + r*row_stride), with tokens
 * outside [mask_lo, mask_hi) treated as -inf.  Output indices (plus index_offset) in the
 * order (score descending, index ascending) to out_idx [rows][out_stride] int64, and the
 * selected scores to out_scores [rows][kk] if not NULL.  kk in 1..4096, kk <= n.
 * The selection step of sink_local_topk (kernels/bitplane.py:372-378, torch.topk :376). */
int fathom_select_topk(const float* scores, int64_t rows, int64_t n, int64_t row_stride, int64_t kk, int64_t mask_lo,
                       int64_t mask_hi, int64_t index_offset, int64_t* out_idx, int64_t out_stride, float* out_scores,
                       void* workspace, size_t workspace_bytes, void* stream);

/* sink_local_topk (kernels/bitplane.py:372-378): idx [rows][k] int64 = the top (k-sink-local)
 * of tokens [sink, n-local) followed by 0..sink-1 and n-local..n-1. */
int fathom_sink_local_topk(const float* scores, int64_t rows, int64_t n, int64_t k, int64_t sink, int64_t local,
                           int64_t* idx, void* workspace, size_t workspace_bytes, void* stream);

/* Rows the library-owned scratch of fathom_sink_local_topk_static holds. */
#define FATHOM_STATIC_TOPK_MAX_ROWS 64

/* sink_local_topk exactly as fathom_sink_local_topk, but with no workspace argument and no
 * allocation of any kind: for callers that cannot allocate device memory on the call path (a host
 * whose device memory is all handed to its own pool, or a decode loop that cannot take
 * cudaMalloc's implicit device synchronisation).  No counterpart in the reference.
 * Scratch: one library-owned device array of about 5.3 MB, sized for FATHOM_STATIC_TOPK_MAX_ROWS
 * rows, held by every GPU that loads the library until the process exits.  rows above that limit
 * are rejected with FATHOM_ERR_SHAPE.  The array comes into existence when the driver loads the
 * library's selection module on a device; under CUDA's default lazy module loading that is the
 * first call on the device that uses the module (this function, or any selection call), which is
 * where its 5.3 MB are taken.  So make one such call on each device before handing the rest of
 * its memory to a pool and before any stream capture (or run with CUDA_MODULE_LOADING=EAGER).
 * Every call looks up the array's device address (cudaGetSymbolAddress) with the device current.
 * All calls on a device share the array: calls whose GPU work overlaps (different streams or
 * threads) race on it, so serialise them. */
int fathom_sink_local_topk_static(const float* scores, int64_t rows, int64_t n, int64_t k, int64_t sink,
                                  int64_t local, int64_t* idx, void* stream);

/* Final top-kk of candidate lists [rows][m] (scores, distinct global int64 indices < 2^32) in the
 * (score descending, index ascending) order: the merge of per-shard candidates of a
 * context-sharded scan.  No reference counterpart (the reference runs on one GPU);
 * it restates the top-k of sink_local_topk (kernels/bitplane.py:376) over a union.
 * m in 1..8192, kk <= min(m, 4096). */
int fathom_merge_topk(const float* cand_scores, const int64_t* cand_idx, int64_t rows, int64_t m, int64_t kk,
                      int64_t* out_idx, float* out_scores, void* stream);

/* ---------------------------------------------------------------- rows + attention */

/* dst[bh][r][:] = src[bh][idx[bh][r]][:] for bf16 rows of D (D*2 a multiple of 16);
 * idx < 0 skips the row (no traffic, dst row untouched); so does idx >= cap.  src may be a mapped host alias
 * (gather_rows_kernel, scripts/B_e2e_offload_v2.py:73-83). */
int fathom_gather_rows(const uint16_t* src, int64_t cap, const int32_t* idx, int64_t BH, int64_t R, int64_t D,
                       uint16_t* dst, void* stream);

/* Workspace bytes of fathom_decode_attention. */
size_t fathom_decode_workspace_bytes(int64_t BH, int G, int64_t k);

/* Decode attention over selected rows (offload_attn tail, scripts/B_e2e_offload_v2.py:226-244;
 * HBM twin gather_attn, scripts/B_kernel_bench.py:26-31):
 *   q [BH][G][128] fp32; idx [BH][G][k] int64 token indices.
 *   Rows in host memory (mapped aliases): each unique index of a KV head is fetched once over the
 *   link, in ascending order, into the workspace.  Rows in device memory (K_src, V_src and the recent
 *   buffers all device allocations): each pick's rows are read in place and the workspace is unused.
 *   Either way the sums run in pick order, so both give the same bits.  Index < n_host reads row idx of
 *   K_src/V_src [BH][cap] rows of 128 bf16, kv_row_stride elements apart (0 = 128; 256 for a cache
 *   that interleaves each token's K and V rows), in device memory or a mapped host alias; index >= n_host
 *   reads row idx-n_host of K_recent/V_recent [BH][recent_cap][128] bf16 (device).
 *   out = softmax(q K_sel^T / sqrt(128)) V_sel in fp32 math, to out_f32 [BH][G][128]
 *   and/or out_bf16 (either may be NULL).  Picks at or beyond n_host + recent_cap are ignored. */
int fathom_decode_attention(const float* q, int64_t BH, int G, const int64_t* idx, int64_t k, const uint16_t* K_src,
                            const uint16_t* V_src, int64_t cap, int64_t kv_row_stride, int64_t n_host,
                            const uint16_t* K_recent, const uint16_t* V_recent, int64_t recent_cap, float* out_f32,
                            uint16_t* out_bf16, void* workspace, size_t workspace_bytes, void* stream);

/* Workspace bytes of fathom_decode_attention_partial. */
size_t fathom_decode_partial_workspace_bytes(int64_t BH, int G, int64_t k);

/* Partial decode attention of one context shard.  Only picks in [idx_lo, idx_hi) are owned by this
 * shard; they read row idx-idx_lo of K_src/V_src [BH][cap][128] (cap >= idx_hi-idx_lo).  Writes,
 * per (bh, g), out_packed [BH][G][130] fp32 = (sum_r e^(s_r - m) V_r [128], m, l) with
 * m = max owned score (-inf if none) and l = sum_r e^(s_r - m).  No reference counterpart (the
 * reference runs on one GPU); it splits the attention of offload_attn
 * (scripts/B_e2e_offload_v2.py:242-244) across context shards. */
int fathom_decode_attention_partial(const float* q, int64_t BH, int G, const int64_t* idx, int64_t k,
                                    const uint16_t* K_src, const uint16_t* V_src, int64_t cap, int64_t kv_row_stride,
                                    int64_t idx_lo, int64_t idx_hi, float* out_packed, void* workspace,
                                    size_t workspace_bytes, void* stream);

/* Log-sum-exp merge of P shards' packed partials [P][rows][130] -> out [rows][128] (fp32 and/or
 * bf16): out = sum_p o_p e^(m_p - M) / sum_p l_p e^(m_p - M), M = max_p m_p. */
int fathom_attention_combine(const float* parts, int64_t P, int64_t rows, float* out_f32, uint16_t* out_bf16,
                             void* stream);

/* ---------------------------------------------------------------- copy-index staging */

/* Copy run r = int32 words [off[r], off[r] + len[r]) of src into dst at the same word offsets, for
 * r < nrun[0] (a device scalar, so the run count needs no host sync); CTA (r, y) copies words
 * [y*ch, (y+1)*ch) of its run.  Zero lengths and negative offsets are skipped; every run must lie
 * inside both buffers.  src and dst need the same alignment modulo 16 bytes; src is normally the
 * mapped host alias of a host-resident store and dst its device staging (gather_runs_kernel,
 * scripts/B_e2e_offload_v2.py:62-71).  R runs (grid x), ceil(max_len / ch) <= 65535 chunks. */
int fathom_gather_runs(const uint32_t* src, uint32_t* dst, const int32_t* off, const int32_t* len,
                       const int32_t* nrun, int64_t R, int64_t max_len, int64_t ch, void* stream);

/* One chunk of the pipelined copy-index scan (the per-chunk copies of stream_planes,
 * scripts/B_e2e_offload_v2.py:118-133): for every (bh, channel) with depth t = t[bh][channel] >= 1,
 * planes 0..t-1 of blocks [b0, b1) and the fp16 scales of those blocks, from a store in the run
 * order (planes [BH][1][128][4][nblk] uint64, scales [BH][1][128][nblk]; normally mapped host
 * memory) into a device buffer of the same layout at the same offsets.  Moves bytes_planes(t) of
 * the block range, nothing for inactive channels.  Sources and staging need the same alignment
 * modulo 16 bytes. */
int fathom_stage_planes(const uint64_t* planes_src, const uint16_t* scales_src, const int8_t* t, int64_t BH,
                        int64_t nblk, int64_t b0, int64_t b1, uint64_t* planes_dst, uint16_t* scales_dst,
                        void* stream);

/* ---------------------------------------------------------------- host memory */

/* Pinned, portable, mapped host allocation and its device alias (host_mapped,
 * scripts/B_e2e_offload_v2.py:33-38, which calls cudaHostAlloc(flags=3) and
 * cudaHostGetDevicePointer through ctypes). */
int fathom_host_alloc_mapped(size_t bytes, void** host_ptr, void** dev_ptr);
/* Flags of fathom_host_alloc_mapped_ex. */
#define FATHOM_HOST_HUGEPAGES 1

/* fathom_host_alloc_mapped with options.  FATHOM_HOST_HUGEPAGES: anonymous memory advised to use
 * 2 MB transparent huge pages (size rounded up to 2 MB, pre-faulted), pinned and mapped with
 * cudaHostRegister(Mapped | Portable), so the GPU translates fewer pages on random row reads.
 * No reference counterpart (the reference allocates with cudaHostAlloc only). */
int fathom_host_alloc_mapped_ex(size_t bytes, int flags, void** host_ptr, void** dev_ptr);

/* free_host (scripts/B_e2e_offload_v2.py:39); frees either kind of mapped allocation. */
int fathom_host_free(void* host_ptr);

#ifdef __cplusplus
}
#endif

#endif /* FATHOM_B200_H */
