"""Host-resident regime: bit-plane index and bf16 K/V rows in pinned, mapped host memory.

Mirrors the pieces of `scripts/B_e2e_offload_v2.py` that sit on the decode step:
  host_mapped / free_host / DevPtr   :29-39   (here through fathom_host_alloc_mapped)
  build_store (copy-index order)     :41-60, 267, 299-309
  gather_rows                        :73-83
  offload_attn (planes method)       :163-244 (plan, scan, sink/local top-k, unique-row gather,
                                               exact attention)
The scan reads the host store directly over the host link (zero-copy loads, one contiguous
run per (kv-head, channel, plane) in the SUB = nblk order); the rows are gathered once per
unique index per KV head.  Everything runs on CUDA kernels of libfathom_b200.so.
"""
import ctypes
import math

import torch

from . import _lib, bitplane as bp
from ._lib import check, lib, ptr, require_cuda, stream_of
from .klt import klt_query

_CAI_TYPESTR = {torch.int8: "|i1", torch.uint8: "|u1", torch.int16: "<i2", torch.int32: "<i4", torch.int64: "<i8",
                torch.float16: "<f2", torch.float32: "<f4"}


class DevPtr:
    """Device address with a dtype (scripts/B_e2e_offload_v2.py:30-32)."""

    def __init__(self, ptr_, dtype):
        self.ptr, self.dtype = ptr_, dtype

    def data_ptr(self):
        return self.ptr


class _CudaArray:
    def __init__(self, dev_ptr, shape, typestr):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (dev_ptr, False),
                                         "version": 3, "strides": None}


class MappedBuffer:
    """Pinned, portable, mapped host allocation of `shape`/`dtype`.

    .host  CPU tensor view of the memory (for filling / checking on the host)
    .dev   CUDA tensor aliasing the same memory through its device address: kernels that read it
           pull the bytes over the host link (zero-copy)
    hugepages=True backs it with 2 MB transparent huge pages (cudaHostRegister) instead of
    cudaHostAlloc.  Freed with .free() or when garbage-collected."""

    def __init__(self, shape, dtype, device=None, hugepages=False):
        self.shape, self.dtype = tuple(shape), dtype
        elem = torch.empty((), dtype=dtype).element_size()
        self.nbytes = int(math.prod(self.shape)) * elem
        hp, dp = ctypes.c_void_p(), ctypes.c_void_p()
        flags = _lib.HOST_HUGEPAGES if hugepages else 0
        check(lib().fathom_host_alloc_mapped_ex(self.nbytes, flags, ctypes.byref(hp), ctypes.byref(dp)),
              "host_alloc_mapped")
        self.hp, self.dp = hp.value, dp.value
        raw = (ctypes.c_byte * self.nbytes).from_address(self.hp)
        self.host = torch.frombuffer(raw, dtype=dtype).view(self.shape)
        cai_dtype = torch.int16 if dtype == torch.bfloat16 else dtype
        device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        alias = torch.as_tensor(_CudaArray(self.dp, self.shape, _CAI_TYPESTR[cai_dtype]), device=device)
        self.dev = alias.view(dtype) if cai_dtype != dtype else alias

    def free(self):
        if getattr(self, "hp", None):
            self.host = self.dev = None
            lib().fathom_host_free(self.hp)
            self.hp = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


_live = {}


def host_mapped(t):
    """Copy tensor t into pinned, GPU-mapped host memory (scripts/B_e2e_offload_v2.py:33-38).
    Returns (cpu view tensor, DevPtr for kernels, host pointer)."""
    buf = MappedBuffer(t.shape, t.dtype, t.device if t.is_cuda else None)
    if t.is_cuda:
        buf.dev.copy_(t)
    else:
        buf.host.copy_(t)
    _live[buf.hp] = buf
    return buf.host, DevPtr(buf.dp, t.dtype), buf.hp


def free_host(hp):
    """scripts/B_e2e_offload_v2.py:39."""
    buf = _live.pop(hp, None)
    if buf is not None:
        buf.free()


class HostPlaneStore(bp.PlaneStore):
    """A PlaneStore whose planes and scales live in pinned, mapped host memory in the copy-index order
    (SUB = nblk: every (bh, channel, plane) is one contiguous run of nblk*8 bytes).

    Built on the GPU by the fused quantise+pack kernel, then copied to the host; the device copy is
    released.  scan() reads the host memory directly (zero-copy), with the same kernel as the HBM
    store."""

    def __init__(self, K, scale_dtype=torch.float16, hugepages=False, basis=None):
        require_cuda(K)
        old = bp.SUB
        try:
            bp.SUB = math.ceil(K.shape[1] / bp.BLK)
            super().__init__(K, scale_dtype, basis)
        finally:
            bp.SUB = old
        self.planes_buf = MappedBuffer(self.planes_k.shape, torch.int64, K.device, hugepages)
        self.scales_buf = MappedBuffer(self.scales_k.shape, torch.float16, K.device, hugepages)
        self.planes_buf.dev.copy_(self.planes_k)
        self.scales_buf.dev.copy_(self.scales_k)
        torch.cuda.current_stream(K.device).synchronize()
        self.planes_k = self.planes_buf.dev
        self.planes32 = self.planes_k.view(torch.int32)
        self.scales_k = self.scales_buf.dev

    def free(self):
        self.planes_k = self.planes32 = self.scales_k = None
        self.planes_buf.free()
        self.scales_buf.free()


class HostChan4Store(bp.Chan4Store):
    """The comparator store (Chan4Store) in pinned, mapped host memory in the run order SUB = nblk: the
    full 4-bit codes of one (bh, channel) are one contiguous run of nblk*32 bytes, the layout the
    reference times its host-resident channel scans on (scripts/B_e2e_offload_v2.py:135-148, 290-296).
    Built on the GPU, copied to the host; the device copies (and the codes) are released.  scan()
    reads the listed channels' runs straight from host memory (zero-copy)."""

    def __init__(self, K, scale_dtype=torch.float16, hugepages=False):
        require_cuda(K)
        old = bp.SUB
        try:
            bp.SUB = math.ceil(K.shape[1] / bp.BLK)
            super().__init__(K, scale_dtype)
        finally:
            bp.SUB = old
        self.chan_buf = MappedBuffer(self.chan_k.shape, torch.int32, K.device, hugepages)
        self.scales_buf = MappedBuffer(self.scales_k.shape, torch.float16, K.device, hugepages)
        self.chan_buf.dev.copy_(self.chan_k)
        self.scales_buf.dev.copy_(self.scales_k)
        torch.cuda.current_stream(K.device).synchronize()
        self.chan_k = self.chan_buf.dev
        self.scales_k = self.scales_buf.dev
        self.code = None

    def free(self):
        self.chan_k = self.scales_k = None
        self.chan_buf.free()
        self.scales_buf.free()


def gather_rows(src, cap, idx, BH, dtype=torch.bfloat16, D=128):
    """dst[bh, r, :] = src[bh, idx[bh, r], :] for bf16 rows; idx < 0 leaves the row zero; src may be a
    mapped host alias (scripts/B_e2e_offload_v2.py:73-83)."""
    require_cuda(idx)
    idx = idx.to(torch.int32).contiguous()
    R = idx.shape[1]
    dst = torch.zeros(BH, R, D, device=idx.device, dtype=dtype)
    check(lib().fathom_gather_rows(ptr(src), cap, ptr(idx), BH, R, D, ptr(dst), stream_of(idx.device)),
          "gather_rows")
    return dst


def gather_runs(src, dst, off, ln, nrun, max_len, CH=4096):
    """Copy run r (int32 words [off[r], off[r] + ln[r])) of src into dst at the same word offsets, for
    r < nrun[0] (scripts/B_e2e_offload_v2.py:62-71).  off / ln int32 [R] and nrun int32 [1] are device
    tensors, so the call needs no host sync; zero lengths are skipped.  src / dst: int32 tensors or
    objects with data_ptr() (a mapped host alias, a DevPtr); every run must lie inside both."""
    require_cuda(off, ln, nrun)
    off = off.to(torch.int32).contiguous()
    ln = ln.to(torch.int32).contiguous()
    nrun = nrun.to(torch.int32).contiguous()
    check(lib().fathom_gather_runs(ptr(src), ptr(dst), ptr(off), ptr(ln), ptr(nrun), off.numel(), int(max_len),
                                   int(CH), stream_of(off.device)), "gather_runs")


class PlaneStaging:
    """Device buffers in the run order of a host store (planes [BH, 1, 128, 4, nblk] int64, scales
    [BH, 1, 128, nblk] fp16) that receive the staged block ranges of stream_planes.  One staging serves
    every layer of the same shape; it exposes the attributes PlaneStore.scan reads."""

    def __init__(self, BH, n, device):
        nblk = math.ceil(n / bp.BLK)
        self.BH, self.n, self.nblk, self.sub, self.nsb, self.basis = BH, n, nblk, nblk, 1, None
        self.planes_k = torch.empty(BH, 1, bp.D, 4, nblk, dtype=torch.int64, device=device)
        self.planes32 = self.planes_k.view(torch.int32)
        self.scales_k = torch.empty(BH, 1, bp.D, nblk, dtype=torch.float16, device=device)


_stagings = {}
_copy_streams = {}


def _staging_for(BH, n, dev):
    key = (dev, BH, n)
    s = _stagings.get(key)
    if s is None:
        s = _stagings[key] = PlaneStaging(BH, n, dev)
    return s


def release_staging(device=None):
    """Drop the kept PlaneStaging buffers (all devices, or one): ~68 B per token and KV head each."""
    for key in [k for k in _stagings if device is None or k[0] == torch.device(device)]:
        del _stagings[key]


def _pipeline_streams(dev):
    s = _copy_streams.get(dev)
    if s is None:
        s = _copy_streams[dev] = (torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev))
    return s


def chunk_bounds(nblk, parts, align=64):
    """Block ranges [(b0, b1), ...] covering [0, nblk) in `parts` chunks whose inner boundaries are
    multiples of `align` blocks; empty ranges dropped (scripts/B_e2e_offload_v2.py:106-109)."""
    parts = max(1, int(parts))
    bs = [0] + [min(nblk, ((nblk * i // parts) // align) * align) for i in range(1, parts)] + [nblk]
    return [(a, b) for a, b in zip(bs[:-1], bs[1:]) if b > a]


def stream_planes(st, qf, plan, n=None, BH=None, parts=4, staging=None, scores=None):
    """The chunk-pipelined copy-index scan (stream_planes, scripts/B_e2e_offload_v2.py:118-133) of a
    host store `st` (HostPlaneStore, run order): for each block chunk, the first t planes of every
    active channel and its block scales are staged from host memory into device memory on a copy
    stream (fathom_stage_planes), and the chunk's scan runs from device memory on a scan stream once
    its copy has landed, so chunk i+1's copy overlaps chunk i's scan.  parts=1 is the unpipelined
    copy-index mode (:186-196).  The scores are those of st.scan(qf, plan), bit for bit.  staging: a
    PlaneStaging of the store's shape (otherwise one per (device, BH, n) is kept until
    release_staging()).  Calls that share a staging must be ordered on the current stream: each call
    joins its copy and scan streams back into it before returning."""
    require_cuda(qf)
    BH_, G, _ = qf.shape
    n = st.n if n is None else n
    BH = BH_ if BH is None else BH
    if BH != st.BH or n != st.n or st.sub != math.ceil(n / bp.BLK):
        raise ValueError("stream_planes: the store must hold BH x n tokens in the run order (sub = nblk)")
    dev = qf.device
    staging = _staging_for(BH, n, dev) if staging is None else staging
    if staging.BH != BH or staging.n != n or staging.planes_k.device != dev:
        raise ValueError(f"stream_planes: the staging must be a PlaneStaging({BH}, {n}) on {dev}")
    scores = torch.empty(BH, G, n, device=dev, dtype=torch.float32) if scores is None else scores
    t = plan["t"]
    if t.dtype != torch.int8 or not t.is_contiguous():
        t = t.to(torch.int8).contiguous()
    cur = torch.cuda.current_stream(dev)
    s_copy, s_scan = _pipeline_streams(dev)
    s_copy.wait_stream(cur)
    s_scan.wait_stream(cur)
    for b0, b1 in chunk_bounds(staging.nblk, parts):
        with torch.cuda.stream(s_copy):
            check(lib().fathom_stage_planes(ptr(st.planes_k), ptr(st.scales_k), ptr(t), BH, staging.nblk, b0, b1,
                                            ptr(staging.planes_k), ptr(staging.scales_k), s_copy.cuda_stream),
                  "stage_planes")
        s_scan.wait_stream(s_copy)
        with torch.cuda.stream(s_scan):
            bp.PlaneStore.scan(staging, qf, plan, out=scores, blocks=(b0, b1))
    cur.wait_stream(s_scan)
    return scores


def _row_stride(t):
    """Elements between consecutive rows of a K/V source (128 unless it is a strided tensor view)."""
    return t.stride(-2) if isinstance(t, torch.Tensor) and t.dim() >= 2 else 0


def decode_attention(q, idx, K_src, V_src, cap, n_host=None, K_recent=None, V_recent=None, recent_cap=0,
                     out_dtype=torch.float32):
    """Exact attention over the selected rows (scripts/B_e2e_offload_v2.py:226-244):
    q [BH, G, 128] fp32, idx [BH, G, k] int64.  Unique indices of a KV head are fetched once; an index
    >= n_host reads row idx - n_host of the device-resident recent buffers [BH, recent_cap, 128].
    Returns [BH, G, 128] in out_dtype (float32 or bfloat16)."""
    require_cuda(q, idx)
    BH, G, D = q.shape
    k = idx.shape[-1]
    n_host = cap if n_host is None else n_host
    dev = q.device
    qc = q.contiguous().float()
    ic = idx.contiguous().to(torch.int64)
    out = torch.empty(BH, G, D, device=dev, dtype=out_dtype)
    if out_dtype not in (torch.float32, torch.bfloat16):
        raise TypeError("decode_attention: out_dtype must be float32 or bfloat16")
    ws = _lib.workspace(dev, lib().fathom_decode_workspace_bytes(BH, G, k), "decode")
    check(lib().fathom_decode_attention(ptr(qc), BH, G, ptr(ic), k, ptr(K_src), ptr(V_src), cap,
                                        _row_stride(K_src), n_host,
                                        ptr(K_recent), ptr(V_recent), recent_cap,
                                        ptr(out) if out_dtype == torch.float32 else None,
                                        ptr(out) if out_dtype == torch.bfloat16 else None,
                                        ptr(ws), ws.numel(), stream_of(dev)), "decode_attention")
    return out


def decode_step(q, g, budget, store, K_src, V_src, cap, k=580, sink=4, local=64, n_host=None, K_recent=None,
                V_recent=None, recent_cap=0, scores=None, out_dtype=torch.float32, stream_parts=0):
    """One layer of an offloaded decode step (offload_attn, scripts/B_e2e_offload_v2.py:180-244, planes
    method): plan -> plane-prefix scan of the (host or HBM) store -> sink+local top-k -> unique-row
    gather + exact attention.  Returns (out [BH,G,128], idx [BH,G,k]).

    stream_parts > 0 (host store only) scans through the copy-index pipeline, stream_planes with that
    many chunks (the reference's --copy-index --pipeline mode, :182-185), then selects with
    sink_local_topk; the results are those of the default zero-copy scan, bit for bit.

    A store built with a KLT basis (planesK, scripts/R_ruler.py:82-84) is scanned with the rotated
    queries q @ Vt and planned on their gains sum_g (q Vt)^2 * lam (g is then ignored and may be None);
    attention always uses q itself."""
    qs = q
    if getattr(store, "basis", None) is not None:
        qs, g = klt_query(q, store.basis)
    plan = bp.make_plan(g, budget)
    if stream_parts:
        scores = stream_planes(store, qs, plan, parts=stream_parts, scores=scores)
        idx = bp.sink_local_topk(scores, k, sink, local)
    else:
        idx = bp.scan_topk(store, qs, plan, k, sink, local, scores=scores)
    out = decode_attention(q, idx, K_src, V_src, cap, n_host, K_recent, V_recent, recent_cap, out_dtype)
    return out, idx


def decode_attention_partial(q, idx, K_src, V_src, cap, idx_lo, idx_hi):
    """Attention of one context shard over the picks it owns ([idx_lo, idx_hi), rows idx - idx_lo of
    K_src/V_src).  Returns packed partials fp32 [BH, G, 130] = (unnormalised output[128], max, sum-exp)."""
    require_cuda(q, idx)
    BH, G, D = q.shape
    k = idx.shape[-1]
    dev = q.device
    qc = q.contiguous().float()
    ic = idx.contiguous().to(torch.int64)
    out = torch.empty(BH, G, D + 2, device=dev, dtype=torch.float32)
    ws = _lib.workspace(dev, lib().fathom_decode_partial_workspace_bytes(BH, G, k), "decode_partial")
    check(lib().fathom_decode_attention_partial(ptr(qc), BH, G, ptr(ic), k, ptr(K_src), ptr(V_src), cap,
                                                _row_stride(K_src), idx_lo, idx_hi,
                                                ptr(out), ptr(ws), ws.numel(), stream_of(dev)),
          "decode_attention_partial")
    return out


def attention_combine(parts, out_dtype=torch.float32):
    """Log-sum-exp merge of packed partials [P, BH, G, 130] -> [BH, G, 128]."""
    require_cuda(parts)
    P, BH, G, W = parts.shape
    pc = parts.contiguous().float()
    out = torch.empty(BH, G, W - 2, device=parts.device, dtype=out_dtype)
    check(lib().fathom_attention_combine(ptr(pc), P, BH * G, ptr(out) if out_dtype == torch.float32 else None,
                                         ptr(out) if out_dtype == torch.bfloat16 else None,
                                         stream_of(parts.device)), "attention_combine")
    return out
