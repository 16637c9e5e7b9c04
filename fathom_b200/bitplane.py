"""Drop-in replacement for the reference module `kernels/bitplane.py` on B200.

Same names, argument meanings, shapes and dtypes as the reference; every operation runs
on hand-written sm_100a CUDA kernels through the C ABI of libfathom_b200.so.  There is no
Triton, no CPU path and no backend dispatch: tensors must be CUDA tensors.

Store semantics (kernels/bitplane.py:3-11): per 64-token block and channel, a 4-bit mid-rise
code c in [0, 16) with an absmax scale s; value = (c + 0.5 - 8) * s / 8.  Bit p (0 = MSB) of the
64 codes of a block is one 64-bit plane word; reading the first t planes of a channel is the
t-bit quantiser.  `planes_k` is in superblock order [BH][nsb][128][4][SUB].

Module globals BLK, SUB, D, SBT mirror the reference (kernels/bitplane.py:19-20); callers that
mutate SUB (the host "copy-index" order, SUB = nblk) get stores in that order.
"""
import math

import torch

from . import _lib
from ._lib import check, lib, ptr, require_cuda, stream_of

BLK, SUB, D = 64, 16, 128
SBT = BLK * SUB


def _nblk(n):
    return math.ceil(n / BLK)


# ------------------------------------------------------------------ store build
def quantise_u4(K, scale_dtype=torch.float16):
    """K [..., n, D] -> codes uint8 [..., n, D] in [0, 16) and scales [..., nblk, D] in scale_dtype
    (kernels/bitplane.py:23-32).  The codes are computed from the fp16-rounded absmax when
    scale_dtype is float16 and from the fp32 absmax when it is float32."""
    require_cuda(K)
    if K.dtype not in _lib.DTYPE_CODE:
        raise TypeError(f"quantise_u4: unsupported key dtype {K.dtype}")
    if scale_dtype not in (torch.float16, torch.float32):
        raise TypeError("quantise_u4: scale_dtype must be torch.float16 or torch.float32")
    *lead, n, d = K.shape
    if d != D:
        raise ValueError(f"quantise_u4: head dimension must be {D} (got {d})")
    Kc = K.reshape(-1, n, d).contiguous()
    BH, nb = Kc.shape[0], _nblk(n)
    code = torch.empty(BH, n, d, dtype=torch.uint8, device=K.device)
    scales = torch.empty(BH, nb, d, dtype=scale_dtype, device=K.device)
    check(lib().fathom_quantise_pack(ptr(Kc), _lib.DTYPE_CODE[K.dtype], BH, n, n * d, 1,
                                     int(scale_dtype == torch.float16), ptr(code), ptr(scales),
                                     int(scale_dtype == torch.float32), None, None, stream_of(K.device)),
          "quantise_u4")
    return code.view(*lead, n, d), scales.view(*lead, nb, d)


def pack_planes(code):
    """codes uint8 [..., n, D] -> logical planes int64 [..., nblk, D, 4]; bit i of planes[b, j, p]
    is bit p (0 = MSB) of token 64b+i's code (kernels/bitplane.py:44-50)."""
    require_cuda(code)
    *lead, n, d = code.shape
    if d != D or code.dtype != torch.uint8:
        raise ValueError("pack_planes: codes must be uint8 [..., n, 128]")
    cc = code.reshape(-1, n, d).contiguous()
    BH, nb = cc.shape[0], _nblk(n)
    planes = torch.empty(BH, nb, d, 4, dtype=torch.int64, device=code.device)
    check(lib().fathom_pack_codes(ptr(cc), BH, n, 1, ptr(planes), stream_of(code.device)), "pack_planes")
    return planes.view(*lead, nb, d, 4)


def unpack_planes(planes, n):
    """Inverse of pack_planes: int64 [..., nblk, D, 4] -> codes uint8 [..., n, D] (kernels/bitplane.py:52-58)."""
    require_cuda(planes)
    *lead, nb, d, four = planes.shape
    if d != D or four != 4 or nb != _nblk(n):
        raise ValueError("unpack_planes: planes must be [..., ceil(n/64), 128, 4]")
    pc = planes.reshape(-1, nb, d, 4).contiguous()
    code = torch.empty(pc.shape[0], n, d, dtype=torch.uint8, device=planes.device)
    check(lib().fathom_unpack_planes(ptr(pc), pc.shape[0], n, 1, ptr(code), stream_of(planes.device)),
          "unpack_planes")
    return code.view(*lead, n, d)


def to_superblocks(planes, scales):
    """Logical [..., nblk, D, 4] / [..., nblk, D] -> kernel order [..., nsb, D, 4, SUB] int64 /
    [..., nsb, D, SUB] fp16, padded to whole superblocks (kernels/bitplane.py:60-65).
    Uses the module global SUB, as the reference does."""
    require_cuda(planes, scales)
    if scales.dtype != torch.float16:
        raise TypeError("to_superblocks: scales must be float16 (the store's scale dtype)")
    *lead, nb, d, _ = planes.shape
    sub = SUB
    nsb = math.ceil(nb / sub)
    pc = planes.reshape(-1, nb, d, 4).contiguous()
    sc = scales.reshape(-1, nb, d).contiguous()
    BH = pc.shape[0]
    pk = torch.empty(BH, nsb, d, 4, sub, dtype=torch.int64, device=planes.device)
    sk = torch.empty(BH, nsb, d, sub, dtype=torch.float16, device=planes.device)
    check(lib().fathom_relayout(ptr(pc), ptr(sc), BH, nb, 1, ptr(pk), ptr(sk), sub, stream_of(planes.device)),
          "to_superblocks")
    return pk.view(*lead, nsb, d, 4, sub), sk.view(*lead, nsb, d, sub)


def bytes_planes(t, n):
    """Bytes a scan moves for plans t [BH, D] over n tokens: sum_j 8*t_j + 2*#active per 64-token block
    (kernels/bitplane.py:76-78).  Returns a Python float (synchronises)."""
    nb = _nblk(n)
    return float(((t.float().sum(-1) * 8 + (t > 0).float().sum(-1) * 2) * nb).sum())


# ------------------------------------------------------------------ dense reference helpers
def _scales_arg(scales):
    if scales.dtype == torch.float16:
        return scales.contiguous(), 0
    return scales.contiguous().float(), 1


def dequant_planes(code, scales, t):
    """Dequantisation of the top-t planes: code uint8 [..., n, D], scales [..., nblk, D] (fp16 or fp32),
    t a depth (int), depths [D], or per-row depths [..., D] -> fp32 [..., n, D] with
    ((c >> (4-t)) + 0.5 - 2^(t-1)) * s / 2^(t-1), 0 where t == 0 (kernels/bitplane.py:34-42)."""
    require_cuda(code, scales)
    *lead, n, d = code.shape
    if d != D or code.dtype != torch.uint8:
        raise ValueError("dequant_planes: codes must be uint8 [..., n, 128]")
    rows = math.prod(lead) if lead else 1
    sc, sf32 = _scales_arg(scales)
    if tuple(sc.shape) != (*lead, _nblk(n), D):
        raise ValueError(f"dequant_planes: scales must be [..., {_nblk(n)}, {D}]")
    tt = torch.as_tensor(t, device=code.device).to(torch.int32)
    if tt.dim() == 0:
        tt = tt.expand(D)
    if tt.dim() == 1:
        stride = 0
    elif tuple(tt.shape) == (*lead, D):
        stride = D
    else:
        raise ValueError("dequant_planes: t must be a scalar, [128] or [..., 128] matching the codes")
    tt = tt.contiguous()
    out = torch.empty(*lead, n, D, dtype=torch.float32, device=code.device)
    check(lib().fathom_dequant_planes(ptr(code.contiguous()), ptr(sc), sf32, rows, n, ptr(tt), stride, ptr(out),
                                      stream_of(code.device)), "dequant_planes")
    return out


def _ref_scan_args(q, code, scales):
    require_cuda(q, code, scales)
    BH, G, d = q.shape
    if d != D or code.dim() != 3 or code.shape[0] != BH or code.shape[2] != D or code.dtype != torch.uint8:
        raise ValueError("scan reference: q [BH, G, 128] and codes uint8 [BH, n, 128] expected")
    n = code.shape[1]
    sc, sf32 = _scales_arg(scales)
    if tuple(sc.shape) != (BH, _nblk(n), D):
        raise ValueError(f"scan reference: scales must be [BH, {_nblk(n)}, {D}]")
    out = torch.empty(BH, G, n, dtype=torch.float32, device=q.device)
    return BH, G, n, q.contiguous().float(), code.contiguous(), sc, sf32, out


def scan_planes_reference(q, code, scales, t):
    """Dense scan of the plane semantics: q [BH, G, D] against dequant_planes(code[b], scales[b], t[b]) for
    codes uint8 [BH, n, D], scales [BH, nblk, D] and depths t [BH, D] -> fp32 [BH, G, n]
    (kernels/bitplane.py:357-363)."""
    BH, G, n, qc, cc, sc, sf32, out = _ref_scan_args(q, code, scales)
    tt = torch.as_tensor(t, device=q.device).to(torch.int32).expand(BH, D).contiguous()
    check(lib().fathom_scan_planes_reference(ptr(qc), BH, G, n, ptr(cc), ptr(sc), sf32, ptr(tt), ptr(out),
                                             stream_of(q.device)), "scan_planes_reference")
    return out


def scan_chan4_reference(q, code, scales, active):
    """Dense scan of the comparator semantics: every channel at 4 bits times its active flag (active bool
    [BH, D]) against q [BH, G, D] -> fp32 [BH, G, n] (kernels/bitplane.py:365-370)."""
    BH, G, n, qc, cc, sc, sf32, out = _ref_scan_args(q, code, scales)
    act = torch.as_tensor(active, device=q.device).to(torch.uint8).expand(BH, D).contiguous()
    check(lib().fathom_scan_chan4_reference(ptr(qc), BH, G, n, ptr(cc), ptr(sc), sf32, ptr(act), ptr(out),
                                            stream_of(q.device)), "scan_chan4_reference")
    return out


# ------------------------------------------------------------------ plan
_BUDGETS = {}


def _budget_tensor(value, BH, dev):
    """A [BH] fp32 tensor holding a scalar budget, kept per (device, BH, value) so a decode loop does not
    launch a fill kernel per call.  A tensor first needed while a CUDA graph is being captured is made
    fresh for that graph (which then owns it) and not kept."""
    key = (dev.index if dev.index is not None else torch.cuda.current_device(), BH, value)
    t = _BUDGETS.get(key)
    if t is None:
        if torch.cuda.is_current_stream_capturing():
            return torch.full((BH,), value, device=dev)
        if len(_BUDGETS) > 256:
            _BUDGETS.clear()
        t = _BUDGETS[key] = torch.full((BH,), value, device=dev)
    return t


def make_plan(g, budget, bmax=4, iters=30):
    """g [BH, D] fp32 group-summed gain q_j^2 Var(k_j); budget scalar or [BH] (bits per token).
    Returns dict of device tensors t int8 [BH,D], pairs int32 [BH,D*bmax], npairs [BH], act [BH,D],
    nact [BH], cls [BH,bmax,D], clsn [BH,bmax] (kernels/bitplane.py:108-116)."""
    require_cuda(g)
    BH, d = g.shape
    if d != D:
        raise ValueError(f"make_plan: g must be [BH, {D}]")
    dev = g.device
    if not torch.is_tensor(budget):
        budget = _budget_tensor(float(budget), BH, dev)
    budget = budget.to(device=dev, dtype=torch.float32).reshape(-1).expand(BH).contiguous()
    gc = g.contiguous().float()
    t = torch.empty(BH, d, dtype=torch.int8, device=dev)
    pairs = torch.empty(BH, d * bmax, dtype=torch.int32, device=dev)
    npairs = torch.empty(BH, dtype=torch.int32, device=dev)
    act = torch.empty(BH, d, dtype=torch.int32, device=dev)
    nact = torch.empty(BH, dtype=torch.int32, device=dev)
    cls = torch.empty(BH, bmax, d, dtype=torch.int32, device=dev)
    clsn = torch.empty(BH, bmax, dtype=torch.int32, device=dev)
    check(lib().fathom_make_plan(ptr(gc), ptr(budget), BH, bmax, iters, ptr(t), ptr(pairs), ptr(npairs), ptr(act),
                                 ptr(nact), ptr(cls), ptr(clsn), stream_of(dev)), "make_plan")
    return {"t": t, "pairs": pairs, "npairs": npairs, "act": act, "nact": nact, "cls": cls, "clsn": clsn}


def make_plan_torch(g, budget, bmax=4, iters=30):
    """The water-filling depths alone, as float [BH, D] (kernels/bitplane.py:118-126): the same bisection
    (lo = -60, hi = 60, `iters` halvings, round half to even, clip to 0..bmax) as make_plan, whose
    depths it returns."""
    return make_plan(g, budget, bmax, iters)["t"].float()


# ------------------------------------------------------------------ store + scan
class PlaneStore:
    """K [BH, n, D] (any float dtype) -> superblock-ordered bit-plane store on the same device
    (kernels/bitplane.py:310-340).  One fused kernel quantises, packs and orders the store.

    Attributes as the reference: BH, n, nsb, planes_k [BH,nsb,D,4,SUB] int64, scales_k
    [BH,nsb,D,SUB] fp16, planes32 (int32 view), code / scales_blk (decoded on first access).
    The class attributes kernel / cls_cfg / fma_cfg are accepted for compatibility; every
    setting runs the same CUDA scan (the reference's cls and fma kernels compute the same sums).
    """
    kernel = "cls"
    fma_cfg = {"NB": 2, "KK": 8, "num_warps": 1, "num_stages": 1}
    cls_cfg = {"NB": 4, "KK": 4, "num_warps": 1, "num_stages": 1}

    def __init__(self, K, scale_dtype=torch.float16, basis=None):
        """basis: an optional KLT basis (fathom_b200.klt.KLTBasis: mu [BH,D], Vt [BH,D,D], lam [BH,D]).
        Given one, the store holds the planes of (K - mu) @ Vt -- the planesK store of
        scripts/R_ruler.py:63-64 -- built by one fused rotate + quantise + pack kernel, and scans take the
        rotated queries q @ Vt (fathom_b200.klt.klt_query)."""
        require_cuda(K)
        self.BH, self.n, d = K.shape
        assert d == D
        if K.dtype not in _lib.DTYPE_CODE:
            K = K.float()
        if scale_dtype not in (torch.float16, torch.float32):
            raise TypeError("PlaneStore: scale_dtype must be torch.float16 or torch.float32")
        self.basis = None if basis is None else basis.checked(self.BH, K.device)
        self.sub = SUB
        nb = _nblk(self.n)
        self.nsb = math.ceil(nb / self.sub)
        dev = K.device
        Kc = K if K.stride(-1) == 1 and K.stride(-2) == D else K.contiguous()
        self.planes_k = torch.empty(self.BH, self.nsb, D, 4, self.sub, dtype=torch.int64, device=dev)
        self.scales_k = torch.empty(self.BH, self.nsb, D, self.sub, dtype=torch.float16, device=dev)
        self._scale_dtype = scale_dtype
        self._scales_blk = None
        if scale_dtype == torch.float32:        # fp32 absmax is not recoverable from the fp16 store
            self._scales_blk = torch.empty(self.BH, nb, D, dtype=torch.float32, device=dev)
        if self.basis is None:
            check(lib().fathom_quantise_pack(ptr(Kc), _lib.DTYPE_CODE[Kc.dtype], self.BH, self.n, Kc.stride(0),
                                             self.sub, int(scale_dtype == torch.float16), None, ptr(self._scales_blk),
                                             int(scale_dtype == torch.float32), ptr(self.planes_k), ptr(self.scales_k),
                                             stream_of(dev)), "PlaneStore")
        else:
            check(lib().fathom_klt_quantise_pack(ptr(Kc), _lib.DTYPE_CODE[Kc.dtype], self.BH, self.n, Kc.stride(0),
                                                 ptr(self.basis.mu), ptr(self.basis.Vt), self.sub,
                                                 int(scale_dtype == torch.float16), None, ptr(self._scales_blk),
                                                 int(scale_dtype == torch.float32), ptr(self.planes_k),
                                                 ptr(self.scales_k), None, stream_of(dev)), "PlaneStore(basis)")
        self.planes32 = self.planes_k.view(torch.int32)
        self._code = None

    @property
    def code(self):
        """uint8 [BH, n, D] codes, decoded from the planes on first access."""
        if self._code is None:
            dev = self.planes_k.device
            self._code = torch.empty(self.BH, self.n, D, dtype=torch.uint8, device=dev)
            check(lib().fathom_unpack_planes(ptr(self.planes_k), self.BH, self.n, self.sub, ptr(self._code),
                                             stream_of(dev)), "PlaneStore.code")
        return self._code

    @code.setter
    def code(self, v):
        self._code = v

    @property
    def scales_blk(self):
        """Block scales [BH, nblk, D] in the store's scale dtype."""
        if self._scales_blk is None:
            dev = self.scales_k.device
            nb = _nblk(self.n)
            sb = torch.empty(self.BH, nb, D, dtype=torch.float16, device=dev)
            check(lib().fathom_relayout(None, ptr(self.scales_k), self.BH, nb, self.sub, None, ptr(sb), 1,
                                        stream_of(dev)), "PlaneStore.scales_blk")
            self._scales_blk = sb
        return self._scales_blk

    @scales_blk.setter
    def scales_blk(self, v):
        self._scales_blk = v

    def scan(self, q, plan, out=None, blocks=None):
        """q [BH, G, D] fp32, plan from make_plan -> scores fp32 [BH, G, n]; blocks=(b0, b1) scans only
        64-token blocks [b0, b1) (kernels/bitplane.py:319-338)."""
        require_cuda(q)
        BH, G, d = q.shape
        assert BH == self.BH
        dev = q.device
        out = torch.empty(BH, G, self.n, device=dev, dtype=torch.float32) if out is None else out
        nb = _nblk(self.n)
        b0, b1 = (0, nb) if blocks is None else blocks
        sub = getattr(self, "sub", None) or SUB
        qc = q.contiguous().float()
        cls, clsn = plan["cls"], plan["clsn"]
        check(lib().fathom_scan(ptr(qc), BH, G, self.n, sub, ptr(cls), ptr(clsn), cls.shape[1], ptr(self.planes32),
                                ptr(self.scales_k), b0, b1, ptr(out), stream_of(dev)), "PlaneStore.scan")
        return out

    def nbytes(self):
        return self.planes_k.numel() * 8 + self.scales_k.numel() * 2


# ------------------------------------------------------------------ selection
# ------------------------------------------------------------------ Chan4 comparator store
def pack_chan4(code):
    """codes uint8 [BH, n, D] -> channel-major 4-bit store int32 [BH, nsb, D, SUB, 8]: nibble k of word m
    of a block is the code of token 8m+k of that block (kernels/bitplane.py:67-74; module SUB)."""
    require_cuda(code)
    BH, n, d = code.shape
    if d != D:
        raise ValueError(f"pack_chan4: codes must be [BH, n, {D}]")
    nsb = math.ceil(_nblk(n) / SUB)
    out = torch.empty(BH, nsb, D, SUB, 8, dtype=torch.int32, device=code.device)
    check(lib().fathom_pack_chan4(ptr(code.contiguous().to(torch.uint8)), BH, n, SUB, ptr(out), stream_of(code.device)),
          "pack_chan4")
    return out


def channel_list(active):
    """active bool [BH, D] -> act int32 [BH, D] (active channels ascending, then the inactive ones
    ascending), nact int32 [BH] (kernels/bitplane.py:128-132)."""
    require_cuda(active)
    BH, d = active.shape
    if d != D:
        raise ValueError(f"channel_list: active must be [BH, {D}]")
    a = active.contiguous().to(torch.uint8)
    act = torch.empty(BH, D, dtype=torch.int32, device=active.device)
    nact = torch.empty(BH, dtype=torch.int32, device=active.device)
    check(lib().fathom_channel_list(ptr(a), BH, ptr(act), ptr(nact), stream_of(active.device)), "channel_list")
    return act, nact


def bytes_chan4(nact, n):
    """Bytes a Chan4Store.scan moves: sum_bh nact * (32 + 2) per 64-token block (kernels/bitplane.py:79-80)."""
    return float((nact.float() * (32 + 2) * _nblk(n)).sum())


class Chan4Store:
    """The reference's comparator store (kernels/bitplane.py:342-355): K [BH, n, D] quantised as for
    PlaneStore, kept channel-major at full 4 bits (chan_k [BH, nsb, D, SUB, 8] int32) with the same
    block scales (scales_k [BH, nsb, D, SUB] fp16); scan(q, act, nact) reads the first nact[bh]
    channels of act at 4 bits.  Attributes as the reference: BH, n, code, scales_blk, chan_k,
    scales_k, nsb; the class attribute cfg is accepted and ignored (one CUDA scan serves all)."""
    cfg = {"NB": 2, "KK": 1, "num_warps": 1, "num_stages": 1}

    def __init__(self, K, scale_dtype=torch.float16):
        require_cuda(K)
        self.BH, self.n, d = K.shape
        assert d == D
        if K.dtype not in _lib.DTYPE_CODE:
            K = K.float()
        if scale_dtype not in (torch.float16, torch.float32):
            raise TypeError("Chan4Store: scale_dtype must be torch.float16 or torch.float32")
        self.sub = SUB
        nb = _nblk(self.n)
        self.nsb = math.ceil(nb / self.sub)
        dev = K.device
        Kc = K if K.stride(-1) == 1 and K.stride(-2) == D else K.contiguous()
        self.code = torch.empty(self.BH, self.n, D, dtype=torch.uint8, device=dev)
        self.scales_blk = torch.empty(self.BH, nb, D, dtype=scale_dtype, device=dev)
        self.scales_k = torch.empty(self.BH, self.nsb, D, self.sub, dtype=torch.float16, device=dev)
        planes = torch.empty(self.BH, self.nsb, D, 4, self.sub, dtype=torch.int64, device=dev)   # construction only
        check(lib().fathom_quantise_pack(ptr(Kc), _lib.DTYPE_CODE[Kc.dtype], self.BH, self.n, Kc.stride(0), self.sub,
                                         int(scale_dtype == torch.float16), ptr(self.code), ptr(self.scales_blk),
                                         int(scale_dtype == torch.float32), ptr(planes), ptr(self.scales_k),
                                         stream_of(dev)), "Chan4Store")
        del planes
        self.chan_k = torch.empty(self.BH, self.nsb, D, self.sub, 8, dtype=torch.int32, device=dev)
        check(lib().fathom_pack_chan4(ptr(self.code), self.BH, self.n, self.sub, ptr(self.chan_k), stream_of(dev)),
              "Chan4Store")

    def scan(self, q, act, nact, out=None, blocks=None):
        """q [BH, G, D] fp32 -> scores fp32 [BH, G, n] over the listed channels at 4 bits; blocks=(b0, b1)
        restricts the written range (kernels/bitplane.py:346-352)."""
        require_cuda(q, act, nact)
        BH, G, d = q.shape
        dev = q.device
        out = torch.empty(BH, G, self.n, device=dev, dtype=torch.float32) if out is None else out
        b0, b1 = (0, _nblk(self.n)) if blocks is None else blocks
        qc = q.contiguous().float()
        check(lib().fathom_scan_chan4(ptr(qc), BH, G, self.n, self.sub, ptr(act.contiguous().to(torch.int32)),
                                      ptr(nact.contiguous().to(torch.int32)), ptr(self.chan_k), ptr(self.scales_k),
                                      b0, b1, ptr(out), stream_of(dev)), "Chan4Store.scan")
        return out

    def nbytes(self):
        return self.chan_k.numel() * 4 + self.scales_k.numel() * 2


def sink_local_topk(scores, k, sink=4, local=32):
    """scores [BH, G, n] -> selected indices int64 [BH, G, k] = top-(k - sink - local) among the
    non-sink / non-local tokens (score descending, ties by index ascending), then 0..sink-1, then the
    last `local` tokens (kernels/bitplane.py:372-378)."""
    require_cuda(scores)
    *lead, n = scores.shape
    sc = scores.reshape(-1, n).contiguous().float()
    rows = sc.shape[0]
    dev = scores.device
    idx = torch.empty(rows, k, dtype=torch.int64, device=dev)
    nbytes = lib().fathom_select_workspace_bytes(rows, n, k - sink - local)
    ws = _lib.workspace(dev, nbytes, "select")
    check(lib().fathom_sink_local_topk(ptr(sc), rows, n, k, sink, local, ptr(idx), ptr(ws), ws.numel(),
                                       stream_of(dev)), "sink_local_topk")
    return idx.view(*lead, k)


def select_topk(scores, kk, mask_lo=0, mask_hi=None, index_offset=0, with_scores=False):
    """Top-kk of each row of scores [..., n] with tokens outside [mask_lo, mask_hi) excluded, ordered by
    (score desc, index asc); indices shifted by index_offset.  Returns idx int64 [..., kk] (and the
    selected scores fp32 [..., kk] if with_scores)."""
    require_cuda(scores)
    *lead, n = scores.shape
    mask_hi = n if mask_hi is None else mask_hi
    sc = scores.reshape(-1, n).contiguous().float()
    rows = sc.shape[0]
    dev = scores.device
    idx = torch.empty(rows, kk, dtype=torch.int64, device=dev)
    vals = torch.empty(rows, kk, dtype=torch.float32, device=dev) if with_scores else None
    ws = _lib.workspace(dev, lib().fathom_select_workspace_bytes(rows, n, kk), "select")
    check(lib().fathom_select_topk(ptr(sc), rows, n, n, kk, mask_lo, mask_hi, index_offset, ptr(idx), kk, ptr(vals),
                                   ptr(ws), ws.numel(), stream_of(dev)), "select_topk")
    if with_scores:
        return idx.view(*lead, kk), vals.view(*lead, kk)
    return idx.view(*lead, kk)


def merge_topk(cand_scores, cand_idx, kk):
    """Final top-kk of candidate lists [..., m] (scores fp32, global int64 indices) in the (score desc,
    index asc) order.  Returns (idx int64 [..., kk], scores fp32 [..., kk])."""
    require_cuda(cand_scores, cand_idx)
    *lead, m = cand_scores.shape
    cs = cand_scores.reshape(-1, m).contiguous().float()
    ci = cand_idx.reshape(-1, m).contiguous().to(torch.int64)
    rows = cs.shape[0]
    dev = cs.device
    idx = torch.empty(rows, kk, dtype=torch.int64, device=dev)
    vals = torch.empty(rows, kk, dtype=torch.float32, device=dev)
    check(lib().fathom_merge_topk(ptr(cs), ptr(ci), rows, m, kk, ptr(idx), ptr(vals), stream_of(dev)), "merge_topk")
    return idx.view(*lead, kk), vals.view(*lead, kk)


# ------------------------------------------------------------------ scan + selection in one call
def scan_select(store, q, plan, kk, mask_lo=0, mask_hi=None, index_offset=0, append_sink=0, append_local=0,
                scores=None, with_scores=False, scan_done_event=None, idx_out=None):
    """store.scan(q, plan) and the top-kk selection of its rows in one library call.  Returns
    (idx int64 [BH, G, kk+append_sink+append_local], vals fp32 [BH, G, kk] or None, scores fp32 [BH, G, n]).
    scan_done_event (torch.cuda.Event) is recorded right after the scan kernel.  idx_out: an int64
    [BH, G, W] CUDA tensor (W >= the width) to write the indices into (its first columns); returned."""
    require_cuda(q)
    BH, G, d = q.shape
    assert BH == store.BH
    dev = q.device
    n = store.n
    mask_hi = n if mask_hi is None else mask_hi
    scores = torch.empty(BH, G, n, device=dev, dtype=torch.float32) if scores is None else scores
    width = kk + append_sink + append_local
    if idx_out is None:
        idx = torch.empty(BH, G, width, device=dev, dtype=torch.int64)
    else:
        idx = idx_out
        if (idx.dtype != torch.int64 or idx.device != dev or idx.dim() != 3 or tuple(idx.shape[:2]) != (BH, G)
                or idx.shape[2] < width or not idx.is_contiguous()):
            raise ValueError(f"scan_select: idx_out must be contiguous int64 [{BH}, {G}, >= {width}] on {dev}")
    vals = torch.empty(BH, G, kk, device=dev, dtype=torch.float32) if with_scores else None
    ws = _lib.workspace(dev, lib().fathom_scan_select_workspace_bytes(BH, G, n, kk), "select")
    sub = getattr(store, "sub", None) or SUB
    qc = q.contiguous().float()
    cls, clsn = plan["cls"], plan["clsn"]
    check(lib().fathom_scan_select(ptr(qc), BH, G, n, sub, ptr(cls), ptr(clsn), cls.shape[1], ptr(store.planes32),
                                   ptr(store.scales_k), kk, mask_lo, mask_hi, index_offset, append_sink, append_local,
                                   ptr(scores), ptr(idx), idx.shape[2], ptr(vals), ptr(ws), ws.numel(),
                                   scan_done_event.cuda_event if scan_done_event is not None else None,
                                   stream_of(dev)),
          "scan_select")
    return idx, vals, scores


def scan_topk(store, q, plan, k, sink=4, local=32, scores=None, scan_done_event=None):
    """sink_local_topk(store.scan(q, plan), k, sink, local) in one call; int64 [BH, G, k]."""
    idx, _, _ = scan_select(store, q, plan, k - sink - local, mask_lo=sink, mask_hi=store.n - local,
                            append_sink=sink, append_local=local, scores=scores, scan_done_event=scan_done_event)
    return idx
