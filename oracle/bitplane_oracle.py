"""CPU oracle for the Fathom key-scan path -- TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, the algorithm of the reference module
`kernels/bitplane.py` and of the decode-step tail of `scripts/B_e2e_offload_v2.py`.
It exists to check the CUDA path; nothing in the product package imports it.
Only `tests/`, `__graft_entry__.smoke()` and the CPU-baseline leg of `bench.py`
may use it.

Parity pin: `tests/golden/make_golden.py` imports the real reference (torch, CPU)
and writes fixtures; `tests/test_oracle.py` checks every function here against
them (bit-exact for codes, planes, scales and plans; index sets for top-k;
fp32 tolerance for scores).

Conventions follow the reference:
  * K is [..., n, D] float32 (bf16 inputs are widened exactly first);
  * one 64-token block (BLK) per scale; D = 128 in the store, any D here;
  * bit p of a 4-bit code is plane p, p = 0 is the MSB; bit i of a plane word
    is token 64*b + i of block b (least significant bit first).
"""
import math

import numpy as np

BLK = 64          # tokens per block          (kernels/bitplane.py:19)
SUB_HBM = 16      # blocks per superblock in HBM order (kernels/bitplane.py:19)
BMAX = 4          # planes per channel         (kernels/bitplane.py:108)


def nblocks(n):
    return (n + BLK - 1) // BLK


# ---------------------------------------------------------------- store build
def quantise_u4(K, scale_dtype="f16"):
    """kernels/bitplane.py:23-32.  K [..., n, D] float32 -> (code u8 [..., n, D], scales [..., nblk, D]).

    amax per (block, channel), clamped to >= 1e-8, rounded to fp16; s = amax/8;
    code = clamp(floor(x / s), -8, 7) + 8.  Pad tokens are zero.  A NaN
    quotient (0/0 when the fp16 amax underflows to 0) gives code 0, which is
    what torch's NaN -> uint8 conversion yields on the reference's CPU path.
    """
    K = np.asarray(K, dtype=np.float32)
    *lead, n, d = K.shape
    nb = nblocks(n)
    cb = np.zeros((*lead, nb * BLK, d), np.float32)
    cb[..., :n, :] = K
    cb = cb.reshape(*lead, nb, BLK, d)
    amax = np.maximum(np.abs(cb).max(axis=-2, keepdims=True), np.float32(1e-8))
    with np.errstate(over="ignore"):
        amax16 = amax.astype(np.float16)
    if scale_dtype == "f32":                      # scale_dtype=torch.float32: codes from the fp32 absmax
        s = amax / np.float32(8.0)
    else:
        s = amax16.astype(np.float32) / np.float32(8.0)
    with np.errstate(divide="ignore", invalid="ignore"):
        qv = cb / s
    fl = np.clip(np.floor(qv), -8, 7) + 8
    code = np.where(np.isnan(qv), 0, fl).astype(np.uint8)
    code = code.reshape(*lead, nb * BLK, d)[..., :n, :]
    return code, (amax[..., 0, :] if scale_dtype == "f32" else amax16[..., 0, :])


def pack_planes(code):
    """kernels/bitplane.py:44-50.  code u8 [..., n, D] -> planes uint64 [..., nblk, D, 4]."""
    code = np.asarray(code, dtype=np.uint8)
    *lead, n, d = code.shape
    nb = nblocks(n)
    cb = np.zeros((*lead, nb * BLK, d), np.uint8)
    cb[..., :n, :] = code
    cb = cb.reshape(*lead, nb, BLK, d)
    out = np.zeros((*lead, nb, d, 4), np.uint64)
    for p in range(4):
        bits = ((cb >> (3 - p)) & 1).astype(np.uint8)                 # [..., nb, 64, d]
        packed = np.packbits(bits, axis=-2, bitorder="little")         # [..., nb, 8, d] bytes, token i -> bit i
        words = np.ascontiguousarray(np.moveaxis(packed, -2, -1)).view("<u8")[..., 0]  # [..., nb, d]
        out[..., p] = words
    return out


def unpack_planes(planes, n):
    """kernels/bitplane.py:52-58.  planes uint64 [..., nblk, D, 4] -> code u8 [..., n, D]."""
    planes = np.asarray(planes).view(np.uint64)
    *lead, nb, d, _ = planes.shape
    code = np.zeros((*lead, nb, BLK, d), np.uint8)
    for p in range(4):
        by = np.ascontiguousarray(planes[..., p]).view(np.uint8).reshape(*lead, nb, d, 8)
        bits = np.unpackbits(by, axis=-1, bitorder="little")          # [..., nb, d, 64]
        code |= (np.moveaxis(bits, -1, -2) << (3 - p)).astype(np.uint8)
    return code.reshape(*lead, nb * BLK, d)[..., :n, :]


def to_superblocks(planes, scales, sub=SUB_HBM):
    """kernels/bitplane.py:60-65.  Logical planes [..., nblk, D, 4] / scales [..., nblk, D] ->
    planes_k [..., nsb, D, 4, sub] uint64 and scales_k [..., nsb, D, sub] fp16 (zero padded)."""
    *lead, nb, d, _ = planes.shape
    nsb = (nb + sub - 1) // sub
    pl = np.zeros((*lead, nsb * sub, d, 4), np.uint64)
    pl[..., :nb, :, :] = planes
    pl = pl.reshape(*lead, nsb, sub, d, 4)
    nl = len(lead)
    pl = np.ascontiguousarray(np.transpose(pl, (*range(nl), nl, nl + 2, nl + 3, nl + 1)))
    sc = np.zeros((*lead, nsb * sub, d), np.float16)
    sc[..., :nb, :] = scales
    sc = np.ascontiguousarray(np.swapaxes(sc.reshape(*lead, nsb, sub, d), -1, -2))
    return pl, sc


def from_superblocks(planes_k, scales_k, nb):
    """Inverse of to_superblocks (logical order, first nb blocks)."""
    *lead, nsb, d, four, sub = planes_k.shape
    nl = len(lead)
    pl = np.transpose(planes_k, (*range(nl), nl, nl + 3, nl + 1, nl + 2)).reshape(*lead, nsb * sub, d, four)[..., :nb, :, :]
    sc = np.swapaxes(scales_k, -1, -2).reshape(*lead, nsb * sub, d)[..., :nb, :]
    return np.ascontiguousarray(pl), np.ascontiguousarray(sc)


def bytes_planes(t, n):
    """kernels/bitplane.py:76-78.  Bytes one scan moves: sum_bh (8*sum_j t_j + 2*#active) * nblk."""
    t = np.asarray(t, np.float64)
    return float(((t.sum(-1) * 8 + (t > 0).sum(-1) * 2) * nblocks(n)).sum())


# ---------------------------------------------------------------- Chan4 comparator store
def pack_chan4(code, sub=SUB_HBM):
    """kernels/bitplane.py:67-74.  Codes uint8 [..., n, D] -> channel-major 4-bit store int32
    [..., nsb, D, sub, 8]: nibble k of word m of block s = code of token 64*(sb*sub+s) + 8*m + k
    (zero padded to whole superblocks; two's complement in int32)."""
    code = np.asarray(code, np.uint8)
    *lead, n, d = code.shape
    nb = nblocks(n)
    nsb = (nb + sub - 1) // sub
    cb = np.zeros((*lead, nsb * sub * BLK, d), np.int64)
    cb[..., :n, :] = code
    cb = cb.reshape(*lead, nsb, sub, 8, 8, d)
    k = np.arange(8, dtype=np.int64).reshape(8, 1)
    words = (cb << (4 * k)).sum(-2)                                    # [..., nsb, sub, 8, d]
    words = words.astype(np.uint32).view(np.int32)
    nl = len(lead)
    return np.ascontiguousarray(np.transpose(words, (*range(nl), nl, nl + 3, nl + 1, nl + 2)))


def bytes_chan4(nact, n):
    """kernels/bitplane.py:79-80.  Bytes one chan4 scan moves: sum_bh nact * (32 + 2) * nblk."""
    return float((np.asarray(nact, np.float64) * (32 + 2) * nblocks(n)).sum())


def channel_list(active):
    """kernels/bitplane.py:128-132.  active bool [BH, D] -> act int32 [BH, D] (active channels ascending,
    then the inactive ones ascending) and nact int32 [BH]."""
    active = np.asarray(active, bool)
    order = np.argsort((~active).astype(np.int8), axis=-1, kind="stable")
    return order.astype(np.int32), active.sum(-1).astype(np.int32)


def scan_chan4(q, code, scales, active):
    """kernels/bitplane.py:365-370 (scan_chan4_reference): the full 4-bit dequantised keys of the active
    channels, (c - 7.5) * s / 8, against q [BH, G, D] -> fp32 [BH, G, n]."""
    q = np.asarray(q, np.float32)
    out = np.empty((q.shape[0], q.shape[1], code.shape[-2]), np.float32)
    for b in range(q.shape[0]):
        val = dequant_planes(code[b], scales[b], np.full(code.shape[-1], 4)) * np.asarray(active[b], np.float32)[None]
        out[b] = q[b] @ val.T
    return out


# ---------------------------------------------------------------- plan
def _log2_f32(g):
    """log2 in float32 of max(g, 1e-30), rounded from a double-precision log2."""
    g = np.maximum(np.asarray(g, np.float32), np.float32(1e-30))
    return np.log2(g.astype(np.float64)).astype(np.float32)


def plan_depths(g, budget, bmax=BMAX, iters=30):
    """kernels/bitplane.py:118-126 (make_plan_torch; same bisection as plan_kernel :83-95).

    lo=-60, hi=60; `iters` times: mid=(lo+hi)/2, t=clip(rint((lg-mid)/2),0,bmax),
    lo=mid if sum(t) > budget else hi=mid.  Returns t from hi (float32 [BH, D]).
    All arithmetic in float32, rint = round half to even.
    """
    lg = _log2_f32(g)
    BH = lg.shape[0]
    Br = np.broadcast_to(np.asarray(budget, np.float32).reshape(-1, 1) if np.ndim(budget) else np.float32(budget), (BH, 1))
    lo = np.full((BH, 1), -60.0, np.float32)
    hi = np.full((BH, 1), 60.0, np.float32)
    bf = np.float32(bmax)
    half = np.float32(0.5)
    for _ in range(iters):
        mid = (lo + hi) * half
        t = np.minimum(np.maximum(np.rint((lg - mid) * half), np.float32(0)), bf)
        tot = t.sum(-1, keepdims=True, dtype=np.float32)
        over = tot > Br
        lo = np.where(over, mid, lo)
        hi = np.where(over, hi, mid)
    return np.minimum(np.maximum(np.rint((lg - hi) * half), np.float32(0)), bf).astype(np.float32)


def make_plan(g, budget, bmax=BMAX, iters=30):
    """kernels/bitplane.py:83-116 (plan_kernel + make_plan): depths plus compacted lists.

    t int8 [BH, D]; act: active channels ascending, nact; pairs: ch*4+p for p<t_ch
    in channel order, npairs = sum t; cls[c-1]: channels with t == c ascending,
    clsn.  Unused list tails are zero, as make_plan allocates them with zeros.
    """
    t = plan_depths(g, budget, bmax, iters).astype(np.int32)
    BH, d = t.shape
    out = {"t": t.astype(np.int8),
           "pairs": np.zeros((BH, d * bmax), np.int32), "npairs": np.zeros(BH, np.int32),
           "act": np.zeros((BH, d), np.int32), "nact": np.zeros(BH, np.int32),
           "cls": np.zeros((BH, bmax, d), np.int32), "clsn": np.zeros((BH, bmax), np.int32)}
    for b in range(BH):
        act = np.nonzero(t[b] > 0)[0]
        out["act"][b, :len(act)] = act
        out["nact"][b] = len(act)
        pairs = [ch * bmax + p for ch in range(d) for p in range(t[b, ch])]
        out["pairs"][b, :len(pairs)] = pairs
        out["npairs"][b] = len(pairs)
        for c in range(1, bmax + 1):
            ch = np.nonzero(t[b] == c)[0]
            out["cls"][b, c - 1, :len(ch)] = ch
            out["clsn"][b, c - 1] = len(ch)
    return out


# ---------------------------------------------------------------- scan
def dequant_planes(code, scales, t):
    """kernels/bitplane.py:34-42.  Top-t planes dequantised: (c>>(4-t) + 0.5 - 2^(t-1)) * s / 2^(t-1), 0 where t == 0."""
    code = np.asarray(code)
    n, d = code.shape[-2:]
    nb = nblocks(n)
    cb = np.zeros((*code.shape[:-2], nb * BLK, d), np.int64)
    cb[..., :n, :] = code
    cb = cb.reshape(*code.shape[:-2], nb, BLK, d)
    t = np.asarray(t, np.int64)
    half = (2.0 ** (t.astype(np.float32) - 1)).astype(np.float32)
    ct = (cb >> (4 - np.minimum(t, 4))).astype(np.float32)
    with np.errstate(invalid="ignore"):
        val = (ct + np.float32(0.5) - half) * np.asarray(scales, np.float32)[..., :, None, :] / half
    val = np.where(t > 0, val, np.float32(0)).astype(np.float32)
    return val.reshape(*code.shape[:-2], nb * BLK, d)[..., :n, :]


def scan_scores(q, code, scales, t):
    """kernels/bitplane.py:357-363 (scan_planes_reference): q [BH, G, D] x dequantised keys -> fp32 [BH, G, n]."""
    q = np.asarray(q, np.float32)
    out = np.empty((q.shape[0], q.shape[1], code.shape[-2]), np.float32)
    for b in range(q.shape[0]):
        val = dequant_planes(code[b], scales[b], t[b])
        out[b] = q[b] @ val.T
    return out


def scan_scores_threaded(q, code, scales, t, threads=None, chunk=1 << 15):
    """scan_scores over token chunks on a thread pool (numpy releases the GIL in its array loops and the
    BLAS product), so the restatement uses every host core as the reference's torch path does.  Chunks
    are whole 64-token blocks; each chunk is scan_scores of its tokens and blocks."""
    import os
    from concurrent.futures import ThreadPoolExecutor
    q = np.asarray(q, np.float32)
    n = code.shape[-2]
    chunk = max(BLK, chunk // BLK * BLK)
    out = np.empty((q.shape[0], q.shape[1], n), np.float32)

    def work(c0):
        c1 = min(n, c0 + chunk)
        out[..., c0:c1] = scan_scores(q, code[:, c0:c1], scales[:, c0 // BLK:nblocks(c1)], t)

    with ThreadPoolExecutor(threads or os.cpu_count()) as ex:
        list(ex.map(work, range(0, n, chunk)))
    return out


# ---------------------------------------------------------------- KLT-rotated store (planesK)
def klt_basis(K, skip=16):
    """scripts/R_agent.py:59-63 (self_klt).  Keys [BH, n, D] after the first `skip` tokens (4 * SINK):
    mu = mean, (lam, V) = eigendecomposition of the centred covariance X^T X / m (eigenvalues ascending,
    eigenvectors as columns), lam clamped at 0.  float64; the basis is unique only up to the sign of
    each column (and the order within equal eigenvalues)."""
    X = np.asarray(K, np.float64)[:, skip:]
    mu = X.mean(1)
    Xc = X - mu[:, None]
    C = np.einsum("hnd,hne->hde", Xc, Xc) / X.shape[1]
    lam, V = np.linalg.eigh(C)
    return mu, V, np.maximum(lam, 0.0)


def klt_rotate(K, mu, Vt):
    """scripts/R_ruler.py:63-64: (K - mu) @ Vt per head, in float64 from the fp32 difference (the
    reference's and the CUDA path's fp32 products differ from it by summation rounding only)."""
    X = (np.asarray(K, np.float32) - np.asarray(mu, np.float32)[:, None]).astype(np.float64)
    return np.einsum("hnd,hde->hne", X, np.asarray(Vt, np.float64))


def klt_rotate_bound(K, mu, Vt):
    """|X| @ |Vt| per entry: the scale of the summation error of an fp32 rotation."""
    X = np.abs((np.asarray(K, np.float32) - np.asarray(mu, np.float32)[:, None]).astype(np.float64))
    return np.einsum("hnd,hde->hne", X, np.abs(np.asarray(Vt, np.float64)))


def klt_query(q, Vt, lam):
    """scripts/R_ruler.py:83: qr = q @ Vt (float64, rounded to fp32), gains = sum_g (qr^2 * lam) in
    fp32, element-wise products rounded, g ascending."""
    qr = np.einsum("hgd,hde->hge", np.asarray(q, np.float64), np.asarray(Vt, np.float64)).astype(np.float32)
    lam = np.asarray(lam, np.float32)
    gains = np.zeros(lam.shape, np.float32)
    for g in range(qr.shape[1]):
        gains = gains + (qr[:, g] * qr[:, g]) * lam
    return qr, gains


def allocate_layer_budgets(err, budgets, mean_target):
    """scripts/l4_final_alloc.py:143-154 (allocate): per-layer scan budgets from a calibration table
    err[B][L] (error of layer L at budget B).  Every layer starts at budgets[0]; while the mean budget is
    below mean_target, the layer with the largest error drop per budget unit of its next step (first
    layer on ties; a drop must exceed -1) moves up one step.  Returns {L: budget}."""
    layers = list(next(iter(err.values())).keys())
    idx = {L: 0 for L in layers}
    while sum(budgets[i] for i in idx.values()) / len(layers) < mean_target:
        best, best_L = -1, None
        for L in layers:
            i = idx[L]
            if i + 1 >= len(budgets):
                continue
            d = (err[budgets[i]][L] - err[budgets[i + 1]][L]) / (budgets[i + 1] - budgets[i])
            if d > best:
                best, best_L = d, L
        if best_L is None:
            break
        idx[best_L] += 1
    return {L: budgets[i] for L, i in idx.items()}


# ---------------------------------------------------------------- selection
def topk_desc(scores, kk):
    """Largest kk per row, ordered by (score desc, index asc): the deterministic
    tie-break that the CUDA path and the multi-GPU merge also use."""
    s = np.asarray(scores, np.float32)
    lead = s.shape[:-1]
    s2 = s.reshape(-1, s.shape[-1])
    out = np.empty((s2.shape[0], kk), np.int64)
    idx_all = np.arange(s2.shape[1])
    for r in range(s2.shape[0]):
        row = s2[r]
        if kk < row.size:
            part = np.argpartition(-row, kk - 1)[:kk]
            thr = row[part].min()
            cand = np.nonzero(row >= thr)[0]          # every tie at the threshold
        else:
            cand = idx_all
        order = np.lexsort((cand, -row[cand].astype(np.float64)))
        out[r] = cand[order][:kk]
    return out.reshape(*lead, kk)


def sink_local_topk(scores, k, sink=4, local=32):
    """kernels/bitplane.py:372-378.  Mask the first `sink` and last `local` tokens to -inf,
    take the top (k - sink - local), then append arange(sink) and arange(n-local, n)."""
    s = np.array(scores, np.float32, copy=True)
    n = s.shape[-1]
    s[..., :sink] = -np.inf
    if local > 0:
        s[..., n - local:] = -np.inf
    top = topk_desc(s, k - sink - local)
    fixed = np.concatenate([np.arange(sink), np.arange(n - local, n)]).astype(np.int64)
    return np.concatenate([top, np.broadcast_to(fixed, (*top.shape[:-1], fixed.size))], -1)


def merge_candidates(scores, indices, kk):
    """Final top-kk over candidate (score, global index) lists [..., m] with the
    (score desc, index asc) order: the merge step of a context-sharded scan."""
    s = np.asarray(scores, np.float32)
    i = np.asarray(indices, np.int64)
    lead = s.shape[:-1]
    s2, i2 = s.reshape(-1, s.shape[-1]), i.reshape(-1, i.shape[-1])
    out = np.empty((s2.shape[0], kk), np.int64)
    for r in range(s2.shape[0]):
        order = np.lexsort((i2[r], -s2[r].astype(np.float64)))
        out[r] = i2[r][order][:kk]
    return out.reshape(*lead, kk)


# ---------------------------------------------------------------- rows + attention
def gather_rows(src, idx):
    """scripts/B_e2e_offload_v2.py:73-83.  dst[bh, r] = src[bh, idx[bh, r]]; idx < 0 leaves zeros."""
    src = np.asarray(src)
    idx = np.asarray(idx, np.int64)
    BH, R = idx.shape
    dst = np.zeros((BH, R, src.shape[-1]), src.dtype)
    for b in range(BH):
        ok = idx[b] >= 0
        dst[b, ok] = src[b, idx[b, ok]]
    return dst


def decode_attention(q, K, V, idx, recent_K=None, recent_V=None, n_host=None):
    """scripts/B_e2e_offload_v2.py:226-244 (and the HBM twin scripts/B_kernel_bench.py:26-31).

    q [BH, G, D] fp32; K, V [BH, n_host, D] (rows as fp32 values); idx [BH, G, k].
    Indices >= n_host address the device-resident recent buffers (row idx - n_host).
    Returns softmax(q . K_sel^T / sqrt(D)) . V_sel per query head, fp32 [BH, G, D].
    The reference fetches each unique row of a KV head once; that is a traffic
    optimisation and does not change these values.
    """
    q = np.asarray(q, np.float32)
    BH, G, D = q.shape
    n_host = K.shape[1] if n_host is None else n_host
    out = np.empty((BH, G, D), np.float32)
    for b in range(BH):
        for g in range(G):
            ix = np.asarray(idx[b, g], np.int64)
            host = ix < n_host
            Ks = np.empty((ix.size, D), np.float32)
            Vs = np.empty((ix.size, D), np.float32)
            Ks[host] = np.asarray(K[b], np.float32)[ix[host]]
            Vs[host] = np.asarray(V[b], np.float32)[ix[host]]
            if (~host).any():
                Ks[~host] = np.asarray(recent_K[b], np.float32)[ix[~host] - n_host]
                Vs[~host] = np.asarray(recent_V[b], np.float32)[ix[~host] - n_host]
            s = (Ks @ q[b, g]) * np.float32(D ** -0.5)
            s = s - s.max()
            p = np.exp(s.astype(np.float64)).astype(np.float32)
            p /= p.sum(dtype=np.float32)
            out[b, g] = p @ Vs
    return out


def bf16_to_f32(u16):
    """bf16 bit patterns (uint16) -> float32 values (exact)."""
    return (np.asarray(u16, np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x):
    """float32 -> bf16 bit patterns, round to nearest even (as torch's .to(torch.bfloat16))."""
    u = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    nan = np.isnan(np.asarray(x, np.float32))
    return np.where(nan, 0x7FC0, rounded).astype(np.uint16)
