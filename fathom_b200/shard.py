"""Context-sharded decode step: one process per GPU, the context split into contiguous chunks.

No counterpart in the reference (it runs on one GPU).  Each rank holds the bit-plane index and the
K/V rows of its chunk (tokens [lo, hi) of n_total) in its own host memory and scans them through its
own host link.  Per layer:

  1 plan            identical on every rank (same query and gains)
  2 scan            the rank's chunk
  3 local select    top-kk of the chunk with the global sink window masked on the rank that holds
                    it and the global local window masked on the rank(s) that hold it; indices are
                    global (chunk offset added); the selected scores are kept
  4 all-gather      (score, index) candidates of every rank (NCCL over NVLink)
  5 merge           top-kk of the union in (score desc, index asc) order: the global top-kk is
                    contained in the union of the local top-kk's, so the result equals a single-GPU
                    selection over the whole context, bit for bit
  6 attention       each rank attends over the final picks it owns (partial max / sum-exp /
                    unnormalised output), an all-gather of the partials, and a log-sum-exp combine

Chunk boundaries are multiples of 64 tokens, so every chunk's block scales equal those of the
single-GPU store.  The per-rank kernels and the collective are parameters so that the host logic
can be exercised with CPU ranks (gloo) and the CPU oracle.
"""
import torch

BLK = 64


def chunk_bounds(n_total, world, align=BLK):
    """Contiguous [lo, hi) per rank; interior boundaries are multiples of `align`."""
    nb = -(-n_total // align)
    cuts = [0] + [min(n_total, (nb * r // world) * align) for r in range(1, world)] + [n_total]
    return [(cuts[r], cuts[r + 1]) for r in range(world)]


def local_window(lo, hi, n_total, sink, local):
    """Chunk-local [mask_lo, mask_hi): the tokens of [lo, hi) outside the global sink and local windows."""
    n = hi - lo
    mask_lo = min(max(sink - lo, 0), n)
    mask_hi = min(max(n_total - local - lo, 0), n)
    return mask_lo, max(mask_hi, mask_lo)


def fixed_indices(n_total, sink, local, device=None):
    return torch.cat([torch.arange(sink, device=device), torch.arange(n_total - local, n_total, device=device)])


def all_gather(t, group=None):
    """[W, *t.shape] of every rank's t (NCCL: one all_gather_into_tensor; gloo: list all_gather)."""
    import torch.distributed as dist
    W = dist.get_world_size(group)
    if dist.get_backend(group) == "nccl":
        out = torch.empty((W, *t.shape), dtype=t.dtype, device=t.device)
        dist.all_gather_into_tensor(out, t.contiguous(), group=group)
        return out
    parts = [torch.empty_like(t) for _ in range(W)]
    dist.all_gather(parts, t.contiguous(), group=group)
    return torch.stack(parts)


def sharded_select(scores, kk, lo, hi, n_total, sink, local, select_fn=None, merge_fn=None, gather_fn=None):
    """Global top-kk indices [BH, G, kk] (int64, global) of a context-sharded score row set.

    scores [BH, G, hi-lo] are this rank's chunk (or anything select_fn accepts).
    select_fn(scores, kk, mask_lo, mask_hi, offset) -> (idx, vals); merge_fn(vals [..., m], idx [..., m],
    kk) -> idx; gather_fn(t) -> [W, *t.shape]."""
    if select_fn is None:
        from .bitplane import select_topk
        select_fn = lambda s, k, a, b, off: select_topk(s, k, mask_lo=a, mask_hi=b, index_offset=off,
                                                        with_scores=True)
    mlo, mhi = local_window(lo, hi, n_total, sink, local)
    idx, vals = select_fn(scores, kk, mlo, mhi, lo)
    return merge_shards(idx, vals, kk, merge_fn, gather_fn)


def merge_shards(idx, vals, kk, merge_fn=None, gather_fn=None):
    """All-gather of every rank's local (idx, vals) [BH, G, kk] and the merge to the global top-kk."""
    if merge_fn is None:
        from .bitplane import merge_topk
        merge_fn = lambda v, i, k: merge_topk(v, i, k)[0]
    gather_fn = gather_fn or all_gather
    BH, G, _ = idx.shape
    packed = torch.stack([vals.float().view(torch.int32), idx.to(torch.int32)])      # one collective
    allp = gather_fn(packed)                                                        # [W, 2, BH, G, kk]
    W = allp.shape[0]
    cv = allp[:, 0].view(torch.float32).permute(1, 2, 0, 3).reshape(BH, G, W * kk)
    ci = allp[:, 1].to(torch.int64).permute(1, 2, 0, 3).reshape(BH, G, W * kk)
    return merge_fn(cv, ci, kk)


def concurrent_probe(probe, rounds=5, group=None, sync=None):
    """Runs probe() -> (bytes, seconds) on every rank at the same time, `rounds` times, each round started
    by a barrier (and `sync`, e.g. a device synchronise).  Returns (aggregate, per_rank): the best
    round's sum of bytes over its slowest rank's time, and each rank's own bytes / seconds in that
    round.  All ranks take the same collective steps."""
    import torch.distributed as dist
    best = None
    for _ in range(rounds):
        if sync:
            sync()
        dist.barrier(group=group)
        nbytes, sec = probe()
        t = torch.tensor([float(nbytes), float(sec)], dtype=torch.float64)
        allv = all_gather(t.to(_collective_device(group)), group).cpu()
        agg = float(allv[:, 0].sum() / allv[:, 1].max())
        if best is None or agg > best[0]:
            best = (agg, [float(b / s) for b, s in allv.tolist()])
    return best


def _collective_device(group=None):
    import torch.distributed as dist
    if dist.get_backend(group) == "nccl":
        return torch.device("cuda", torch.cuda.current_device())
    return torch.device("cpu")


def merged_equals_single(scores, top, n_total, kk, sink, local, select_fn=None, gather_fn=None):
    """Checks a merged context-sharded selection against one selection over the whole context.

    scores [BH, G, c] is this rank's chunk of the context's scores (equal chunks, rank order = context
    order), top [BH, G, kk] the merged global indices.  The chunks are all-gathered into the full rows,
    the top-kk of tokens [sink, n_total - local) is selected once, and the result is compared with `top`
    (order included).  Per-token scores do not depend on the chunking (block-aligned chunks keep every
    block's scale), so the full rows are exactly what a single-GPU scan of the context gives."""
    if select_fn is None:
        from .bitplane import select_topk
        select_fn = lambda s, k, a, b: select_topk(s, k, mask_lo=a, mask_hi=b)
    gather_fn = gather_fn or all_gather
    parts = gather_fn(scores.contiguous())                  # [W, BH, G, c]
    full = parts.permute(1, 2, 0, 3).reshape(scores.shape[0], scores.shape[1], -1)
    assert full.shape[-1] == n_total, (full.shape, n_total)
    single = select_fn(full, kk, sink, n_total - local)
    return bool(torch.equal(single.to(top.device).to(torch.int64), top.to(torch.int64)))


def sharded_decode_step(a, layers, kv, scores, outs, rank, world, q_in=None, g_in=None, scan_events=None):
    """One decode step over all layers on a context-sharded index (see the module docstring).
    `layers[L].store` holds this rank's chunk of a.ctx tokens; the context has a.ctx * world tokens."""
    from . import bitplane as bp
    from . import offload as off
    n_total = a.ctx * world
    lo, hi = rank * a.ctx, (rank + 1) * a.ctx
    for L, lay in enumerate(layers):
        q = lay.q if q_in is None else q_in[L]
        g = lay.g if g_in is None else g_in[L]
        plan = bp.make_plan(g, a.budget)
        if scan_events is not None:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e1.record()    # creates the handle; the library records it again right after the scan kernel
            e0.record()
        mlo, mhi = local_window(lo, hi, n_total, a.sink, a.local)
        idx_l, vals_l, _ = bp.scan_select(lay.store, q, plan, a.k, mask_lo=mlo, mask_hi=mhi, index_offset=lo,
                                          scores=scores, with_scores=True,
                                          scan_done_event=e1 if scan_events is not None else None)
        if scan_events is not None:
            scan_events.append((e0, e1, lay.bytes))
        top = merge_shards(idx_l, vals_l, a.k)
        BH, G, _ = top.shape
        fixed = fixed_indices(n_total, a.sink, a.local, top.device).expand(BH, G, -1)
        idx = torch.cat([top, fixed], -1)
        rows = kv[L % len(kv)]
        part = off.decode_attention_partial(q, idx, rows["K"], rows["V"], a.ctx, lo, hi)
        outs[L] = off.attention_combine(all_gather(part))
    return outs
