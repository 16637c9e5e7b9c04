"""Host logic of the context-sharded selection with two CPU ranks over gloo: chunk bounds, the
sink/local windows per rank, the packed all-gather and the merge.  The per-rank GPU kernels are
replaced by the CPU oracle (injected), so this runs without a GPU; the GPU kernels themselves are
checked against the oracle by the -m gpu tests."""
import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import bitplane_oracle as O


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _oracle_select(scores, kk, mask_lo, mask_hi, offset):
    s = scores.numpy().copy()
    s[..., :mask_lo] = -np.inf
    s[..., mask_hi:] = -np.inf
    idx = O.topk_desc(s, kk)
    vals = np.take_along_axis(s, idx, -1)
    return torch.from_numpy(idx + offset), torch.from_numpy(vals)


def _oracle_merge(cv, ci, kk):
    return torch.from_numpy(O.merge_candidates(cv.numpy(), ci.numpy(), kk))


def _rank(rank, world, port, scores, kk, sink, local, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from fathom_b200 import shard
        n = scores.shape[-1]
        lo, hi = shard.chunk_bounds(n, world)[rank]
        got = shard.sharded_select(scores[..., lo:hi], kk, lo, hi, n, sink, local,
                                   select_fn=_oracle_select, merge_fn=_oracle_merge)
        out[rank] = got.numpy()
    finally:
        dist.destroy_process_group()


def test_two_rank_sharded_select_matches_single():
    g = torch.Generator().manual_seed(0)
    scores = torch.randn(2, 3, 64 * 90 + 17, generator=g)
    kk, sink, local = 200, 4, 64
    ref = O.sink_local_topk(scores.numpy(), kk + sink + local, sink, local)[..., :kk]
    with mp.Manager() as mgr:
        out = mgr.dict()
        mp.spawn(_rank, args=(2, _free_port(), scores, kk, sink, local, out), nprocs=2, join=True)
        for r in range(2):
            assert np.array_equal(out[r], ref)


def test_chunk_bounds_and_windows():
    from fathom_b200 import shard
    for n in (1, 63, 64, 1000, 1 << 20, 4194304):
        for world in (1, 2, 3, 4, 8):
            b = shard.chunk_bounds(n, world)
            assert b[0][0] == 0 and b[-1][1] == n and len(b) == world
            for (a, c), (d, e) in zip(b, b[1:]):
                assert c == d and c % 64 == 0 and a <= c
    # sink window only on the first chunk, local window only where it falls
    assert shard.local_window(0, 1000, 4000, 4, 64) == (4, 1000)
    assert shard.local_window(3000, 4000, 4000, 4, 64) == (0, 936)
    assert shard.local_window(3968, 4000, 4000, 4, 64) == (0, 0)


def _oracle_single(s, kk, mask_lo, mask_hi):
    m = s.numpy().copy()
    m[..., :mask_lo] = -np.inf
    m[..., mask_hi:] = -np.inf
    return torch.from_numpy(O.topk_desc(m, kk))


def _parity_rank(rank, world, port, scores, kk, sink, local, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from fathom_b200 import shard
        n = scores.shape[-1]
        c = n // world
        lo, hi = rank * c, (rank + 1) * c
        top = shard.sharded_select(scores[..., lo:hi], kk, lo, hi, n, sink, local,
                                   select_fn=_oracle_select, merge_fn=_oracle_merge)
        good = shard.merged_equals_single(scores[..., lo:hi], top, n, kk, sink, local, select_fn=_oracle_single)
        bad_top = top.clone()
        bad_top[0, 0, [0, 1]] = bad_top[0, 0, [1, 0]]          # a merge that broke the order
        bad = shard.merged_equals_single(scores[..., lo:hi], bad_top, n, kk, sink, local, select_fn=_oracle_single)
        # concurrent probe: rank r moves (r + 1) GB in (r + 1) * 0.5 s -> aggregate 3 GB / 1 s
        agg, per = shard.concurrent_probe(lambda: ((rank + 1) * 1e9, (rank + 1) * 0.5), rounds=2)
        out[rank] = (good, bad, agg, per)
    finally:
        dist.destroy_process_group()


def test_merged_parity_check_and_concurrent_probe_two_ranks():
    """The bench's multi-GPU parity check (merged top-k vs one selection over the all-gathered score
    chunks) accepts a correct merge and rejects a planted wrong one; the synchronised probe sums the
    ranks' bytes over the slowest rank's time."""
    g = torch.Generator().manual_seed(3)
    scores = torch.randn(2, 3, 64 * 100, generator=g)
    with mp.Manager() as mgr:
        out = mgr.dict()
        mp.spawn(_parity_rank, args=(2, _free_port(), scores, 300, 4, 64, out), nprocs=2, join=True)
        for r in range(2):
            good, bad, agg, per = out[r]
            assert good and not bad
            assert abs(agg - 3e9) < 1 and per == [2e9, 2e9]
