"""Context-sharded selection and attention on 2 GPUs with NCCL (skipped with fewer GPUs).

Each rank builds the store of its contiguous chunk of one shared context, selects its local top-kk
with the fused scan, and the ranks all-gather and merge the candidates; the merged indices must equal
the single-GPU selection over the whole context bit for bit, and the log-sum-exp combine of the
ranks' partial attention must equal the single-GPU attention.
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, result):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=120))
    try:
        from fathom_b200 import bitplane as bp, offload as off, shard
        from fathom_b200.synth import make_layer
        n, k, sink, local = 2 * 64 * 400, 580, 4, 64
        kk = k - sink - local
        d = make_layer(4, 4, n, seed=5, kv_dtype=torch.bfloat16, with_v=True)   # same data on every rank (CPU RNG)
        K, V, q, g = d["K"].to(dev), d["V"].to(dev), d["q"].to(dev), d["g"].to(dev)
        plan = bp.make_plan(g, 48.0)
        full = bp.PlaneStore(K)
        ref_idx = bp.scan_topk(full, q, plan, k, sink, local)
        ref_out = off.decode_attention(q, ref_idx, K, V, n)
        lo, hi = shard.chunk_bounds(n, world)[rank]
        st = off.HostPlaneStore(K[:, lo:hi].contiguous())
        mlo, mhi = shard.local_window(lo, hi, n, sink, local)
        idx_l, vals_l, _ = bp.scan_select(st, q, plan, kk, mask_lo=mlo, mask_hi=mhi, index_offset=lo, with_scores=True)
        top = shard.merge_shards(idx_l, vals_l, kk)
        idx = torch.cat([top, shard.fixed_indices(n, sink, local, dev).expand(4, 4, -1)], -1)
        part = off.decode_attention_partial(q, idx, K[:, lo:hi].contiguous(), V[:, lo:hi].contiguous(), hi - lo, lo, hi)
        out = off.attention_combine(shard.all_gather(part))
        result[rank] = (bool(torch.equal(idx, ref_idx)),
                        float((out - ref_out).abs().max() / ref_out.abs().max()))
        st.free()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_sharded_decode_matches_single_gpu():
    with mp.Manager() as mgr:
        result = mgr.dict()
        mp.spawn(_rank, args=(2, _free_port(), result), nprocs=2, join=True)
        for r in range(2):
            same, err = result[r]
            assert same, f"rank {r}: merged indices differ from the single-GPU selection"
            assert err < 1e-5, f"rank {r}: combined attention differs by {err}"
