"""The copy-index path of the host-resident regime (scripts/B_e2e_offload_v2.py:62-71, 105-133,
182-196): gather_runs copies device-described runs exactly; stream_planes stages the needed planes of
a host store chunk by chunk and scans them from device memory with the same scores as the zero-copy
scan, bit for bit; a decode step through it matches the default one."""
import numpy as np
import pytest
import torch

from oracle import bitplane_oracle as O
from tests.helpers import SCORE_RTOL, score_rel_err

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("where", ["device", "host"])
def test_gather_runs_copies_exactly_the_listed_runs(where):
    from fathom_b200.offload import MappedBuffer, gather_runs
    gen = torch.Generator().manual_seed(11)
    W = 200_000
    src_cpu = torch.randint(-2**31, 2**31 - 1, (W,), generator=gen, dtype=torch.int64).to(torch.int32)
    buf = None
    if where == "host":
        buf = MappedBuffer((W,), torch.int32)
        buf.host.copy_(src_cpu)
        src = buf.dev
    else:
        src = src_cpu.cuda()
    # disjoint runs with every alignment of the start word, zero and odd lengths, runs past nrun and a
    # negative offset (both skipped)
    lens = [0, 1, 2, 3, 4, 5, 7, 17, 255, 4096, 4097, 10_000, 3, 1, 0, 9000, 6, 1023, 12, 5000]
    off, pos = [], 1
    for i, ln in enumerate(lens):
        pos += i % 4                     # start words at every residue modulo 4 (16-byte vectors)
        off.append(pos)
        pos += ln + 5
    off[3] = -7
    R, nrun = len(lens), len(lens) - 2
    dst = torch.full((W,), -1, dtype=torch.int32, device="cuda")
    gather_runs(src, dst, torch.tensor(off, dtype=torch.int32).cuda(), torch.tensor(lens, dtype=torch.int32).cuda(),
                torch.tensor([nrun], dtype=torch.int32).cuda(), max(lens), CH=1000)
    torch.cuda.synchronize()
    want = torch.full((W,), -1, dtype=torch.int32)
    for r in range(nrun):
        if off[r] >= 0 and lens[r] > 0:
            want[off[r]:off[r] + lens[r]] = src_cpu[off[r]:off[r] + lens[r]]
    assert torch.equal(dst.cpu(), want)
    if buf is not None:
        buf.free()


@pytest.mark.parametrize("n,G,parts,budget", [(131072, 4, 4, 48.0), (70000, 7, 3, 40.0), (20000, 4, 1, 80.0),
                                              (5000, 2, 8, 48.0)])
def test_stream_planes_scores_equal_the_zero_copy_scan(n, G, parts, budget):
    from fathom_b200 import bitplane as bp
    from fathom_b200.offload import HostPlaneStore, PlaneStaging, stream_planes
    from fathom_b200.synth import make_layer
    BH = 3
    d = make_layer(BH, G, n, seed=n + G, layer=2)
    store = HostPlaneStore(d["K"].cuda())
    q, g = d["q"].cuda(), d["g"].cuda()
    plan = bp.make_plan(g, budget)
    direct = store.scan(q, plan)
    staging = PlaneStaging(BH, n, q.device)
    staging.planes_k.fill_(0x5A5A5A5A5A5A5A5A)      # stale contents must never reach a score
    staging.scales_k.fill_(float("nan"))
    streamed = stream_planes(store, q, plan, parts=parts, staging=staging)
    torch.cuda.synchronize()
    assert torch.equal(streamed, direct)
    # the staging holds exactly the planes below each channel's depth and the active channels' scales
    t = plan["t"].long().cpu()
    on_p = (torch.arange(4)[None, None, :] < t[:, :, None])
    hp, sp = store.planes_k.cpu()[:, 0], staging.planes_k.cpu()[:, 0]
    assert torch.equal(sp[on_p], hp[on_p])
    act = t > 0
    assert torch.equal(staging.scales_k.cpu()[:, 0][act].view(torch.int16), store.scales_k.cpu()[:, 0][act].view(torch.int16))
    if n <= 20000:
        code, sc = O.quantise_u4(d["K"].float().numpy())
        ref = O.scan_scores(d["q"].numpy(), code, sc, O.make_plan(d["g"].numpy(), budget)["t"])
        assert score_rel_err(streamed.cpu().numpy(), ref) < SCORE_RTOL
    store.free()


def test_decode_step_through_the_copy_index_pipeline_equals_the_default():
    from fathom_b200.offload import HostPlaneStore, MappedBuffer, decode_step
    from fathom_b200.synth import make_layer
    BH, G, n, k, sink, local = 2, 4, 65536, 580, 4, 64
    d = make_layer(BH, G, n, seed=21, layer=0, kv_dtype=torch.bfloat16, with_v=True)
    store = HostPlaneStore(d["K"].cuda())
    kv = MappedBuffer((BH, n, 2, 128), torch.bfloat16)
    kv.host[:, :, 0].copy_(d["K"])
    kv.host[:, :, 1].copy_(d["V"])
    q, g = d["q"].cuda(), d["g"].cuda()
    out0, idx0 = decode_step(q, g, 48.0, store, kv.dev[:, :, 0], kv.dev[:, :, 1], n, k, sink, local)
    for parts in (1, 4):
        out1, idx1 = decode_step(q, g, 48.0, store, kv.dev[:, :, 0], kv.dev[:, :, 1], n, k, sink, local,
                                 stream_parts=parts)
        torch.cuda.synchronize()
        assert torch.equal(idx1, idx0)
        assert torch.equal(out1, out0)
    kv.free()
    store.free()


def test_stream_planes_rejects_a_store_not_in_the_run_order():
    from fathom_b200 import bitplane as bp
    from fathom_b200.offload import stream_planes
    from fathom_b200.synth import make_layer
    d = make_layer(2, 4, 4096, seed=1, layer=0)
    st = bp.PlaneStore(d["K"].cuda())            # SUB = 16 superblocks, not the run order
    plan = bp.make_plan(d["g"].cuda(), 48.0)
    with pytest.raises(ValueError):
        stream_planes(st, d["q"].cuda(), plan)


def test_stream_planes_at_the_bench_context_equals_the_zero_copy_scan():
    """The headline context (T = 1,048,576, 2 KV heads, G = 4, budget 48), 4 pipelined chunks: bit for bit."""
    from fathom_b200 import bitplane as bp
    from fathom_b200.offload import HostPlaneStore, PlaneStaging, stream_planes
    from fathom_b200.synth import make_layer
    BH, G, n = 2, 4, 1048576
    d = make_layer(BH, G, n, seed=5, layer=0, device="cuda", kv_dtype=torch.bfloat16)
    store = HostPlaneStore(d["K"])
    del d["K"]
    plan = bp.make_plan(d["g"], 48.0)
    direct = store.scan(d["q"], plan)
    staging = PlaneStaging(BH, n, d["q"].device)
    streamed = stream_planes(store, d["q"], plan, parts=4, staging=staging)
    torch.cuda.synchronize()
    assert torch.equal(streamed, direct)
    store.free()


def test_decode_step_through_the_copy_index_pipeline_with_a_klt_store():
    """A KLT-rotated host store (planesK): the copy-index path scans the rotated queries like the default."""
    from fathom_b200 import klt
    from fathom_b200.offload import HostPlaneStore, MappedBuffer, decode_step
    from fathom_b200.synth import make_layer
    BH, G, n, k = 2, 4, 30000, 580
    d = make_layer(BH, G, n, seed=13, kv_dtype=torch.bfloat16, with_v=True)
    K, q = d["K"].cuda(), d["q"].cuda()
    st = HostPlaneStore(K, torch.float32, basis=klt.klt_basis(K))
    kb, vb = MappedBuffer(K.shape, torch.bfloat16), MappedBuffer(K.shape, torch.bfloat16)
    kb.host.copy_(d["K"])
    vb.host.copy_(d["V"])
    out0, idx0 = decode_step(q, None, 48.0, st, kb.dev, vb.dev, n, k, 4, 64)
    out1, idx1 = decode_step(q, None, 48.0, st, kb.dev, vb.dev, n, k, 4, 64, stream_parts=3)
    torch.cuda.synchronize()
    assert torch.equal(idx1, idx0)
    assert torch.equal(out1, out0)
    kb.free()
    vb.free()
    st.free()
