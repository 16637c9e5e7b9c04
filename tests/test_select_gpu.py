"""Top-k selection on the GPU: sink_local_topk, select_topk and merge_topk against the oracle
(exact, including the deterministic tie order) and the reference's fixtures (sets up to ties)."""
import numpy as np
import pytest
import torch

from oracle import bitplane_oracle as O
from tests.helpers import CASES, load, topk_sets_agree

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", [c for c in CASES if c != "s4_b0"])
def test_sink_local_topk_golden(name):
    from fathom_b200 import bitplane as bp
    z = load(name)
    k, sink, local = int(z["topk_k"]), int(z["topk_sink"]), int(z["topk_local"])
    idx = bp.sink_local_topk(torch.from_numpy(z["scores"]).cuda(), k, sink, local).cpu().numpy()
    kk = k - sink - local
    masked = z["scores"].copy()
    masked[..., :sink] = -np.inf
    masked[..., masked.shape[-1] - local:] = -np.inf
    assert topk_sets_agree(masked, idx, z["topk"], kk)
    assert np.array_equal(idx[..., kk:], z["topk"][..., kk:])
    assert np.array_equal(idx, O.sink_local_topk(z["scores"], k, sink, local))


@pytest.mark.parametrize("rows,n,k,sink,local", [(32, 131072, 580, 4, 64), (8, 16384, 580, 4, 64), (3, 1000, 1000, 0, 0),
                                                 (5, 777, 1, 0, 0), (4, 70000, 2116, 4, 64), (2, 300000, 4096, 0, 0)])
def test_sink_local_topk_random_exact(rows, n, k, sink, local):
    from fathom_b200 import bitplane as bp
    g = torch.Generator().manual_seed(n + k)
    s = torch.randn(rows, n, generator=g)
    idx = bp.sink_local_topk(s.cuda(), k, sink, local).cpu().numpy()
    assert np.array_equal(idx, O.sink_local_topk(s.numpy(), k, sink, local))


@pytest.mark.parametrize("levels", [1, 3, 50, 5000])
def test_ties_follow_index_order(levels):
    """Heavy ties (few distinct values; `levels=1` is an all-equal row that forces the exact
    whole-row path): the result is the oracle's (score desc, index asc) order exactly."""
    from fathom_b200 import bitplane as bp
    g = torch.Generator().manual_seed(levels)
    s = torch.randint(0, levels, (6, 40000), generator=g).float()
    idx = bp.sink_local_topk(s.cuda(), 600, 4, 64).cpu().numpy()
    assert np.array_equal(idx, O.sink_local_topk(s.numpy(), 600, 4, 64))


def test_select_topk_offset_mask_scores():
    from fathom_b200 import bitplane as bp
    g = torch.Generator().manual_seed(1)
    s = torch.randn(4, 9000, generator=g)
    idx, vals = bp.select_topk(s.cuda(), 300, mask_lo=10, mask_hi=8000, index_offset=123456, with_scores=True)
    m = s.numpy().copy()
    m[:, :10] = -np.inf
    m[:, 8000:] = -np.inf
    ref = O.topk_desc(m, 300)
    assert np.array_equal(idx.cpu().numpy(), ref + 123456)
    assert np.array_equal(vals.cpu().numpy(), np.take_along_axis(m, ref, -1))


def test_select_with_neg_inf_and_small_rows():
    """kk larger than the unmasked count: masked (-inf) tokens fill the tail in index order."""
    from fathom_b200 import bitplane as bp
    s = torch.randn(3, 50)
    idx = bp.select_topk(s.cuda(), 20, mask_lo=5, mask_hi=15).cpu().numpy()
    m = s.numpy().copy()
    m[:, :5] = -np.inf
    m[:, 15:] = -np.inf
    assert np.array_equal(idx, O.topk_desc(m, 20))


@pytest.mark.parametrize("m,kk", [(4096, 512), (2048, 2048), (8192, 100), (3, 2)])
def test_merge_topk(m, kk):
    from fathom_b200 import bitplane as bp
    g = torch.Generator().manual_seed(m)
    cs = torch.randn(7, m, generator=g)
    half = m // 2
    cs[:, half:2 * half] = cs[:, :half]                     # duplicate scores: tie order by index
    ci = torch.randperm(1 << 22, generator=g)[: 7 * m].view(7, m)
    idx, vals = bp.merge_topk(cs.cuda(), ci.cuda(), kk)
    ref = O.merge_candidates(cs.numpy(), ci.numpy(), kk)
    assert np.array_equal(idx.cpu().numpy(), ref)


def test_shard_merge_equals_single():
    """Context split into 4 chunks: per-chunk select (global indices) + merge == single-pass select."""
    from fathom_b200 import bitplane as bp
    g = torch.Generator().manual_seed(7)
    n, kk, sink, local = 40000, 512, 4, 64
    s = torch.randn(8, n, generator=g).cuda()
    full = bp.select_topk(s, kk, mask_lo=sink, mask_hi=n - local)
    bounds = [0, 9984, 20032, 30016, n]                       # 64-token aligned boundaries
    cs, ci = [], []
    for r in range(4):
        a, b = bounds[r], bounds[r + 1]
        lo = max(sink - a, 0)
        hi = min(n - local, b) - a
        i, v = bp.select_topk(s[:, a:b], kk, mask_lo=lo, mask_hi=max(hi, 0), index_offset=a, with_scores=True)
        cs.append(v)
        ci.append(i)
    idx, _ = bp.merge_topk(torch.cat(cs, -1), torch.cat(ci, -1), kk)
    assert torch.equal(idx, full)


@pytest.mark.parametrize("world", [2, 3, 8])
def test_sharded_select_emulated_equals_single(world):
    """shard.sharded_select with every rank emulated on this GPU (the collective is a stack of the
    ranks' packed candidates): merged indices bit-exact vs the single-pass sink+local selection."""
    from fathom_b200 import bitplane as bp, shard
    g = torch.Generator().manual_seed(world)
    n, kk, sink, local = 64 * 700, 512, 4, 64
    s = torch.randn(8, 4, n, generator=g).cuda()
    full = bp.sink_local_topk(s, kk + sink + local, sink, local)[..., :kk]
    bounds = shard.chunk_bounds(n, world)
    packs = []
    def capture(t):
        packs.append(t)
        raise StopIteration
    for lo, hi in bounds:
        try:
            shard.sharded_select(s[..., lo:hi], kk, lo, hi, n, sink, local, gather_fn=capture)
        except StopIteration:
            pass
    allp = torch.stack(packs)
    for lo, hi in bounds:
        got = shard.sharded_select(s[..., lo:hi], kk, lo, hi, n, sink, local, gather_fn=lambda t: allp)
        assert torch.equal(got, full)


@pytest.mark.parametrize("G,n,k", [(4, 131072, 580), (4, 700, 100), (7, 33000, 2116), (1, 5000, 300), (8, 20000, 1000)])
@pytest.mark.parametrize("sub", [16, "nblk"])
def test_scan_topk_fused_equals_unfused(G, n, k, sub):
    """scan_topk / scan_select in one call select exactly what scan + sink_local_topk selects (same scores,
    same order)."""
    import math
    from fathom_b200 import bitplane as bp
    from fathom_b200.synth import make_layer
    d = make_layer(2, G, n, seed=G + n, with_v=False)
    old = bp.SUB
    try:
        bp.SUB = math.ceil(n / 64) if sub == "nblk" else sub
        st = bp.PlaneStore(d["K"].cuda())
    finally:
        bp.SUB = old
    plan = bp.make_plan(d["g"].cuda(), 48.0)
    q = d["q"].cuda()
    s = st.scan(q, plan)
    ref = bp.sink_local_topk(s, k, 4, 64)
    got = bp.scan_topk(st, q, plan, k, 4, 64)
    assert torch.equal(got, ref)
    idx, vals, s2 = bp.scan_select(st, q, plan, 200, mask_lo=10, mask_hi=n - 5, index_offset=1000, with_scores=True)
    r_idx, r_vals = bp.select_topk(s, 200, mask_lo=10, mask_hi=n - 5, index_offset=1000, with_scores=True)
    assert torch.equal(s2, s) and torch.equal(idx, r_idx) and torch.equal(vals, r_vals)


def test_scan_topk_all_ties():
    """Budget 0: every score is 0 (massive ties, the exact whole-row path): lowest indices first."""
    from fathom_b200 import bitplane as bp
    from fathom_b200.synth import make_layer
    d = make_layer(2, 4, 30000, seed=1, with_v=False)
    st = bp.PlaneStore(d["K"].cuda())
    plan = bp.make_plan(d["g"].cuda(), 0.0)
    got = bp.scan_topk(st, d["q"].cuda(), plan, 580, 4, 64).cpu().numpy()
    assert np.array_equal(got, O.sink_local_topk(np.zeros((2, 4, 30000), np.float32), 580, 4, 64))


def _hist_path_bytes(rows):
    a = lambda x: (x + 255) // 256 * 256
    return a(rows * 4096 * 4) + 3 * a(rows * 4) + a(rows * 8192 * 8)


@pytest.mark.parametrize("sink,local,kk", [(0, 0, 500), (4, 64, 508), (5, 33, 4000), (100, 1000, 64)])
def test_group_path_equals_histogram_path(sink, local, kk):
    """The group-key selection (a workspace that holds the group keys) and the histogram selection
    (a workspace sized for the histogram path only) give the oracle's exact output."""
    import ctypes
    from fathom_b200 import _lib
    rows, n = 2, (1 << 20) + 77
    g = torch.Generator().manual_seed(kk + sink)
    s = torch.randn(rows, n, generator=g)
    s[:, 5000:5010] = 3.0                  # a few exact ties near the top
    sd = s.cuda()
    k = kk + sink + local
    full = _lib.lib().fathom_select_workspace_bytes(rows, n, kk)
    small = _hist_path_bytes(rows)
    assert full > small                    # the group keys need more than the histogram path
    outs = []
    for nbytes in (full, small):
        ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
        idx = torch.empty(rows, k, dtype=torch.int64, device="cuda")
        _lib.check(_lib.lib().fathom_sink_local_topk(_lib.ptr(sd), rows, n, k, sink, local, _lib.ptr(idx), _lib.ptr(ws),
                                                     ctypes.c_size_t(nbytes), None), "sink_local_topk")
        outs.append(idx.cpu().numpy())
    ref = O.sink_local_topk(s.numpy(), k, sink, local)
    assert np.array_equal(outs[0], ref) and np.array_equal(outs[1], ref)


@pytest.mark.parametrize("n", [31, 32, 33, 64 * 37 + 5, 40000])
def test_group_path_ragged_rows(n):
    """Rows whose length is not a multiple of the 32-token group, masks that cut groups, scan-written
    group keys (fused) against the oracle."""
    from fathom_b200 import bitplane as bp
    from fathom_b200.synth import make_layer
    d = make_layer(2, 4, n, seed=n, with_v=False)
    st = bp.PlaneStore(d["K"].cuda())
    plan = bp.make_plan(d["g"].cuda(), 48.0)
    q = d["q"].cuda()
    kk = max(1, min(300, n // 70))
    lo, hi = 3, n - 7 if n > 20 else n
    idx, vals, s = bp.scan_select(st, q, plan, kk, mask_lo=lo, mask_hi=hi, with_scores=True)
    m = s.cpu().numpy().copy()
    m[..., :lo] = -np.inf
    m[..., hi:] = -np.inf
    assert np.array_equal(idx.cpu().numpy(), O.topk_desc(m, kk))
