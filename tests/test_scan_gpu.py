"""Plane-prefix scan on the GPU against the reference's scores (golden fixtures) and the oracle,
in the HBM order, the host run order, and from pinned mapped host memory (zero-copy)."""
import ctypes
import math

import numpy as np
import pytest
import torch

from oracle import bitplane_oracle as O
from tests.helpers import CASES, SCORE_RTOL, load, load_config0, score_rel_err

pytestmark = pytest.mark.gpu


def keys(z):
    return torch.from_numpy(O.bf16_to_f32(z["K_bf16"].view(np.uint16))).cuda()


@pytest.mark.parametrize("name", CASES)
@pytest.mark.parametrize("sub", [16, "nblk"])
def test_scan_golden(name, sub):
    from fathom_b200 import bitplane as bp
    z = load(name)
    K = keys(z)
    old = bp.SUB
    try:
        bp.SUB = math.ceil(K.shape[1] / 64) if sub == "nblk" else sub
        st = bp.PlaneStore(K)
    finally:
        bp.SUB = old
    plan = bp.make_plan(torch.from_numpy(z["g"]).cuda(), float(z["budget"]))
    s = st.scan(torch.from_numpy(z["q"]).cuda(), plan)
    err = score_rel_err(s.cpu().numpy(), z["scores"])
    assert err < SCORE_RTOL, err
    assert err < 1e-5                    # fp32 accumulation-order differences only


@pytest.mark.parametrize("G", [1, 2, 3, 4, 5, 7, 8])
@pytest.mark.parametrize("n", [700, 4096, 33000])
def test_scan_random_vs_oracle(G, n):
    from fathom_b200 import bitplane as bp
    from fathom_b200.synth import make_layer
    d = make_layer(3, G, n, seed=G, layer=n, with_v=False)
    st = bp.PlaneStore(d["K"].cuda())
    plan = bp.make_plan(d["g"].cuda(), 48.0)
    s = st.scan(d["q"].cuda(), plan).cpu().numpy()
    code, sc = O.quantise_u4(d["K"].numpy())
    ref = O.scan_scores(d["q"].numpy(), code, sc, plan["t"].cpu().numpy())
    assert score_rel_err(s, ref) < 1e-5


@pytest.mark.parametrize("budget", [0.0, 1.0, 31.0, 33.0, 48.0, 65.0, 92.0, 130.0, 200.0, 300.0, 512.0])
def test_scan_budgets(budget):
    from fathom_b200 import bitplane as bp
    from fathom_b200.synth import make_layer
    d = make_layer(2, 4, 3000, seed=9, with_v=False)
    st = bp.PlaneStore(d["K"].cuda())
    plan = bp.make_plan(d["g"].cuda(), budget)
    s = st.scan(d["q"].cuda(), plan).cpu().numpy()
    code, sc = O.quantise_u4(d["K"].numpy())
    ref = O.scan_scores(d["q"].numpy(), code, sc, plan["t"].cpu().numpy())
    if budget == 0.0:
        assert np.all(s == 0)
    else:
        assert score_rel_err(s, ref) < 1e-5


def test_scan_block_range_and_out():
    from fathom_b200 import bitplane as bp
    from fathom_b200.synth import make_layer
    d = make_layer(2, 4, 5000, seed=11, with_v=False)
    st = bp.PlaneStore(d["K"].cuda())
    plan = bp.make_plan(d["g"].cuda(), 48.0)
    q = d["q"].cuda()
    full = st.scan(q, plan)
    out = torch.full_like(full, 123.0)
    for b0, b1 in ((0, 5), (5, 21), (21, 40), (40, 79)):
        st.scan(q, plan, out=out, blocks=(b0, b1))
    assert torch.equal(out, full)
    out2 = torch.full_like(full, 7.0)
    st.scan(q, plan, out=out2, blocks=(3, 9))
    assert torch.equal(out2[..., 3 * 64:9 * 64], full[..., 3 * 64:9 * 64])
    assert torch.all(out2[..., :3 * 64] == 7.0) and torch.all(out2[..., 9 * 64:] == 7.0)


@pytest.mark.parametrize("n", [20000, 20480])
def test_host_store_zero_copy_equals_hbm(n):
    """Host run order in pinned mapped memory, read over the host link by the same kernel: bit-identical
    to the HBM store's scores (313 blocks: per-lane copies; 320 blocks: bulk copies of whole tiles)."""
    from fathom_b200 import _lib
    from fathom_b200 import bitplane as bp
    from fathom_b200.offload import HostPlaneStore
    from fathom_b200.synth import make_layer
    d = make_layer(4, 4, n, seed=3, kv_dtype=torch.bfloat16, with_v=False)
    K = d["K"].cuda()
    hs = HostPlaneStore(K)
    hb = bp.PlaneStore(K)
    plan = bp.make_plan(d["g"].cuda(), 48.0)
    q = d["q"].cuda()
    a, b = hs.scan(q, plan), hb.scan(q, plan)
    assert torch.equal(a, b)
    count = ctypes.c_ulonglong(1)
    _lib.check(_lib.lib().fathom_wait_timeouts(ctypes.byref(count), 0), "wait_timeouts")
    assert count.value == 0
    assert hs.sub == math.ceil(n / 64) and hs.nsb == 1
    code, sc = O.quantise_u4(d["K"].float().numpy())
    pk, sk = O.to_superblocks(O.pack_planes(code), sc, hs.sub)
    assert np.array_equal(hs.planes_buf.host.numpy().view(np.uint64), pk)
    hs.free()


def test_config0_scores_sample():
    from fathom_b200 import bitplane as bp
    from fathom_b200.synth import make_config0
    meta, _ = load_config0()
    d = make_config0("cpu")
    st = bp.PlaneStore(d["K"].cuda())
    plan = bp.make_plan(d["g"].cuda(), meta["budget"])
    s = st.scan(d["q"].cuda(), plan).reshape(-1).cpu().numpy()
    got = s[np.asarray(meta["score_sample_idx"])]
    ref = np.asarray(meta["score_sample"], np.float32)
    assert np.abs(got - ref).max() / meta["score_max_abs"] < 1e-5


@pytest.mark.parametrize("G,budget", [(7, 200.0), (8, 512.0), (3, 70.0)])
def test_scan_wide_groups_many_batches(G, budget):
    from fathom_b200 import bitplane as bp
    from fathom_b200.synth import make_layer
    d = make_layer(2, G, 2500, seed=G, layer=7, with_v=False)
    st = bp.PlaneStore(d["K"].cuda())
    plan = bp.make_plan(d["g"].cuda(), budget)
    s = st.scan(d["q"].cuda(), plan).cpu().numpy()
    code, sc = O.quantise_u4(d["K"].numpy())
    ref = O.scan_scores(d["q"].numpy(), code, sc, plan["t"].cpu().numpy())
    assert score_rel_err(s, ref) < 1e-5


@pytest.mark.parametrize("tpl", ["8", "16", "32"])
@pytest.mark.parametrize("G,n", [(4, 131072), (4, 777), (7, 20000), (1, 5000)])
def test_scan_token_splits(tpl, G, n, monkeypatch):
    """Every tokens-per-lane split (forced through FATHOM_SCAN_TPL) gives the oracle's scores and the
    same fused selection."""
    from fathom_b200 import bitplane as bp
    from fathom_b200.synth import make_layer
    monkeypatch.setenv("FATHOM_SCAN_TPL", tpl)
    d = make_layer(2, G, n, seed=n + G, layer=3, with_v=False)
    st = bp.PlaneStore(d["K"].cuda())
    plan = bp.make_plan(d["g"].cuda(), 48.0)
    q = d["q"].cuda()
    s = st.scan(q, plan)
    code, sc = O.quantise_u4(d["K"].numpy())
    ref = O.scan_scores(d["q"].numpy(), code, sc, plan["t"].cpu().numpy())
    assert score_rel_err(s.cpu().numpy(), ref) < 1e-5
    k = min(580, n)
    assert torch.equal(bp.scan_topk(st, q, plan, k, 4, 64), bp.sink_local_topk(s, k, 4, 64))
    out = torch.full_like(s, 5.0)
    st.scan(q, plan, out=out, blocks=(1, 3))
    assert torch.equal(out[..., 64:192], s[..., 64:192]) and torch.all(out[..., :64] == 5.0)


@pytest.mark.parametrize("tpl", ["8", "16", "32"])
@pytest.mark.parametrize("sub", [1, 2, 3, 6, 16, 64, "nblk"])
def test_scan_layouts_and_copy_paths(sub, tpl, monkeypatch):
    """Every superblock order gives bit-identical scores: even orders take the CTA's 16-byte copies,
    odd orders and a planes array that is only 8-byte aligned take the per-lane 4-byte copies."""
    from fathom_b200 import bitplane as bp
    from fathom_b200.synth import make_layer
    monkeypatch.setenv("FATHOM_SCAN_TPL", tpl)
    n = 64 * 37 + 21                      # 38 blocks: ragged last block, odd tile tail
    d = make_layer(2, 4, n, seed=11, layer=2, with_v=False)
    K = d["K"].cuda()
    ref = bp.PlaneStore(K)
    plan = bp.make_plan(d["g"].cuda(), 64.0)
    q = d["q"].cuda()
    want = ref.scan(q, plan)
    old = bp.SUB
    try:
        bp.SUB = math.ceil(n / 64) if sub == "nblk" else sub
        st = bp.PlaneStore(K)
    finally:
        bp.SUB = old
    assert torch.equal(st.scan(q, plan), want)
    # the same words at an address that is 8 but not 16 bytes aligned
    buf = torch.zeros(st.planes_k.numel() + 1, dtype=torch.int64, device="cuda")
    buf[1:] = st.planes_k.reshape(-1)
    st.planes_k = buf[1:].view(st.planes_k.shape)
    st.planes32 = st.planes_k.view(torch.int32)
    assert st.planes32.data_ptr() % 16 == 8
    assert torch.equal(st.scan(q, plan), want)
