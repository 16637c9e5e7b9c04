"""Chan4 comparator store and scan on the GPU against the reference's own outputs (fixtures made by
running kernels/bitplane.py, its Triton scan_chan4_kernel included) and the oracle."""
import math
import os

import numpy as np
import pytest
import torch

from oracle import bitplane_oracle as O
from tests.helpers import score_rel_err

pytestmark = pytest.mark.gpu

CASES = ("c1", "c2", "c3", "c4")


def _fixture():
    return np.load(os.path.join(os.path.dirname(__file__), "golden", "chan4.npz"))


def _store(bp, K, sub):
    old = bp.SUB
    try:
        bp.SUB = sub
        return bp.Chan4Store(K)
    finally:
        bp.SUB = old


def _scores_agree(got, ref, tol):
    """+-inf at the same positions (fp16 amax overflow rows), finite rows within tol."""
    assert np.array_equal(np.isinf(got), np.isinf(ref)) and np.array_equal(got[np.isinf(got)], ref[np.isinf(ref)])
    fin = np.isfinite(ref).all(-1)
    assert score_rel_err(got[fin], ref[fin]) < tol


@pytest.mark.parametrize("c", CASES)
def test_chan4_store_and_scan_match_reference(c):
    from fathom_b200 import bitplane as bp
    z = _fixture()
    K = torch.from_numpy(O.bf16_to_f32(z[f"{c}_K_bf16"].view(np.uint16))).cuda()
    st = _store(bp, K, int(z[f"{c}_sub"]))
    assert np.array_equal(st.code.cpu().numpy(), z[f"{c}_code"])
    assert np.array_equal(st.chan_k.cpu().numpy(), z[f"{c}_chan_k"])
    assert np.array_equal(st.scales_k.cpu().view(torch.int16).numpy(), z[f"{c}_scales_k"])
    act, nact = bp.channel_list(torch.from_numpy(z[f"{c}_active"]).cuda())
    assert np.array_equal(act.cpu().numpy(), z[f"{c}_act"]) and np.array_equal(nact.cpu().numpy(), z[f"{c}_nact"])
    assert bp.bytes_chan4(nact, K.shape[1]) == float(z[f"{c}_bytes"])
    s = st.scan(torch.from_numpy(z[f"{c}_q"]).cuda(), act, nact).cpu().numpy()
    _scores_agree(s, z[f"{c}_scores"], 1e-5)
    if f"{c}_scores_triton" in z.files:
        _scores_agree(s, z[f"{c}_scores_triton"], 1e-5)


@pytest.mark.parametrize("G", [1, 3, 4, 7, 8])
@pytest.mark.parametrize("n,r", [(777, 16), (20000, 32), (4096, 128)])
def test_chan4_random_vs_oracle(G, n, r):
    """SparQ's rule (top-r channels of sum_g |q_g|), the reference benchmark's channel sets."""
    from fathom_b200 import bitplane as bp
    from fathom_b200.synth import make_layer
    d = make_layer(3, G, n, seed=n + G + r, with_v=False)
    st = bp.Chan4Store(d["K"].cuda())
    q = d["q"].cuda()
    a = torch.zeros(3, 128, dtype=torch.bool, device="cuda")
    a.scatter_(1, q.abs().sum(1).topk(r, -1).indices, True)
    act, nact = bp.channel_list(a)
    s = st.scan(q, act, nact).cpu().numpy()
    code, sc = O.quantise_u4(d["K"].numpy())
    ref = O.scan_chan4(d["q"].numpy(), code, sc, a.cpu().numpy())
    assert score_rel_err(s, ref) < 1e-5


def test_chan4_orders_and_block_range():
    """HBM order (SUB = 16) and host run order (SUB = nblk) give the same bits; blocks=(b0, b1) writes only
    those tokens."""
    from fathom_b200 import bitplane as bp
    from fathom_b200.synth import make_layer
    n = 64 * 37 + 9
    d = make_layer(2, 4, n, seed=3, with_v=False)
    K, q = d["K"].cuda(), d["q"].cuda()
    a = torch.rand(2, 128, device="cuda", generator=torch.Generator(device="cuda").manual_seed(0)) < 0.3
    act, nact = bp.channel_list(a)
    s16 = _store(bp, K, 16).scan(q, act, nact)
    sN = _store(bp, K, math.ceil(n / 64)).scan(q, act, nact)
    assert torch.equal(s16, sN)
    out = torch.full_like(s16, 3.0)
    _store(bp, K, 16).scan(q, act, nact, out=out, blocks=(5, 11))
    assert torch.equal(out[..., 5 * 64:11 * 64], s16[..., 5 * 64:11 * 64])
    assert torch.all(out[..., :5 * 64] == 3.0) and torch.all(out[..., 11 * 64:] == 3.0)


def test_host_chan4_store_matches_device_store():
    """HostChan4Store (pinned mapped host memory, run order SUB = nblk, zero-copy scan) gives the same bits
    as the device store in the same order."""
    from fathom_b200 import bitplane as bp
    from fathom_b200.offload import HostChan4Store
    from fathom_b200.synth import make_layer
    n = 20000
    d = make_layer(2, 4, n, seed=9, kv_dtype=torch.bfloat16, with_v=False)
    K, q = d["K"].cuda(), d["q"].cuda()
    a = torch.zeros(2, 128, dtype=torch.bool, device="cuda")
    a.scatter_(1, q.abs().sum(1).topk(16, -1).indices, True)
    act, nact = bp.channel_list(a)
    hs = HostChan4Store(K)
    try:
        assert hs.sub == math.ceil(n / 64) and hs.nsb == 1
        s_host = hs.scan(q, act, nact)
        s_dev = _store(bp, K, math.ceil(n / 64)).scan(q, act, nact)
        assert torch.equal(s_host, s_dev)
        code, sc = O.quantise_u4(d["K"].float().numpy())
        ref = O.scan_chan4(d["q"].numpy(), code, sc, a.cpu().numpy())
        assert score_rel_err(s_host.cpu().numpy(), ref) < 1e-5
    finally:
        hs.free()
