"""The reference module's dense torch helpers (dequant_planes, scan_planes_reference, scan_chan4_reference,
make_plan_torch) on the GPU, against outputs of the reference itself (golden fixtures) and the oracle."""
import math
import os

import numpy as np
import pytest
import torch

from oracle import bitplane_oracle as O
from tests.helpers import CASES, load, score_rel_err

pytestmark = pytest.mark.gpu


def _fp16(a):
    return torch.from_numpy(np.ascontiguousarray(a)).view(torch.float16).cuda()


@pytest.mark.parametrize("name", CASES)
def test_dequant_planes_bit_exact_and_scores_golden(name):
    from fathom_b200 import bitplane as bp
    z = load(name)
    code = torch.from_numpy(z["code"]).cuda()
    sc = _fp16(z["scales"])
    t = z["plan_t"].astype(np.int64)
    for b in range(code.shape[0]):
        got = bp.dequant_planes(code[b], sc[b], torch.from_numpy(t[b]).cuda()).cpu().numpy()
        ref = O.dequant_planes(z["code"][b], z["scales"][b].view(np.float16), t[b])
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    # per-row depths [BH, D] and a scalar depth
    got = bp.dequant_planes(code, sc, torch.from_numpy(t).cuda()).cpu().numpy()
    for b in range(code.shape[0]):
        assert np.array_equal(got[b], O.dequant_planes(z["code"][b], z["scales"][b].view(np.float16), t[b]))
    for depth in (0, 1, 4):
        got = bp.dequant_planes(code, sc, depth).cpu().numpy()
        ref = O.dequant_planes(z["code"], z["scales"].view(np.float16), np.full(128, depth))
        assert np.array_equal(got, ref)
    # q @ dequant_planes(...).T is the reference's scan_planes_reference (fixture scores)
    dq = bp.dequant_planes(code, sc, torch.from_numpy(t).cuda()).double()
    s = torch.einsum("bgd,bnd->bgn", torch.from_numpy(z["q"]).cuda().double(), dq).cpu().numpy()
    fin = np.isfinite(z["scores"]).all(-1)
    assert score_rel_err(s[fin], z["scores"][fin]) < 1e-5


@pytest.mark.parametrize("name", CASES)
def test_scan_planes_reference_golden(name):
    from fathom_b200 import bitplane as bp
    z = load(name)
    got = bp.scan_planes_reference(torch.from_numpy(z["q"]).cuda(), torch.from_numpy(z["code"]).cuda(),
                                   _fp16(z["scales"]), torch.from_numpy(z["plan_t"]).cuda()).cpu().numpy()
    ref = z["scores"]
    fin = np.isfinite(ref).all(-1)
    assert np.array_equal(np.isfinite(got), np.isfinite(ref))
    assert score_rel_err(got[fin], ref[fin]) < 1e-5


@pytest.mark.parametrize("c", ("c1", "c2", "c3", "c4"))
def test_scan_chan4_reference_golden(c):
    from fathom_b200 import bitplane as bp
    z = np.load(os.path.join(os.path.dirname(__file__), "golden", "chan4.npz"))
    code = z[f"{c}_code"]
    nb = math.ceil(code.shape[1] / 64)
    _, sc = O.from_superblocks(np.zeros((*z[f"{c}_scales_k"].shape[:3], 4, z[f"{c}_scales_k"].shape[3]), np.int64),
                               z[f"{c}_scales_k"].view(np.float16), nb)
    got = bp.scan_chan4_reference(torch.from_numpy(z[f"{c}_q"]).cuda(), torch.from_numpy(code).cuda(),
                                  torch.from_numpy(sc).cuda(), torch.from_numpy(z[f"{c}_active"]).cuda()).cpu().numpy()
    ref = z[f"{c}_scores"]
    assert np.array_equal(np.isnan(got), np.isnan(ref))
    assert np.array_equal(np.isinf(got), np.isinf(ref)) and np.array_equal(got[np.isinf(got)], ref[np.isinf(ref)])
    fin = np.isfinite(ref).all(-1)
    assert score_rel_err(got[fin], ref[fin]) < 1e-5


@pytest.mark.parametrize("name", CASES)
def test_make_plan_torch_golden(name):
    from fathom_b200 import bitplane as bp
    z = load(name)
    t = bp.make_plan_torch(torch.from_numpy(z["g"]).cuda(), float(z["budget"]))
    assert t.dtype == torch.float32
    assert np.array_equal(t.cpu().numpy(), z["plan_t"].astype(np.float32))
    tb = bp.make_plan_torch(torch.from_numpy(z["g"]).cuda(), torch.full((z["g"].shape[0],), float(z["budget"])).cuda())
    assert torch.equal(tb, t)


def test_scan_planes_reference_random_g7_fp32_scales():
    """G = 7, fp32 block scales, a ragged length: against the oracle's restatement."""
    from fathom_b200 import bitplane as bp
    g = torch.Generator().manual_seed(5)
    BH, G, n = 3, 7, 333
    K = torch.randn(BH, n, 128, generator=g) * torch.randn(BH, 1, 128, generator=g).exp()
    q = torch.randn(BH, G, 128, generator=g)
    code, sc = bp.quantise_u4(K.cuda(), torch.float32)
    t = torch.randint(0, 5, (BH, 128), generator=g)
    got = bp.scan_planes_reference(q.cuda(), code, sc, t.cuda()).cpu().numpy()
    ref = O.scan_scores(q.numpy(), code.cpu().numpy(), sc.cpu().numpy(), t.numpy())
    assert score_rel_err(got, ref) < 1e-5
