"""Water-filling plan on the GPU: depths and every compacted list bit-exact against the reference
(golden fixtures) and the oracle."""
import numpy as np
import pytest
import torch

from oracle import bitplane_oracle as O
from tests.helpers import CASES, load, load_config0

pytestmark = pytest.mark.gpu
KEYS = ["t", "pairs", "npairs", "act", "nact", "cls", "clsn"]


@pytest.mark.parametrize("name", CASES)
def test_plan_golden(name):
    from fathom_b200 import bitplane as bp
    z = load(name)
    plan = bp.make_plan(torch.from_numpy(z["g"]).cuda(), float(z["budget"]))
    for k in KEYS:
        assert np.array_equal(plan[k].cpu().numpy(), z["plan_" + k]), k


def test_plan_config0():
    from fathom_b200 import bitplane as bp
    from fathom_b200.synth import make_config0
    meta, _ = load_config0()
    d = make_config0("cpu")
    plan = bp.make_plan(d["g"].cuda(), meta["budget"])
    assert plan["t"].cpu().tolist() == meta["t"]
    assert bp.bytes_planes(plan["t"], 16384) == meta["bytes_planes"]


def test_worked_example_plan():
    from fathom_b200 import bitplane as bp
    z = load("kat")
    g = torch.zeros(1, 128)
    g[0, :4] = torch.from_numpy(z["g"][0])
    for B, want in ((8.0, [4, 3, 1, 0]), (6.0, [3, 2, 1, 0])):
        plan = bp.make_plan(g.cuda(), B)
        assert plan["t"][0, :4].cpu().tolist() == want
        assert int(plan["npairs"][0]) == sum(want)


@pytest.mark.parametrize("seed", range(6))
@pytest.mark.parametrize("bmax", [4, 3, 1])
def test_plan_random_vs_oracle(seed, bmax):
    from fathom_b200 import bitplane as bp
    gen = torch.Generator().manual_seed(seed)
    BH = 37
    g = (torch.randn(BH, 128, generator=gen) * 3).exp() * torch.rand(BH, 128, generator=gen)
    g[0, :10] = 0.0                                      # zero gains clamp to 1e-30
    g[1] = 4.0 ** torch.arange(128).remainder(7)         # exact powers: ties resolved half-to-even
    budget = torch.rand(BH, generator=gen) * 200
    budget[2] = 0.0
    budget[3] = 1e6
    for iters in (30, 0, 7, 45):
        plan = bp.make_plan(g.cuda(), budget.cuda(), bmax=bmax, iters=iters)
        ref = O.make_plan(g.numpy(), budget.numpy(), bmax=bmax, iters=iters)
        for k in KEYS:
            assert np.array_equal(plan[k].cpu().numpy(), ref[k]), (k, iters)
    plan = bp.make_plan(g.cuda(), 48.0, bmax=bmax)
    ref = O.make_plan(g.numpy(), 48.0, bmax=bmax)
    assert np.array_equal(plan["t"].cpu().numpy(), ref["t"])
