"""The phase-interleaved HBM scan in every layout the launcher can pick (one or two phases per lane,
several tiles per warp, an odd last head) against the bulk-copy kernel, bit for bit, for G = 1..8:
plain scans, block ranges, and the fused scan + selection (group keys from the epilogue).

The layouts are forced with the launcher's tuning overrides (environment variables read at each call):
FATHOM_SCAN_P (phases per lane), FATHOM_SCAN_TPW (tiles per warp), FATHOM_SCAN_KERNEL=classic (the
bulk-copy kernel, the reference point)."""
import os

import numpy as np
import pytest
import torch

from oracle import bitplane_oracle as O
from tests.helpers import score_rel_err

pytestmark = pytest.mark.gpu

KNOBS = ("FATHOM_SCAN_P", "FATHOM_SCAN_TPW", "FATHOM_SCAN_KERNEL")


class _env:
    def __init__(self, **kw):
        self.kw = kw

    def __enter__(self):
        self.old = {k: os.environ.get(k) for k in KNOBS}
        for k in KNOBS:
            os.environ.pop(k, None)
        os.environ.update({k: str(v) for k, v in self.kw.items()})

    def __exit__(self, *exc):
        for k, v in self.old.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v


def _layer(BH, G, n, seed):
    from fathom_b200 import bitplane as bp
    from fathom_b200.synth import make_layer
    d = make_layer(BH, G, n, seed=seed, layer=3, device="cuda", kv_dtype=torch.bfloat16, with_v=False)
    return bp.PlaneStore(d["K"]), d["q"], d["g"], d["K"]


LAYOUTS = [dict(FATHOM_SCAN_P=1), dict(FATHOM_SCAN_P=2), dict(FATHOM_SCAN_P=2, FATHOM_SCAN_TPW=3),
           dict(FATHOM_SCAN_P=1, FATHOM_SCAN_TPW=5)]


@pytest.mark.parametrize("G", [1, 2, 3, 4, 5, 6, 7, 8])
def test_phase_layouts_equal_bulk_kernel(G):
    from fathom_b200 import bitplane as bp
    n = 64 * 333 + 17                                         # ragged: a partial last block and tile
    st, q, g, K = _layer(3, G, n, seed=G)
    plan = bp.make_plan(g, 48.0)
    with _env(FATHOM_SCAN_KERNEL="classic"):
        ref = st.scan(q, plan)
    for lay in LAYOUTS:
        with _env(**lay):
            got = st.scan(q, plan)
        assert torch.equal(got, ref), lay
    # and the oracle chain, once per G
    code, sc = O.quantise_u4(O.bf16_to_f32(K.cpu().contiguous().view(torch.int16).numpy().view(np.uint16)))
    assert score_rel_err(ref.cpu().numpy(), O.scan_scores(q.cpu().numpy(), code, sc, plan["t"].cpu().numpy())) < 1e-5


@pytest.mark.parametrize("G", [4, 7])
def test_phase_block_ranges(G):
    """Partial block ranges (tiles cut at both ends) write exactly their tokens."""
    from fathom_b200 import bitplane as bp
    n = 64 * 200 + 5
    st, q, g, _ = _layer(2, G, n, seed=40 + G)
    plan = bp.make_plan(g, 56.0)
    with _env(FATHOM_SCAN_KERNEL="classic"):
        full = st.scan(q, plan)
    for lay in LAYOUTS:
        with _env(**lay):
            out = torch.full_like(full, 7.0)
            for b0, b1 in ((3, 9), (17, 18), (40, 201)):
                st.scan(q, plan, out=out, blocks=(b0, b1))
        for b0, b1 in ((3, 9), (17, 18), (40, 201)):
            assert torch.equal(out[..., b0 * 64:min(n, b1 * 64)], full[..., b0 * 64:min(n, b1 * 64)]), lay
        assert torch.all(out[..., :3 * 64] == 7.0) and torch.all(out[..., 18 * 64:40 * 64] == 7.0)


@pytest.mark.parametrize("G", [1, 3, 4, 7, 8])
def test_phase_fused_select_equals_bulk_kernel(G):
    """scan_select (group keys from the phase kernel's epilogue) selects what the bulk-copy kernel's
    fused path selects, with the same scores."""
    from fathom_b200 import bitplane as bp
    n = 64 * 700 + 33
    st, q, g, _ = _layer(2, G, n, seed=70 + G)
    plan = bp.make_plan(g, 48.0)
    kk, sink, local = 500, 4, 64
    with _env(FATHOM_SCAN_KERNEL="classic"):
        ref_idx, ref_vals, ref_s = bp.scan_select(st, q, plan, kk, mask_lo=sink, mask_hi=n - local, append_sink=sink,
                                                  append_local=local, with_scores=True)
    for lay in LAYOUTS:
        with _env(**lay):
            idx, vals, s = bp.scan_select(st, q, plan, kk, mask_lo=sink, mask_hi=n - local, append_sink=sink,
                                          append_local=local, with_scores=True)
        assert torch.equal(s, ref_s) and torch.equal(idx, ref_idx) and torch.equal(vals, ref_vals), lay


def test_phase_budget_zero_and_full():
    """No active channel (every score 0) and every channel at depth 4."""
    from fathom_b200 import bitplane as bp
    n = 64 * 150
    st, q, g, _ = _layer(2, 4, n, seed=9)
    for budget in (0.0, 512.0):
        plan = bp.make_plan(g, budget)
        with _env(FATHOM_SCAN_KERNEL="classic"):
            ref = st.scan(q, plan)
        for lay in LAYOUTS:
            with _env(**lay):
                got = st.scan(q, plan)
            assert torch.equal(got, ref), (budget, lay)
        if budget == 0.0:
            assert torch.all(ref == 0)
