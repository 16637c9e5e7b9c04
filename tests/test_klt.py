"""Host logic of the KLT-rotated store (planesK) and per-layer budgets, on CPU: the per-layer budget
allocator against the reference's own `allocate` (scripts/l4_final_alloc.py:143-154, fixtures made by
tests/golden/make_golden_klt.py) and the basis checks."""
import os

import numpy as np
import pytest
import torch

from fathom_b200 import klt


def _klt():
    return np.load(os.path.join(os.path.dirname(__file__), "golden", "klt.npz"))


@pytest.mark.parametrize("a", ("a1", "a2", "a3"))
def test_allocate_layer_budgets_matches_reference(a):
    z = _klt()
    budgets = [int(b) for b in z[f"{a}_budgets"]]
    E = z[f"{a}_err"]
    err = {B: {L: float(E[i, L]) for L in range(E.shape[1])} for i, B in enumerate(budgets)}
    alloc = klt.allocate_layer_budgets(err, budgets, float(z[f"{a}_target"]))
    assert [alloc[L] for L in range(E.shape[1])] == z[f"{a}_alloc"].tolist()
    assert sum(alloc.values()) / len(alloc) >= float(z[f"{a}_target"])


def test_allocate_layer_budgets_edges():
    budgets = [24, 48, 96]
    flat = {B: {0: 1.0, 1: 1.0} for B in budgets}                 # no layer gains: ties go to the first layer
    assert klt.allocate_layer_budgets(flat, budgets, 36) == {0: 48, 1: 24}
    assert klt.allocate_layer_budgets(flat, budgets, 24) == {0: 24, 1: 24}
    assert klt.allocate_layer_budgets(flat, budgets, 500) == {0: 96, 1: 96}   # every layer at the top: stops
    worse = {24: {0: 0.0}, 48: {0: 100.0}, 96: {0: 200.0}}         # a step losing > 1 per unit is never taken
    assert klt.allocate_layer_budgets(worse, budgets, 96) == {0: 24}


def test_basis_shapes_are_checked():
    b = klt.KLTBasis(torch.zeros(2, 128), torch.zeros(2, 128, 128), torch.zeros(2, 128))
    assert b.checked(2, "cpu").Vt.shape == (2, 128, 128)
    with pytest.raises(ValueError, match="KLTBasis"):
        b.checked(3, "cpu")
    with pytest.raises(ValueError, match="KLTBasis"):
        klt.KLTBasis(torch.zeros(2, 128), torch.zeros(2, 128, 64), torch.zeros(2, 128)).checked(2, "cpu")
