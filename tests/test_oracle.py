"""The CPU oracle against the reference's own outputs (golden fixtures) and the paper's
worked example.  CPU only."""
import hashlib
import os

import numpy as np
import pytest

from oracle import bitplane_oracle as O
from tests.helpers import CASES, SCORE_RTOL, load, load_config0, score_rel_err, topk_sets_agree


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.mark.parametrize("name", CASES)
def test_store_bit_exact(name):
    z = load(name)
    K = O.bf16_to_f32(z["K_bf16"].view(np.uint16))
    code, sc = O.quantise_u4(K)
    assert np.array_equal(code, z["code"])
    assert np.array_equal(sc.view(np.int16), z["scales"])
    planes = O.pack_planes(code)
    assert np.array_equal(planes.view(np.int64), z["planes"])
    assert np.array_equal(O.unpack_planes(planes, K.shape[1]), code)
    nb = O.nblocks(K.shape[1])
    for sub, tag in ((16, "16"), (nb, "N")):
        pk, sk = O.to_superblocks(planes, sc, sub)
        assert np.array_equal(pk.view(np.int64), z[f"planes_k{tag}"])
        assert np.array_equal(sk.view(np.int16), z[f"scales_k{tag}"])
        pl2, sc2 = O.from_superblocks(pk, sk, nb)
        assert np.array_equal(pl2, planes) and np.array_equal(sc2.view(np.int16), sc.view(np.int16))


@pytest.mark.parametrize("name", CASES)
def test_plan_bit_exact(name):
    z = load(name)
    plan = O.make_plan(z["g"], float(z["budget"]))
    for key, val in plan.items():
        assert np.array_equal(val, z["plan_" + key]), key
    assert O.bytes_planes(plan["t"], z["code"].shape[1]) == float(z["bytes_planes"])


@pytest.mark.parametrize("name", CASES)
def test_scan_matches_reference(name):
    z = load(name)
    s = O.scan_scores(z["q"], z["code"], z["scales"].view(np.float16), z["plan_t"])
    assert score_rel_err(s, z["scores"]) < 1e-6
    if "scores_triton_cls" in z:       # the reference's real Triton kernels agree with its torch reference
        assert score_rel_err(z["scores_triton_cls"], z["scores"]) < 1e-5
        assert score_rel_err(z["scores_triton_fma"], z["scores"]) < 1e-5


@pytest.mark.parametrize("name", [c for c in CASES if c != "s4_b0"])
def test_topk_matches_reference(name):
    z = load(name)
    k, sink, local = int(z["topk_k"]), int(z["topk_sink"]), int(z["topk_local"])
    idx = O.sink_local_topk(z["scores"], k, sink, local)
    kk = k - sink - local
    masked = z["scores"].copy()
    masked[..., :sink] = -np.inf
    masked[..., masked.shape[-1] - local:] = -np.inf
    assert topk_sets_agree(masked, idx, z["topk"], kk)
    assert np.array_equal(idx[..., kk:], z["topk"][..., kk:])          # sink + local tail, same order


def test_topk_all_ties_is_valid():
    """Budget 0: every score is 0, so any kk unmasked tokens are a valid top-k; the oracle takes
    the lowest indices (its index-ascending tie-break)."""
    z = load("s4_b0")
    assert np.all(z["scores"] == 0)
    k, sink, local = int(z["topk_k"]), int(z["topk_sink"]), int(z["topk_local"])
    idx = O.sink_local_topk(z["scores"], k, sink, local)
    kk = k - sink - local
    assert np.array_equal(idx[..., :kk], np.broadcast_to(np.arange(sink, sink + kk), idx[..., :kk].shape))


def test_worked_example():
    """paper/main.tex:298-326: depths (4,3,1,0) at B=8 and (3,2,1,0) at B=6; channel-2 codes
    (4,12,9,14,0,3); head B's approximate scores at depths (4,3,1,0) to two decimals."""
    z = load("kat")
    t8 = O.plan_depths(z["g"], 8.0)
    t6 = O.plan_depths(z["g"], 6.0)
    assert t8.tolist() == [[4, 3, 1, 0]] and t6.tolist() == [[3, 2, 1, 0]]
    assert np.array_equal(t8, z["t8"]) and np.array_equal(t6, z["t6"])
    code, sc = O.quantise_u4(z["K"][None])
    assert code[0, :, 2].tolist() == [4, 12, 9, 14, 0, 3]
    assert np.array_equal(code, z["code"])
    s = O.scan_scores(z["q"], code, sc, t8.astype(np.int64))
    assert [round(float(x), 2) for x in s[0, 1]] == [2.84, 0.24, -2.01, 2.49, -0.61, 3.36]
    assert [round(float(x), 2) for x in s[0, 0]] == [5.01, -1.79, 0.46, 4.96, -2.34, 3.59]
    assert np.allclose(s, z["scores8"], rtol=0, atol=1e-6)


def test_config0_plan_and_bytes():
    """Config 0 (8 KV heads, T=16384, budget 48): plan depths bit-exact against the reference; the
    inputs are regenerated from the seeded generator and hash-checked first."""
    import torch
    from fathom_b200.synth import make_config0
    meta, _ = load_config0()
    d = make_config0("cpu")
    assert sha(d["K"].numpy()) == meta["sha_K"], "torch CPU RNG stream changed: regenerate tests/golden"
    assert sha(d["g"].numpy()) == meta["sha_g"]
    t = O.plan_depths(d["g"].numpy(), meta["budget"])
    assert t.astype(np.int8).tolist() == meta["t"]
    assert O.bytes_planes(t, 16384) == meta["bytes_planes"]


def test_merge_candidates_is_global_topk():
    rng = np.random.RandomState(3)
    scores = rng.randn(3, 4000).astype(np.float32)
    full = O.topk_desc(scores, 100)
    chunks = np.array_split(np.arange(4000), 4)
    cs, ci = [], []
    for ch in chunks:
        local = O.topk_desc(scores[:, ch], 100)
        ci.append(ch[local])
        cs.append(np.take_along_axis(scores, ch[local], -1))
    merged = O.merge_candidates(np.concatenate(cs, -1), np.concatenate(ci, -1), 100)
    assert np.array_equal(merged, full)


CHAN4_CASES = ("c1", "c2", "c3", "c4")


@pytest.mark.parametrize("c", CHAN4_CASES)
def test_chan4_oracle_matches_reference(c):
    """pack_chan4, channel_list, bytes_chan4 and the chan4 scan against the reference's own outputs
    (scan_chan4_reference and, for power-of-two G, its Triton scan_chan4_kernel)."""
    z = np.load(os.path.join(os.path.dirname(__file__), "golden", "chan4.npz"))
    K = O.bf16_to_f32(z[f"{c}_K_bf16"].view(np.uint16))
    sub = int(z[f"{c}_sub"])
    code, sc = O.quantise_u4(K)
    assert np.array_equal(code, z[f"{c}_code"])
    assert np.array_equal(O.pack_chan4(code, sub), z[f"{c}_chan_k"])
    planes_k, scales_k = O.to_superblocks(O.pack_planes(code), sc, sub)
    assert np.array_equal(scales_k.view(np.int16), z[f"{c}_scales_k"])
    act, nact = O.channel_list(z[f"{c}_active"])
    assert np.array_equal(act, z[f"{c}_act"]) and np.array_equal(nact, z[f"{c}_nact"])
    assert O.bytes_chan4(nact, K.shape[1]) == float(z[f"{c}_bytes"])
    s = O.scan_chan4(z[f"{c}_q"], code, sc, z[f"{c}_active"])
    for key in (f"{c}_scores", f"{c}_scores_triton"):
        if key not in z.files:
            continue
        ref = z[key]
        # c3's fp16 amax overflow makes whole rows +-inf in the reference too: same positions and signs
        assert np.array_equal(np.isinf(s), np.isinf(ref)) and np.array_equal(s[np.isinf(s)], ref[np.isinf(ref)])
        fin = np.isfinite(ref).all(-1)
        assert score_rel_err(s[fin], ref[fin]) < 1e-5


KLT_CASES = ("k1", "k2", "k3")


def _klt():
    return np.load(os.path.join(os.path.dirname(__file__), "golden", "klt.npz"))


@pytest.mark.parametrize("c", KLT_CASES)
def test_klt_oracle_matches_reference(c):
    """planesK (scripts/R_ruler.py:63-64, 82-84) restated against the reference's own outputs: the
    rotation to fp32 summation rounding, the codes_u4 store bit-exact from the reference's rotated keys,
    the query rotation and gains, the plan bit-exact from the reference's gains, the scores."""
    z = _klt()
    K = O.bf16_to_f32(z[f"{c}_K_bf16"].view(np.uint16))
    mu, Vt, lam = z[f"{c}_mu"], z[f"{c}_Vt"], z[f"{c}_lam"]
    Kr = z[f"{c}_Kr"]
    bound = O.klt_rotate_bound(K, mu, Vt)
    assert np.all(np.abs(O.klt_rotate(K, mu, Vt) - Kr) <= 1e-5 * bound + 1e-30)
    code, amax = O.quantise_u4(Kr, "f32")
    assert np.array_equal(code, z[f"{c}_code"]) and np.array_equal(amax, z[f"{c}_amax"])
    qr, gains = O.klt_query(z[f"{c}_q"], Vt, lam)
    qbound = np.einsum("hgd,hde->hge", np.abs(z[f"{c}_q"]).astype(np.float64), np.abs(Vt).astype(np.float64))
    assert np.all(np.abs(qr - z[f"{c}_qr"]) <= 1e-5 * qbound + 1e-30)
    assert np.all(np.abs(gains - z[f"{c}_gains"]) <= 1e-5 * np.abs(z[f"{c}_gains"]) + 1e-30)
    t = O.plan_depths(z[f"{c}_gains"], float(z[f"{c}_Br"]))
    assert np.array_equal(t.astype(np.int8), z[f"{c}_t"])
    s = O.scan_scores(z[f"{c}_qr"], code, amax, t)
    assert score_rel_err(s, z[f"{c}_scores"]) < 1e-5


@pytest.mark.parametrize("c", KLT_CASES)
def test_klt_basis_matches_reference(c):
    """self_klt (scripts/R_agent.py:59-63): mean and covariance V diag(lam) V^T agree with the reference's
    fp32 eigendecomposition (the basis itself is unique only up to column signs)."""
    z = _klt()
    K = O.bf16_to_f32(z[f"{c}_K_bf16"].view(np.uint16))
    mu, V, lam = O.klt_basis(K)
    assert np.abs(mu - z[f"{c}_mu"]).max() <= 1e-5 * np.abs(mu).max()
    C = np.einsum("hde,he,hfe->hdf", V, lam, V)
    Vr, lr = z[f"{c}_Vt"].astype(np.float64), z[f"{c}_lam"].astype(np.float64)
    Cr = np.einsum("hde,he,hfe->hdf", Vr, lr, Vr)
    assert np.abs(C - Cr).max() <= 1e-4 * np.abs(C).max()
    assert np.abs(lam - lr).max() <= 1e-4 * lam.max()


@pytest.mark.parametrize("a", ("a1", "a2", "a3"))
def test_layer_budget_allocation_matches_reference(a):
    """allocate (scripts/l4_final_alloc.py:143-154) on seeded error tables: identical budgets."""
    z = _klt()
    budgets = [int(b) for b in z[f"{a}_budgets"]]
    E = z[f"{a}_err"]
    err = {B: {L: float(E[i, L]) for L in range(E.shape[1])} for i, B in enumerate(budgets)}
    alloc = O.allocate_layer_budgets(err, budgets, float(z[f"{a}_target"]))
    assert [alloc[L] for L in range(E.shape[1])] == z[f"{a}_alloc"].tolist()


def test_threaded_scan_equals_scan():
    """The thread-pool scan the CPU baseline times computes the same scores as scan_scores."""
    g = np.random.default_rng(7)
    K = (g.standard_normal((2, 5000, 128)) * np.exp(g.standard_normal((2, 1, 128)))).astype(np.float32)
    q = g.standard_normal((2, 4, 128)).astype(np.float32)
    code, sc = O.quantise_u4(K)
    t = g.integers(0, 5, (2, 128))
    a = O.scan_scores(q, code, sc, t)
    b = O.scan_scores_threaded(q, code, sc, t, threads=4, chunk=1000)
    assert np.allclose(a, b, rtol=0, atol=1e-5 * np.abs(a).max())
