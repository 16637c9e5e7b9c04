"""KLT-rotated store (planesK) on the GPU against the reference's own outputs (fixtures made by
running scripts/R_ruler.py's planesK store and scorer, tests/golden/make_golden_klt.py) and the oracle.

Bars: the rotation within fp32 summation rounding of the reference's; the store bit-exact against the
reference quantiser applied to the rotation the kernel produced; codes against the reference's own
codes equal except next to a code boundary (the two fp32 rotations sum in different orders); the
query rotation and gains within fp32 rounding, the plan bit-exact; scores within 1e-3 of the
reference scorer (which dequantises with fp32 block scales where the store keeps fp16 ones)."""
import os

import numpy as np
import pytest
import torch

from oracle import bitplane_oracle as O
from tests.helpers import score_rel_err, topk_sets_agree

pytestmark = pytest.mark.gpu

CASES = ("k1", "k2", "k3")


def _fixture():
    return np.load(os.path.join(os.path.dirname(__file__), "golden", "klt.npz"))


def _basis(z, c):
    from fathom_b200.klt import KLTBasis
    return KLTBasis(*(torch.from_numpy(z[f"{c}_{k}"]).cuda() for k in ("mu", "Vt", "lam")))


def _K(z, c):
    return torch.from_numpy(O.bf16_to_f32(z[f"{c}_K_bf16"].view(np.uint16))).cuda()


@pytest.mark.parametrize("c", CASES)
def test_klt_store_matches_reference(c):
    from fathom_b200 import bitplane as bp, klt
    z = _fixture()
    K, basis = _K(z, c), _basis(z, c)
    Kf = K.cpu().numpy()
    bound = O.klt_rotate_bound(Kf, z[f"{c}_mu"], z[f"{c}_Vt"])
    Kr = klt.klt_rotate(K, basis).cpu().numpy()
    assert np.all(np.abs(Kr - z[f"{c}_Kr"]) <= 2e-5 * bound + 1e-30)

    st = klt.KLTPlaneStore(K, basis)
    # the store is the reference quantiser of the rotation the kernel computed, bit for bit
    code, amax = O.quantise_u4(Kr, "f32")
    planes_k, scales_k = O.to_superblocks(O.pack_planes(code), amax.astype(np.float16), bp.SUB)
    assert np.array_equal(st.planes_k.cpu().numpy().view(np.uint64), planes_k)
    assert np.array_equal(st.scales_k.cpu().numpy().view(np.uint16), scales_k.view(np.uint16))
    assert np.array_equal(st.scales_blk.cpu().numpy(), amax)
    # against the reference's own codes: equal except at a boundary the two fp32 rotations straddle
    ref_code = z[f"{c}_code"]
    diff = st.code.cpu().numpy().astype(np.int32) - ref_code
    if np.any(diff):
        nb = O.nblocks(K.shape[1])
        s = np.repeat(z[f"{c}_amax"].astype(np.float64) / 8, 64, axis=1)[:, :K.shape[1]]
        x = z[f"{c}_Kr"].astype(np.float64) / s
        near = np.abs(x - np.round(x)) < 1e-3
        assert np.all(np.abs(diff) <= 1) and np.all(near[diff != 0]), "a code differs away from a boundary"
        assert np.count_nonzero(diff) <= 1e-3 * diff.size + 1, nb

    qr, gains = st.query(torch.from_numpy(z[f"{c}_q"]).cuda())
    qb = np.einsum("hgd,hde->hge", np.abs(z[f"{c}_q"]).astype(np.float64), np.abs(z[f"{c}_Vt"]).astype(np.float64))
    assert np.all(np.abs(qr.cpu().numpy() - z[f"{c}_qr"]) <= 2e-5 * qb + 1e-30)
    g = gains.cpu().numpy()
    assert np.all(np.abs(g - z[f"{c}_gains"]) <= 1e-4 * np.abs(z[f"{c}_gains"]) + 1e-30)
    plan = bp.make_plan(gains, float(z[f"{c}_Br"]))
    assert np.array_equal(plan["t"].cpu().numpy(), z[f"{c}_t"])
    s = st.scan(qr, plan).cpu().numpy()
    assert score_rel_err(s, z[f"{c}_scores"]) < 1e-3
    # and the same scan as the oracle chain over the kernel's own store (fp16 scales)
    ref = O.scan_scores(qr.cpu().numpy(), code, amax.astype(np.float16), z[f"{c}_t"])
    assert score_rel_err(s, ref) < 1e-5


def test_klt_basis_matches_oracle():
    from fathom_b200 import klt
    z = _fixture()
    K = _K(z, "k1")
    b = klt.klt_basis(K)
    mu, V, lam = O.klt_basis(K.cpu().numpy())
    assert np.abs(b.mu.cpu().numpy() - mu).max() <= 1e-6 * np.abs(mu).max()
    Vt, lt = b.Vt.cpu().numpy().astype(np.float64), b.lam.cpu().numpy().astype(np.float64)
    C = np.einsum("hde,he,hfe->hdf", V, lam, V)
    assert np.abs(np.einsum("hde,he,hfe->hdf", Vt, lt, Vt) - C).max() <= 1e-5 * np.abs(C).max()
    assert np.abs(np.einsum("hde,hdf->hef", Vt, Vt) - np.eye(128)).max() < 1e-5      # orthonormal columns


@pytest.mark.parametrize("G,n,kv", [(4, 20000, torch.bfloat16), (7, 9000, torch.float32), (1, 777, torch.float16)])
def test_klt_random_vs_oracle(G, n, kv):
    """Basis from the keys themselves (self_klt), store from the fused kernel, rotated query, plan and
    scan; HBM order and host run order give the same bits."""
    from fathom_b200 import bitplane as bp, klt
    from fathom_b200.synth import make_layer
    d = make_layer(3, G, n, seed=n + G, with_v=False)
    mix = torch.linalg.qr(torch.randn(3, 128, 128, generator=torch.Generator().manual_seed(5)))[0]
    K = (d["K"] @ mix + 1.5).to(kv).cuda()
    q = (d["q"] @ mix).cuda()
    basis = klt.klt_basis(K)
    st = klt.KLTPlaneStore(K, basis)
    qr, gains = st.query(q)
    plan = bp.make_plan(gains, 48.0)
    s = st.scan(qr, plan)
    Kr = klt.klt_rotate(K, basis).cpu().numpy()
    Kref = O.klt_rotate(K.float().cpu().numpy(), basis.mu.cpu().numpy(), basis.Vt.cpu().numpy())
    bound = O.klt_rotate_bound(K.float().cpu().numpy(), basis.mu.cpu().numpy(), basis.Vt.cpu().numpy())
    assert np.all(np.abs(Kr - Kref) <= 1e-5 * bound + 1e-30)
    code, amax = O.quantise_u4(Kr, "f32")
    Vt, lam = basis.Vt.cpu().numpy(), basis.lam.cpu().numpy()
    qo, go = O.klt_query(q.cpu().numpy(), Vt, lam)
    # directions of small eigenvalue take their q @ Vt from cancelling terms: bound by |q| @ |Vt|
    qb = np.einsum("hgd,hde->hge", np.abs(q.cpu().numpy()).astype(np.float64), np.abs(Vt).astype(np.float64))
    assert np.all(np.abs(qr.cpu().numpy() - qo) <= 2e-5 * qb + 1e-30)
    gtol = 1e-4 * np.abs(go) + 1e-5 * (qb ** 2 * lam[:, None]).sum(1)
    assert np.all(np.abs(gains.cpu().numpy() - go) <= gtol)
    ref = O.scan_scores(qr.cpu().numpy(), code, amax.astype(np.float16), plan["t"].cpu().numpy())
    assert score_rel_err(s.cpu().numpy(), ref) < 1e-5
    old = bp.SUB
    try:
        bp.SUB = O.nblocks(n)
        sN = klt.KLTPlaneStore(K, basis).scan(qr, plan)
    finally:
        bp.SUB = old
    assert torch.equal(s, sN)


@pytest.mark.parametrize("host", [False, True])
def test_klt_decode_step_vs_oracle(host):
    """decode_step over a KLT store (HBM or host-resident) plans on the rotated gains, scans the rotated
    queries and attends with the original queries; selection and attention match the oracle chain."""
    from fathom_b200 import klt
    from fathom_b200.offload import HostPlaneStore, MappedBuffer, decode_step
    from fathom_b200.synth import make_layer
    n, G, kk = 30000, 4, 580
    d = make_layer(2, G, n, seed=11, kv_dtype=torch.bfloat16, with_v=True)
    K, V, q = d["K"].cuda(), d["V"].cuda(), d["q"].cuda()
    basis = klt.klt_basis(K)
    if host:
        st = HostPlaneStore(K, torch.float32, basis=basis)
        kb, vb = MappedBuffer(K.shape, torch.bfloat16), MappedBuffer(V.shape, torch.bfloat16)
        kb.host.copy_(d["K"])
        vb.host.copy_(d["V"])
        Ks, Vs = kb.dev, vb.dev
    else:
        st = klt.KLTPlaneStore(K, basis)
        Ks, Vs = K, V
    scores = torch.empty(2, G, n, device="cuda")
    out, idx = decode_step(q, None, 48.0, st, Ks, Vs, n, kk, 4, 64, scores=scores)
    torch.cuda.synchronize()
    qr, gains = klt.klt_query(q, basis)
    Kr = klt.klt_rotate(K, basis).cpu().numpy()
    code, amax = O.quantise_u4(Kr, "f32")
    t = O.plan_depths(gains.cpu().numpy(), 48.0)
    ref_s = O.scan_scores(qr.cpu().numpy(), code, amax.astype(np.float16), t)
    assert score_rel_err(scores.cpu().numpy(), ref_s) < 1e-5
    got = idx.cpu().numpy()
    masked = scores.cpu().numpy().copy()
    masked[..., :4] = -np.inf
    masked[..., n - 64:] = -np.inf
    ref_idx = O.sink_local_topk(scores.cpu().numpy(), kk, 4, 64)
    assert topk_sets_agree(masked, got, ref_idx, kk - 68)
    f = lambda x: O.bf16_to_f32(x.contiguous().view(torch.int16).numpy().view(np.uint16))
    ref = O.decode_attention(d["q"].numpy(), f(d["K"]), f(d["V"]), got)
    o = out.cpu().numpy()
    assert np.abs(o - ref).max() <= 1e-5 * np.abs(ref).max() + 1e-6
    if host:
        kb.free()
        vb.free()
        st.free()
