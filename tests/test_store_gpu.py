"""Store build on the GPU: codes, scales, planes and both superblock orders bit-exact against the
reference's outputs (golden fixtures) and the oracle."""
import hashlib
import math

import numpy as np
import pytest
import torch

from oracle import bitplane_oracle as O
from tests.helpers import CASES, load, load_config0

pytestmark = pytest.mark.gpu


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def keys(z, dtype=torch.float32):
    K = torch.from_numpy(O.bf16_to_f32(z["K_bf16"].view(np.uint16))).cuda()
    return K.to(dtype)


@pytest.mark.parametrize("name", CASES)
@pytest.mark.parametrize("kdtype", [torch.float32, torch.bfloat16])
def test_quantise_pack_unpack_golden(name, kdtype):
    from fathom_b200 import bitplane as bp
    z = load(name)
    K = keys(z, kdtype)                     # the fixture keys are bf16-representable: both dtypes are exact
    code, sc = bp.quantise_u4(K)
    assert np.array_equal(code.cpu().numpy(), z["code"])
    assert np.array_equal(sc.cpu().view(torch.int16).numpy(), z["scales"])
    planes = bp.pack_planes(code)
    assert np.array_equal(planes.cpu().numpy(), z["planes"])
    assert torch.equal(bp.unpack_planes(planes, K.shape[1]), code)


@pytest.mark.parametrize("name", CASES)
def test_superblock_orders_golden(name):
    from fathom_b200 import bitplane as bp
    z = load(name)
    K = keys(z)
    n = K.shape[1]
    nb = math.ceil(n / 64)
    old = bp.SUB
    try:
        for sub, tag in ((16, "16"), (nb, "N")):
            bp.SUB = sub
            code, sc = bp.quantise_u4(K)
            pk, sk = bp.to_superblocks(bp.pack_planes(code), sc)
            assert np.array_equal(pk.cpu().numpy(), z[f"planes_k{tag}"])
            assert np.array_equal(sk.cpu().view(torch.int16).numpy(), z[f"scales_k{tag}"])
            st = bp.PlaneStore(K)
            assert np.array_equal(st.planes_k.cpu().numpy(), z[f"planes_k{tag}"])
            assert np.array_equal(st.scales_k.cpu().view(torch.int16).numpy(), z[f"scales_k{tag}"])
            assert st.nsb == math.ceil(nb / sub) and st.planes32.dtype == torch.int32
            assert np.array_equal(st.code.cpu().numpy(), z["code"])
            assert np.array_equal(st.scales_blk.cpu().view(torch.int16).numpy(), z["scales"])
            assert st.nbytes() == st.planes_k.numel() * 8 + st.scales_k.numel() * 2
    finally:
        bp.SUB = old


def test_fp16_keys_and_fp32_scales_match_oracle():
    from fathom_b200 import bitplane as bp
    g = torch.Generator().manual_seed(5)
    K = (torch.randn(3, 333, 128, generator=g) * torch.randn(3, 1, 128, generator=g).exp()).half()
    Kf = K.float().numpy()
    for kd in (torch.float16, torch.float32):
        code, sc = bp.quantise_u4(K.cuda().to(kd))
        c_ref, s_ref = O.quantise_u4(Kf)
        assert np.array_equal(code.cpu().numpy(), c_ref)
        assert np.array_equal(sc.cpu().numpy().view(np.int16), s_ref.view(np.int16))
    code, sc = bp.quantise_u4(K.cuda(), scale_dtype=torch.float32)
    c_ref, s_ref = O.quantise_u4(Kf, "f32")
    assert sc.dtype == torch.float32
    assert np.array_equal(code.cpu().numpy(), c_ref)
    assert np.array_equal(sc.cpu().numpy(), s_ref)
    st = bp.PlaneStore(K.cuda().float(), scale_dtype=torch.float32)
    assert np.array_equal(st.code.cpu().numpy(), c_ref)
    assert np.array_equal(st.scales_blk.cpu().numpy(), s_ref)
    pk, sk = O.to_superblocks(O.pack_planes(c_ref), s_ref.astype(np.float16), 16)
    assert np.array_equal(st.planes_k.cpu().numpy().view(np.uint64), pk)
    assert np.array_equal(st.scales_k.cpu().numpy().view(np.int16), sk.view(np.int16))


@pytest.mark.parametrize("n", [1, 63, 64, 65, 1023, 1024, 1025, 5000])
def test_ragged_lengths_match_oracle(n):
    from fathom_b200 import bitplane as bp
    g = torch.Generator().manual_seed(n)
    K = torch.randn(2, n, 128, generator=g) * torch.randn(2, 1, 128, generator=g).exp()
    st = bp.PlaneStore(K.cuda())
    c_ref, s_ref = O.quantise_u4(K.numpy())
    pk, sk = O.to_superblocks(O.pack_planes(c_ref), s_ref, 16)
    assert np.array_equal(st.planes_k.cpu().numpy().view(np.uint64), pk)
    assert np.array_equal(st.scales_k.cpu().numpy().view(np.int16), sk.view(np.int16))
    assert np.array_equal(st.code.cpu().numpy(), c_ref)


def test_config0_store_hashes():
    """Full config 0 (8 x 16384 x 128 fp32): both store orders hash-identical to the reference's."""
    from fathom_b200 import bitplane as bp
    from fathom_b200.synth import make_config0
    meta, _ = load_config0()
    d = make_config0("cpu")
    assert sha(d["K"].numpy()) == meta["sha_K"]
    K = d["K"].cuda()
    code, sc = bp.quantise_u4(K)
    assert sha(code.cpu().numpy()) == meta["sha_code"]
    assert sha(sc.cpu().view(torch.int16).numpy()) == meta["sha_scales"]
    old = bp.SUB
    try:
        bp.SUB = 16
        st = bp.PlaneStore(K)
        assert sha(st.planes_k.cpu().numpy()) == meta["sha_planes_k16"]
        assert sha(st.scales_k.cpu().view(torch.int16).numpy()) == meta["sha_scales_k16"]
        bp.SUB = 256
        st = bp.PlaneStore(K)
        assert sha(st.planes_k.cpu().numpy()) == meta["sha_planes_kN"]
        assert sha(st.scales_k.cpu().view(torch.int16).numpy()) == meta["sha_scales_kN"]
    finally:
        bp.SUB = old
