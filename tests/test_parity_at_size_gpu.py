"""Parity at the sizes the benchmark reports, against the oracle chain on the same seeded inputs.

  config 2: one layer of the host-resident decode step at T = 1,048,576 (2 of the 8 KV heads, G = 4,
            budget 48, k = 512 + 4 sink + 64 local), index and interleaved K/V rows in mapped host memory
  config 1: one layer of the HBM-resident step at its full shape (8 KV heads, G = 4, T = 131072)
  config 3: the full batched shape (8 sequences x 4 KV heads = 32 rows, G = 7, T = 131072,
            k = 2048 + 4 + 64) through the fused scan + selection, oracle-checked on sampled rows

Bars (the north star's, written here): plan depths bit-exact; scores within SCORE_RTOL (1e-3) of the
row's max |score| (measured ~1e-6); selected indices exactly the oracle's (score desc, index asc)
selection over the device scores, and the same index sets as the oracle's selection over its own
scores up to ties (TIE_EPS); attention within 1e-5 relative.
"""
import math

import numpy as np
import pytest
import torch

from oracle import bitplane_oracle as O
from tests.helpers import SCORE_RTOL, TIE_EPS, score_rel_err, topk_sets_agree

pytestmark = pytest.mark.gpu


def _bf16_np(x):
    return O.bf16_to_f32(x.contiguous().cpu().view(torch.int16).numpy().view(np.uint16))


def test_config2_layer_at_1m_tokens_host_resident():
    from fathom_b200 import bitplane as bp
    from fathom_b200.offload import HostPlaneStore, MappedBuffer, decode_step
    from fathom_b200.synth import make_layer
    BH, G, n, budget, k, sink, local = 2, 4, 1 << 20, 48.0, 580, 4, 64
    d = make_layer(BH, G, n, seed=2, layer=5, device="cuda", kv_dtype=torch.bfloat16, with_v=True)
    K, V, q, g = d["K"], d["V"], d["q"], d["g"]
    store = HostPlaneStore(K)
    kv = MappedBuffer((BH, n, 2, 128), torch.bfloat16, torch.device("cuda"))   # K and V of a token adjacent
    kv.dev[:, :, 0].copy_(K)
    kv.dev[:, :, 1].copy_(V)
    scores = torch.empty(BH, G, n, device="cuda")
    try:
        out, idx = decode_step(q, g, budget, store, kv.dev[:, :, 0], kv.dev[:, :, 1], n, k, sink, local,
                               scores=scores)
        torch.cuda.synchronize()
        plan = O.make_plan(g.cpu().numpy(), budget)
        assert np.array_equal(bp.make_plan(g, budget)["t"].cpu().numpy(), plan["t"])
        Kf, Vf = _bf16_np(K), _bf16_np(V)
        code, sc = O.quantise_u4(Kf)
        ref_scores = O.scan_scores(q.cpu().numpy(), code, sc, plan["t"])
        got_scores = scores.cpu().numpy()
        assert score_rel_err(got_scores, ref_scores) < SCORE_RTOL
        got_idx = idx.cpu().numpy()
        assert np.array_equal(got_idx, O.sink_local_topk(got_scores, k, sink, local))
        kk = k - sink - local
        masked = ref_scores.copy()
        masked[..., :sink] = -np.inf
        masked[..., n - local:] = -np.inf
        assert topk_sets_agree(masked, got_idx[..., :kk], O.sink_local_topk(ref_scores, k, sink, local)[..., :kk], kk,
                               TIE_EPS)
        ref = O.decode_attention(q.cpu().numpy(), Kf, Vf, got_idx)
        o = out.cpu().numpy()
        assert np.abs(o - ref).max() <= 1e-5 * np.abs(ref).max() + 1e-6
    finally:
        kv.free()
        store.free()


def test_config1_layer_full_shape_hbm():
    from fathom_b200 import bitplane as bp
    from fathom_b200 import offload as off
    from fathom_b200.synth import make_layer
    BH, G, n, budget, k, sink, local = 8, 4, 131072, 48.0, 580, 4, 64
    d = make_layer(BH, G, n, seed=1, layer=0, device="cuda", kv_dtype=torch.bfloat16, with_v=True)
    K, V, q, g = d["K"], d["V"], d["q"], d["g"]
    st = bp.PlaneStore(K)
    plan = bp.make_plan(g, budget)
    scores = torch.empty(BH, G, n, device="cuda")
    idx = bp.scan_topk(st, q, plan, k, sink, local, scores=scores)
    out = off.decode_attention(q, idx, K, V, n)
    torch.cuda.synchronize()
    oplan = O.make_plan(g.cpu().numpy(), budget)
    assert np.array_equal(plan["t"].cpu().numpy(), oplan["t"])
    Kf, Vf = _bf16_np(K), _bf16_np(V)
    code, sc = O.quantise_u4(Kf)
    ref_scores = O.scan_scores(q.cpu().numpy(), code, sc, oplan["t"])
    got_scores = scores.cpu().numpy()
    assert score_rel_err(got_scores, ref_scores) < SCORE_RTOL
    got_idx = idx.cpu().numpy()
    assert np.array_equal(got_idx, O.sink_local_topk(got_scores, k, sink, local))
    ref = O.decode_attention(q.cpu().numpy(), Kf, Vf, got_idx)
    assert np.abs(out.cpu().numpy() - ref).max() <= 1e-5 * np.abs(ref).max() + 1e-6


def test_config3_full_shape_scan_select():
    from fathom_b200 import bitplane as bp
    from fathom_b200.synth import make_layer
    B, Hkv, G, n, budget, k, sink, local = 8, 4, 7, 131072, 48.0, 2116, 4, 64
    BH = B * Hkv
    d = make_layer(BH, G, n, seed=3, layer=11, device="cuda", kv_dtype=torch.bfloat16, with_v=False)
    K, q, g = d["K"], d["q"], d["g"]
    st = bp.PlaneStore(K)
    plan = bp.make_plan(g, budget)
    kk = k - sink - local
    idx, vals, scores = bp.scan_select(st, q, plan, kk, mask_lo=sink, mask_hi=n - local, append_sink=sink,
                                       append_local=local, with_scores=True)
    torch.cuda.synchronize()
    got_scores = scores.cpu().numpy()
    got_idx = idx.cpu().numpy()
    # the selection of every row equals the oracle's over the device scores, with the selected scores
    assert np.array_equal(got_idx, O.sink_local_topk(got_scores, k, sink, local))
    assert np.array_equal(vals.cpu().numpy(), np.take_along_axis(got_scores, got_idx[..., :kk], -1))
    oplan = O.make_plan(g.cpu().numpy(), budget)
    assert np.array_equal(plan["t"].cpu().numpy(), oplan["t"])
    # scores of sampled rows (all 7 query heads each) against the oracle chain
    rows = [0, 9, 22, 31]
    Kf = _bf16_np(K[rows])
    code, sc = O.quantise_u4(Kf)
    ref_scores = O.scan_scores(q[rows].cpu().numpy(), code, sc, oplan["t"][rows])
    assert score_rel_err(got_scores[rows], ref_scores) < SCORE_RTOL
    masked = ref_scores.copy()
    masked[..., :sink] = -np.inf
    masked[..., n - local:] = -np.inf
    assert topk_sets_agree(masked, got_idx[rows][..., :kk], O.sink_local_topk(ref_scores, k, sink, local)[..., :kk],
                           kk, TIE_EPS)
