"""One layer of the host-resident decode step through the public API (offload.decode_step: plan ->
plane-prefix scan of a host-resident store -> sink+local top-k -> dedupe, gather and attention over
K/V rows in mapped host memory, with the newest rows in a device-resident recent buffer), checked
stage by stage against the oracle chain on the same seeded inputs."""
import numpy as np
import pytest
import torch

from oracle import bitplane_oracle as O
from tests.helpers import SCORE_RTOL, score_rel_err

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n,G,budget", [(20000, 4, 48.0), (9000, 7, 40.0), (70000, 4, 80.0)])
def test_host_decode_step_matches_oracle(n, G, budget):
    from fathom_b200 import bitplane as bp
    from fathom_b200.offload import HostPlaneStore, MappedBuffer, decode_step
    from fathom_b200.synth import make_layer
    BH, k, sink, local, rc = 2, 580, 4, 64, 16
    d = make_layer(BH, G, n, seed=n, layer=1, kv_dtype=torch.bfloat16, with_v=True)
    K, V, q, g = d["K"], d["V"], d["q"], d["g"]
    n_host = n - rc                                   # the last rc rows live in the recent buffer
    store = HostPlaneStore(K.cuda())
    kb = MappedBuffer((BH, n_host, 128), torch.bfloat16)
    vb = MappedBuffer((BH, n_host, 128), torch.bfloat16)
    kb.host.copy_(K[:, :n_host])
    vb.host.copy_(V[:, :n_host])
    Kr, Vr = K[:, n_host:].contiguous().cuda(), V[:, n_host:].contiguous().cuda()
    scores = torch.empty(BH, G, n, device="cuda")
    out, idx = decode_step(q.cuda(), g.cuda(), budget, store, kb.dev, vb.dev, n_host, k, sink, local,
                           n_host=n_host, K_recent=Kr, V_recent=Vr, recent_cap=rc, scores=scores)
    # oracle chain
    plan = O.make_plan(g.numpy(), budget)
    t = plan["t"] if isinstance(plan, dict) else plan[0]
    code, sc = O.quantise_u4(K.float().numpy())
    ref_scores = O.scan_scores(q.numpy(), code, sc, t)
    assert score_rel_err(scores.cpu().numpy(), ref_scores) < SCORE_RTOL
    got_idx = idx.cpu().numpy()
    # the device scores order the selection: identical to the oracle's selection over those scores
    assert np.array_equal(got_idx, O.sink_local_topk(scores.cpu().numpy(), k, sink, local))
    f = lambda x: O.bf16_to_f32(x.contiguous().view(torch.int16).numpy().view(np.uint16))
    ref = O.decode_attention(q.numpy(), f(K[:, :n_host]), f(V[:, :n_host]), got_idx, f(K[:, n_host:]),
                             f(V[:, n_host:]), n_host)
    o = out.cpu().numpy()
    assert np.abs(o - ref).max() <= 1e-5 * np.abs(ref).max() + 1e-6
    kb.free()
    vb.free()
    store.free()
