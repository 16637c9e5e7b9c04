"""HF decode integration (scripts/B_e2e_offload_v2.py:163-259) on the GPU: a small random-weight
Qwen3 model with its attention patched onto the offloaded key-scan path.

  * with k covering the whole context, the patched decode is dense attention: its logits match the
    unpatched model decoding with its own KV cache;
  * with k < context, one layer's decode attention (recent-token buffer, sink and local windows that
    reach into it, host or HBM index and rows, plain or KLT index) matches the oracle chain."""
import numpy as np
import pytest
import torch

from oracle import bitplane_oracle as O
from tests.helpers import score_rel_err, topk_sets_agree

pytestmark = pytest.mark.gpu


def _model(layers=2, heads=8, kv=2, seed=0):
    from transformers import Qwen3Config, Qwen3ForCausalLM
    torch.manual_seed(seed)
    cfg = Qwen3Config(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=layers,
                      num_attention_heads=heads, num_key_value_heads=kv, head_dim=128, max_position_embeddings=8192,
                      rope_theta=10000.0, attn_implementation="sdpa")
    return Qwen3ForCausalLM(cfg).to("cuda", torch.bfloat16).eval()


def _close(a, b, tol):
    a, b = a.float().cpu().numpy(), b.float().cpu().numpy()
    return float(np.abs(a - b).max() / np.abs(b).max()) < tol


@pytest.mark.parametrize("index,rows,klt", [("hbm", "hbm", False), ("host", "host", False), ("host", "host", True)])
def test_patched_decode_with_full_k_is_dense_decode(index, rows, klt):
    from fathom_b200.hf import OffloadedDecoder
    model = _model()
    B, n, steps = 2, 1500, 3
    ids = torch.randint(0, 512, (B, n + steps), device="cuda", generator=torch.Generator("cuda").manual_seed(1))
    with torch.no_grad():
        out = model(ids[:, :n], use_cache=True)
        past, ref_prefill = out.past_key_values, out.logits[:, -1]
        ref = []
        for s in range(steps):
            o = model(ids[:, n + s:n + s + 1], past_key_values=past, use_cache=True)
            past = o.past_key_values
            ref.append(o.logits[:, -1])
    # per-layer budgets (allocate_layer_budgets' output form): every layer plans on its own budget
    dec = OffloadedDecoder(model, k=600, index=index, rows=rows, klt=klt, max_new=8, prefill_chunk=512,
                           budget={0: 40, 1: 80})
    try:
        got_prefill = dec.prefill(ids[:, :n])
        assert _close(got_prefill, ref_prefill, 3e-2)
        dec.offload()
        for s in range(steps):
            dec.k = dec.context + 1              # every token: sinks + all prefill picks + local window
            logits = dec.decode(ids[:, n + s:n + s + 1])
            assert _close(logits, ref[s], 3e-2), s
            cos = torch.nn.functional.cosine_similarity(logits.float(), ref[s].float(), dim=-1)
            assert cos.min().item() > 0.999
    finally:
        dec.free()
        dec.unpatch()


@pytest.mark.parametrize("index,rows,klt", [("hbm", "hbm", False), ("host", "host", False), ("host", "hbm", True)])
def test_decode_attention_layer_vs_oracle(index, rows, klt):
    """One layer's offloaded decode attention after a few generated tokens (so the local window reaches
    into the recent buffer) against the oracle: store, plan, masked top-k, appended sinks and local
    window, attention over host and recent rows."""
    from fathom_b200 import klt as K_
    from fathom_b200.hf import SKIP, OffloadedDecoder
    from fathom_b200.synth import make_layer
    model = _model(layers=1)
    B, Hkv, G, n, k = 2, 2, 4, 5000, 580
    d = make_layer(B * Hkv, G, n, seed=5, kv_dtype=torch.bfloat16, with_v=True)
    K = d["K"].view(B, Hkv, n, 128).cuda()
    V = d["V"].view(B, Hkv, n, 128).cuda()
    dec = OffloadedDecoder(model, k=k, index=index, rows=rows, klt=klt, max_new=8)
    try:
        dec.load_kv(0, K, V)
        dec.offload()
        gen = torch.Generator("cuda").manual_seed(9)
        Kf = O.bf16_to_f32(d["K"].view(torch.int16).numpy().view(np.uint16))
        Vf = O.bf16_to_f32(d["V"].view(torch.int16).numpy().view(np.uint16))
        rk, rv = [], []
        for step in range(3):
            q = (torch.randn(B, Hkv * G, 1, 128, device="cuda", generator=gen) * d["q"].abs().mean()).bfloat16()
            kn = torch.randn(B, Hkv, 1, 128, device="cuda", generator=gen).bfloat16()
            vn = torch.randn(B, Hkv, 1, 128, device="cuda", generator=gen).bfloat16()
            out = dec._decode_attn(0, q, kn, vn)
            torch.cuda.synchronize()
            rk.append(kn.reshape(B * Hkv, 128).float().cpu().numpy())
            rv.append(vn.reshape(B * Hkv, 128).float().cpu().numpy())
        m = n + 3
        qf = q.reshape(B * Hkv, G, 128).float()
        if klt:
            basis = dec.cache[0].store.basis
            qs, g = K_.klt_query(qf, basis)
            Kr = K_.klt_rotate(d["K"].cuda(), basis).cpu().numpy()
            code, amax = O.quantise_u4(Kr, "f32")
            sc = amax.astype(np.float16)
            qs, g = qs.cpu().numpy(), g.cpu().numpy()
        else:
            code, sc = O.quantise_u4(Kf)
            var = torch.from_numpy(Kf[:, SKIP:]).var(1).numpy()
            qs = qf.cpu().numpy()
            g = (qs * qs * var[:, None]).sum(1)
        t = O.plan_depths(g, 48.0)
        scores = O.scan_scores(qs, code, sc, t)
        assert score_rel_err(dec._scores.cpu().numpy(), scores) < 1e-5
        idx = dec._idx.cpu().numpy()
        kk = k - 68
        masked = dec._scores.cpu().numpy().copy()
        masked[..., :4] = -np.inf
        masked[..., m - 64:] = -np.inf
        ref_top = O.topk_desc(masked, kk)
        assert topk_sets_agree(masked, idx, ref_top, kk)
        assert np.array_equal(idx[..., kk:kk + 4], np.broadcast_to(np.arange(4), (B * Hkv, G, 4)))
        assert np.array_equal(idx[..., kk + 4:], np.broadcast_to(np.arange(m - 64, m), (B * Hkv, G, 64)))
        recK = np.stack(rk, 1)
        recV = np.stack(rv, 1)
        ref = O.decode_attention(qf.cpu().numpy(), Kf, Vf, idx, recK, recV, n)
        o = out.reshape(B * Hkv, G, 128).float().cpu().numpy()
        assert np.abs(o - ref).max() <= 1e-2 * np.abs(ref).max()      # bf16 output rounding
    finally:
        dec.free()
        dec.unpatch()


@pytest.mark.parametrize("klt", [False, True])
def test_qwen2_without_qk_norm(klt):
    """A Qwen2-family model (no QK-norm, biased q/k/v projections; the case the KLT index is for):
    with k covering the whole context the patched decode matches the unpatched model's decode."""
    from transformers import Qwen2Config, Qwen2ForCausalLM
    from fathom_b200.hf import OffloadedDecoder
    torch.manual_seed(3)
    cfg = Qwen2Config(vocab_size=512, hidden_size=1024, intermediate_size=512, num_hidden_layers=2,
                      num_attention_heads=8, num_key_value_heads=2, head_dim=128, max_position_embeddings=8192,
                      attn_implementation="sdpa")
    model = Qwen2ForCausalLM(cfg).to("cuda", torch.bfloat16).eval()
    B, n, steps = 1, 1200, 2
    ids = torch.randint(0, 512, (B, n + steps), device="cuda", generator=torch.Generator("cuda").manual_seed(4))
    with torch.no_grad():
        out = model(ids[:, :n], use_cache=True)
        past, ref = out.past_key_values, []
        for s in range(steps):
            o = model(ids[:, n + s:n + s + 1], past_key_values=past, use_cache=True)
            past = o.past_key_values
            ref.append(o.logits[:, -1])
    dec = OffloadedDecoder(model, k=600, index="host", rows="host", klt=klt, max_new=4, prefill_chunk=512)
    try:
        dec.prefill(ids[:, :n])
        dec.offload()
        for s in range(steps):
            dec.k = dec.context + 1
            logits = dec.decode(ids[:, n + s:n + s + 1])
            assert _close(logits, ref[s], 3e-2), s
    finally:
        dec.free()
        dec.unpatch()


@pytest.mark.parametrize("index,rows", [("host", "host"), ("hbm", "hbm")])
def test_graph_decode_matches_eager(index, rows):
    """graphs=True: eager steps until the local window lies in the recent buffer, then one captured
    graph replayed per token.  Every step's logits equal the all-eager decoder's bit for bit."""
    from fathom_b200.hf import OffloadedDecoder
    model = _model()
    B, n, steps = 2, 1500, 14
    ids = torch.randint(0, 512, (B, n + steps), device="cuda", generator=torch.Generator("cuda").manual_seed(7))

    def run(graphs):
        dec = OffloadedDecoder(model, k=200, sink=4, local=8, index=index, rows=rows, max_new=16, graphs=graphs,
                               prefill_chunk=512)
        try:
            dec.prefill(ids[:, :n])
            dec.offload()
            out = [dec.decode(ids[:, n + s:n + s + 1]) for s in range(steps)]
            used = dec._graph is not None
        finally:
            dec.free()
            dec.unpatch()
        return out, used

    eager, _ = run(False)
    graph, used = run(True)
    assert used
    for s, (a, b) in enumerate(zip(eager, graph)):
        assert torch.equal(a, b), s
