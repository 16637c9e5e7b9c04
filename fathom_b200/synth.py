"""Seeded synthetic inputs for the key-scan workloads.

The reference's real-data inputs (captured Qwen3-8B keys and queries) are not
available, so every workload here draws keys with the same shape and a
lognormal channel spread (the distribution `scripts/bench_scan_cfg.py:11-12`
uses uniform spreads; ours is lognormal(0, 1) per (KV head, channel)):

    scale[h, j] = exp(N(0, 1))
    K[h, t, j]  = N(0, 1) * scale[h, j]
    V[h, t, j]  = N(0, 1) * scale[h, j]
    q[h, g, j]  = N(0, 1) * scale[h, j]      (every query head of KV head h)
    g[h, j]     = sum_g q[h, g, j]^2 * Var_t(K[h, :, j])

`g` is the group-summed gain that the plan water-fills
(`scripts/bench_scan_cfg.py:12`, `scripts/B_e2e_offload_v2.py:181`).
"""
import torch


def make_layer(BH, G, T, D=128, seed=0, layer=0, device="cpu", kv_dtype=torch.float32, with_v=True,
               generator=None):
    """One layer's synthetic K (and V), q and g.

    Returns dict(K [BH,T,D] kv_dtype, V or None, q [BH,G,D] fp32, g [BH,D] fp32).
    The generator is seeded with 1000*seed + layer on `device`.
    """
    gen = generator or torch.Generator(device=device).manual_seed(1000 * seed + layer)
    scale = torch.randn(BH, 1, D, generator=gen, device=device).exp()
    K = torch.randn(BH, T, D, generator=gen, device=device) * scale
    V = torch.randn(BH, T, D, generator=gen, device=device) * scale if with_v else None
    q = torch.randn(BH, G, D, generator=gen, device=device) * scale
    Kf = K
    if kv_dtype != torch.float32:
        K = K.to(kv_dtype)
        V = V.to(kv_dtype) if V is not None else None
        Kf = K.float()
    g = ((q ** 2) * Kf.var(1)[:, None]).sum(1)
    return {"K": K, "V": V, "q": q, "g": g}


def make_config0(device="cpu"):
    """Config 0: Qwen3-8B attention shape, one layer, 8 KV heads x G=4, D=128,
    T=16384, fp32 keys; torch.manual_seed(0) semantics via a seeded generator."""
    return make_layer(8, 4, 16384, 128, seed=0, layer=0, device=device, kv_dtype=torch.float32)
