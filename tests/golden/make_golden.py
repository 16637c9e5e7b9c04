"""Generate the golden fixtures by running the REAL reference implementation.

Run here, where the reference checkout is readable (it is not on the GPU box):

    TRITON_INTERPRET=1 python tests/golden/make_golden.py /path/to/reference

It imports the reference's `kernels/bitplane.py` (torch, CPU) and writes
`tests/golden/*.npz` and `tests/golden/config0.json`.  The CPU oracle is pinned
against these files; the CUDA path is checked against the oracle and, where the
fixture holds full tensors, against the fixtures directly.

Cases
  kat      the paper's worked example (paper/main.tex:298-326)
  s1       BH=2, n=700, G=4, budget 48; also the reference Triton `cls` and `fma`
           scan kernels run under TRITON_INTERPRET=1
  s2       BH=1, n=1025, G=7 (Qwen2.5 group size), budget 40
  s3       edge values: all-zero blocks, fp16 amax overflow / underflow, n=130
  s4       budget 0 and budget 512 (no channel / every plane), n=200
  config0  the full config-0 workload (8 KV heads, G=4, T=16384, budget 48,
           k=580 with 4 sink + 64 local): hashes, plan, top-k indices, score samples
"""
import hashlib
import json
import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def plan_lists(bp, g, budget):
    """The reference's plan lists, built from make_plan_torch's depths the way
    plan_kernel compacts them (kernels/bitplane.py:96-106); plan_kernel itself
    does not run under the Triton interpreter (libdevice.rint)."""
    t = bp.make_plan_torch(g, budget).to(torch.int32)
    BH, d = t.shape
    out = {"t": t.to(torch.int8).numpy(), "pairs": np.zeros((BH, d * 4), np.int32), "npairs": np.zeros(BH, np.int32),
           "act": np.zeros((BH, d), np.int32), "nact": np.zeros(BH, np.int32),
           "cls": np.zeros((BH, 4, d), np.int32), "clsn": np.zeros((BH, 4), np.int32)}
    for b in range(BH):
        tb = t[b].tolist()
        act = [j for j in range(d) if tb[j] > 0]
        out["act"][b, :len(act)] = act; out["nact"][b] = len(act)
        pr = [j * 4 + p for j in range(d) for p in range(tb[j])]
        out["pairs"][b, :len(pr)] = pr; out["npairs"][b] = len(pr)
        for c in range(1, 5):
            ch = [j for j in range(d) if tb[j] == c]
            out["cls"][b, c - 1, :len(ch)] = ch; out["clsn"][b, c - 1] = len(ch)
    return out


def store_outputs(bp, K, budget_g, q):
    n = K.shape[1]
    nb = math.ceil(n / bp.BLK)
    code, sc = bp.quantise_u4(K.float())
    planes = bp.pack_planes(code)
    res = {"code": code.numpy(), "scales": sc.view(torch.int16).numpy(), "planes": planes.numpy()}
    bp.SUB, bp.SBT = 16, 64 * 16
    pk, sk = bp.to_superblocks(planes, sc.to(torch.float16))
    res["planes_k16"], res["scales_k16"] = pk.numpy(), sk.view(torch.int16).numpy()
    bp.SUB, bp.SBT = nb, 64 * nb
    pk, sk = bp.to_superblocks(planes, sc.to(torch.float16))
    res["planes_kN"], res["scales_kN"] = pk.numpy(), sk.view(torch.int16).numpy()
    bp.SUB, bp.SBT = 16, 64 * 16
    assert torch.equal(bp.unpack_planes(planes, n), code)
    return res, code, sc


def case(bp, name, K, q, g, budget, k=None, sink=4, local=32, triton_scan=False):
    res, code, sc = store_outputs(bp, K, budget, q)
    pl = plan_lists(bp, g, budget)
    res.update({f"plan_{k_}": v for k_, v in pl.items()})
    t = torch.from_numpy(pl["t"]).long()
    scores = bp.scan_planes_reference(q, code, sc, t)
    res["scores"] = scores.numpy()
    res["bytes_planes"] = np.float64(bp.bytes_planes(t, K.shape[1]))
    if k is not None:
        res["topk"] = bp.sink_local_topk(scores, k, sink, local).numpy()
        res["topk_k"], res["topk_sink"], res["topk_local"] = np.int64(k), np.int64(sink), np.int64(local)
    if triton_scan:
        st = bp.PlaneStore(K.float())
        plan = {"t": torch.from_numpy(pl["t"]), "pairs": torch.from_numpy(pl["pairs"]), "npairs": torch.from_numpy(pl["npairs"]),
                "act": torch.from_numpy(pl["act"]), "nact": torch.from_numpy(pl["nact"]),
                "cls": torch.from_numpy(pl["cls"]), "clsn": torch.from_numpy(pl["clsn"])}
        bp.PlaneStore.kernel = "cls"; res["scores_triton_cls"] = st.scan(q, plan).numpy()
        bp.PlaneStore.kernel = "fma"; res["scores_triton_fma"] = st.scan(q, plan).numpy()
        bp.PlaneStore.kernel = "cls"
    K16 = K.to(torch.bfloat16)
    assert torch.equal(K16.float(), K.float())
    res.update({"K_bf16": K16.view(torch.int16).numpy(), "q": q.numpy(), "g": g.numpy(), "budget": np.float32(budget)})
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **res)
    print(f"wrote {name}.npz")


def bf16_keys(gen, BH, n, D=128):
    scale = torch.randn(BH, 1, D, generator=gen).exp()
    return (torch.randn(BH, n, D, generator=gen) * scale).to(torch.bfloat16).float(), scale


def main(ref_root):
    sys.path.insert(0, os.path.join(ref_root, "kernels"))
    import bitplane as bp
    torch.set_grad_enabled(False)

    # --- worked example (paper/main.tex:298-326)
    Kx = torch.tensor([[1.8, 0.4, -0.2, 0.05], [-1.1, 0.9, 0.3, -0.02], [0.3, -1.2, 0.1, 0.04],
                       [1.2, 0.7, 0.4, 0.01], [-0.6, -0.3, -0.5, 0.03], [0.9, 1.1, -0.3, -0.05]])
    qx = torch.tensor([[[3.0, 1.0, 2.0, 0.1], [1.0, 2.0, -1.0, 0.2]]])
    gx = torch.tensor([[12.22, 3.77, 0.63, 0.0]])
    code, sc = bp.quantise_u4(Kx[None])
    t8 = bp.make_plan_torch(gx, 8); t6 = bp.make_plan_torch(gx, 6)
    s8 = bp.scan_planes_reference(qx, code, sc, t8.long())
    np.savez_compressed(os.path.join(HERE, "kat.npz"), K=Kx.numpy(), q=qx.numpy(), g=gx.numpy(), code=code.numpy(),
                        scales=sc.view(torch.int16).numpy(), t8=t8.numpy(), t6=t6.numpy(), scores8=s8.numpy())
    print("kat: t8", t8.tolist(), "t6", t6.tolist(), "codes ch2", code[0, :, 2].tolist(), "head B", s8[0, 1].tolist())

    gen = torch.Generator().manual_seed(1)
    K, scale = bf16_keys(gen, 2, 700)
    q = torch.randn(2, 4, 128, generator=gen) * scale
    g = ((q ** 2) * K.var(1)[:, None]).sum(1)
    case(bp, "s1", K, q, g, 48.0, k=100, sink=4, local=32, triton_scan=os.environ.get("TRITON_INTERPRET") == "1")

    K, scale = bf16_keys(gen, 1, 1025)
    q = torch.randn(1, 7, 128, generator=gen) * scale
    g = ((q ** 2) * K.var(1)[:, None]).sum(1)
    case(bp, "s2", K, q, g, 40.0, k=150, sink=4, local=64)

    K, scale = bf16_keys(gen, 2, 130)
    K[0, :64, 0:8] = 0.0                         # all-zero block: fp16 amax underflows to 0, 0/0 -> code 0
    K[0, 64:, 8] = 2e-8                           # amax below fp16's subnormal range: s = 0, x/s = inf -> code 15
    K[0, :, 9] = 7.0e4                            # amax rounds to fp16 inf: s = inf, x/s = 0 -> code 8
    K[1, :64, 10] = 1.0e-6                         # fp16 subnormal amax
    K[1, 5, 11] = -3.0; K[1, :64, 11] = K[1, :64, 11] * 0 + 0.25; K[1, 5, 11] = -3.0
    K = K.to(torch.bfloat16).float()
    q = torch.randn(2, 4, 128, generator=gen) * scale
    g = ((q ** 2) * K.var(1)[:, None]).sum(1)
    case(bp, "s3", K, q, g, 56.0, k=40, sink=4, local=16)

    K, scale = bf16_keys(gen, 2, 200)
    q = torch.randn(2, 4, 128, generator=gen) * scale
    g = ((q ** 2) * K.var(1)[:, None]).sum(1)
    case(bp, "s4_b0", K, q, g, 0.0, k=60, sink=4, local=32)
    case(bp, "s4_b512", K, q, g, 512.0, k=60, sink=4, local=32)

    # --- config 0 (full size): hashes + plan + top-k
    from fathom_b200.synth import make_config0
    d = make_config0("cpu")
    K, q, g = d["K"], d["q"], d["g"]
    code, sc = bp.quantise_u4(K)
    planes = bp.pack_planes(code)
    bp.SUB, bp.SBT = 16, 1024
    pk, sk = bp.to_superblocks(planes, sc.to(torch.float16))
    nb = math.ceil(K.shape[1] / 64)
    bp.SUB, bp.SBT = nb, 64 * nb
    pkN, skN = bp.to_superblocks(planes, sc.to(torch.float16))
    bp.SUB, bp.SBT = 16, 1024
    t = bp.make_plan_torch(g, 48.0)
    scores = bp.scan_planes_reference(q, code, sc, t.long())
    idx = bp.sink_local_topk(scores, 580, 4, 64)
    rng = np.random.RandomState(0)
    samp = rng.randint(0, scores.numel(), 4096)
    meta = {"shape": {"BH": 8, "G": 4, "T": 16384, "D": 128}, "budget": 48.0, "k": 580, "sink": 4, "local": 64,
            "sha_K": sha(K.numpy()), "sha_q": sha(q.numpy()), "sha_g": sha(g.numpy()),
            "sha_code": sha(code.numpy()), "sha_scales": sha(sc.view(torch.int16).numpy()),
            "sha_planes_k16": sha(pk.numpy()), "sha_scales_k16": sha(sk.view(torch.int16).numpy()),
            "sha_planes_kN": sha(pkN.numpy()), "sha_scales_kN": sha(skN.view(torch.int16).numpy()),
            "t": t.to(torch.int8).tolist(), "bytes_planes": bp.bytes_planes(t, K.shape[1]),
            "score_max_abs": float(scores.abs().max()), "score_sample_idx": samp.tolist(),
            "score_sample": scores.reshape(-1)[torch.from_numpy(samp)].tolist()}
    json.dump(meta, open(os.path.join(HERE, "config0.json"), "w"))
    np.savez_compressed(os.path.join(HERE, "config0_topk.npz"), topk=idx.numpy().astype(np.uint16))
    print("config0: nact", (t > 0).sum(-1).tolist(), "bits/row", meta["bytes_planes"] * 8 / (16384 * 8))


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("FATHOM_REFERENCE", "../reference"))
