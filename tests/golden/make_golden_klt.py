"""Generate the KLT-rotated store (planesK) fixtures by running the REAL reference code.

Run here, where the reference checkout is readable (it is not on the GPU box):

    python tests/golden/make_golden_klt.py /path/to/reference

The reference's planesK scorer lives in evaluation scripts that parse arguments and load models at
import time, so the functions themselves are taken out of the script sources (Python's `ast`) and
executed unchanged in a namespace that holds the constants they use from `scripts/sketch.py`:

  * scripts/R_ruler.py   codes_u4, dequant, waterfill_t, Stores ("planesK:u4:Br" store and scorer)
  * scripts/R_agent.py   self_klt (the basis from the session's own keys)
  * scripts/l4_final_alloc.py  allocate (per-layer budgets from a calibration error table)

Writes `tests/golden/klt.npz`.  Cases (prefix in the archive)
  k1  BH=2, n=700, G=4, Br=48: correlated keys with a mean offset (a rotated lognormal channel spread)
  k2  BH=1, n=1025, G=7, Br=32
  k3  BH=2, n=37, G=2, Br=64: one partial block (pad tokens rotate to 0)
  a1..a3  allocate() on seeded error tables (mean targets 32 / 48 / 80)
"""
import ast
import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def extract(path, names, ns):
    tree = ast.parse(open(path).read(), path)
    body = [n for n in tree.body if isinstance(n, (ast.FunctionDef, ast.ClassDef)) and n.name in names]
    assert {n.name for n in body} == set(names), f"{path}: missing {set(names) - {n.name for n in body}}"
    exec(compile(ast.Module(body=body, type_ignores=[]), path, "exec"), ns)


def keys(gen, BH, n, D=128):
    scale = torch.randn(BH, 1, D, generator=gen).exp()
    mix = torch.linalg.qr(torch.randn(BH, D, D, generator=gen))[0]
    off = 2.0 * torch.randn(BH, 1, D, generator=gen)
    K = ((torch.randn(BH, n, D, generator=gen) * scale) @ mix + off).to(torch.bfloat16).float()
    return K, scale, mix


def case(ns, out, name, K, q, Br):
    p = ns["self_klt"](K)
    st = ns["Stores"](f"planesK:u4:{Br}", [p], 1, lambda L: K)
    n = K.shape[1]
    sc, bits = st.scores(q, 0, n)
    H = K.shape[0]
    codes = st.S[0]["codes"].reshape(H, -1, 128)[:, :n].to(torch.uint8)
    Kr = torch.einsum("hnd,hde->hne", K - p["mu"][:, None], p["Vt"])
    qr = torch.einsum("hgd,hde->hge", q, p["Vt"])
    g = ((qr ** 2) * p["lam"][:, None]).sum(1)
    t = ns["waterfill_t"](g, Br)
    out[f"{name}_K_bf16"] = K.to(torch.bfloat16).view(torch.int16).numpy()
    out[f"{name}_q"] = q.numpy()
    out[f"{name}_Br"] = np.float32(Br)
    out[f"{name}_mu"] = p["mu"].numpy()
    out[f"{name}_Vt"] = p["Vt"].numpy()
    out[f"{name}_lam"] = p["lam"].numpy()
    out[f"{name}_Kr"] = Kr.numpy()
    out[f"{name}_code"] = codes.numpy()
    out[f"{name}_amax"] = st.S[0]["amax"].squeeze(2).numpy()
    out[f"{name}_qr"] = qr.numpy()
    out[f"{name}_gains"] = g.numpy()
    out[f"{name}_t"] = t.numpy().astype(np.int8)
    out[f"{name}_scores"] = sc.numpy()
    out[f"{name}_bits"] = np.float64(bits)
    print(f"{name}: BH={H} n={n} G={q.shape[1]} Br={Br} bits/token={bits:.2f} nact={(t > 0).sum(-1).tolist()}")


def alloc_case(ns, out, name, gen, budgets, n_layers, target):
    # a convex-ish error curve per layer: err falls with budget at a layer-specific rate, plus noise
    rate = torch.rand(n_layers, generator=gen) * 0.08 + 0.01
    base = torch.rand(n_layers, generator=gen) + 0.5
    table = {}
    for B in budgets:
        e = base * torch.exp(-rate * B) + 0.002 * torch.rand(n_layers, generator=gen)
        table[B] = {L: float(e[L]) for L in range(n_layers)}
    ns["BUDGETS"] = tuple(budgets)
    ns["LAYERS"] = list(range(n_layers))
    ns["layer_mean"] = lambda split, nm: table[int(nm.split("planes")[-1])]
    alloc = ns["allocate"]("u4", target)
    out[f"{name}_budgets"] = np.array(budgets, np.int64)
    out[f"{name}_err"] = np.array([[table[B][L] for L in range(n_layers)] for B in budgets], np.float64)
    out[f"{name}_target"] = np.float64(target)
    out[f"{name}_alloc"] = np.array([alloc[L] for L in range(n_layers)], np.int64)
    print(f"{name}: target={target} alloc={[alloc[L] for L in range(n_layers)]}")


def main(ref_root):
    sys.path.insert(0, os.path.join(ref_root, "scripts"))
    import sketch
    torch.set_grad_enabled(False)
    ns = {"torch": torch, "math": math, "BLK": sketch.BLK, "SINK": sketch.SINK, "scale_bits": sketch.scale_bits,
          "dev": "cpu"}
    extract(os.path.join(ref_root, "scripts", "R_ruler.py"), ["codes_u4", "dequant", "waterfill_t", "Stores"], ns)
    extract(os.path.join(ref_root, "scripts", "R_agent.py"), ["self_klt"], ns)
    extract(os.path.join(ref_root, "scripts", "l4_final_alloc.py"), ["allocate"], ns)
    out = {}
    gen = torch.Generator().manual_seed(23)

    K, scale, mix = keys(gen, 2, 700)
    case(ns, out, "k1", K, (torch.randn(2, 4, 128, generator=gen) * scale) @ mix, 48)
    K, scale, mix = keys(gen, 1, 1025)
    case(ns, out, "k2", K, (torch.randn(1, 7, 128, generator=gen) * scale) @ mix, 32)
    K, scale, mix = keys(gen, 2, 37)
    case(ns, out, "k3", K, (torch.randn(2, 2, 128, generator=gen) * scale) @ mix, 64)

    budgets = [24, 32, 40, 48, 64, 80, 96, 128]          # scripts/l4_final_alloc.py:18
    alloc_case(ns, out, "a1", gen, budgets, 36, 32)
    alloc_case(ns, out, "a2", gen, budgets, 36, 48)
    alloc_case(ns, out, "a3", gen, budgets, 28, 80)

    np.savez_compressed(os.path.join(HERE, "klt.npz"), **out)
    print("wrote klt.npz")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("FATHOM_REFERENCE", "reference"))
