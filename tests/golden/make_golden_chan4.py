"""Generate the Chan4 comparator fixtures by running the REAL reference implementation.

Run here, where the reference checkout is readable (it is not on the GPU box):

    TRITON_INTERPRET=1 python tests/golden/make_golden_chan4.py /path/to/reference

It imports the reference's `kernels/bitplane.py` (torch, CPU) and writes `tests/golden/chan4.npz`:
for each case the reference's `pack_chan4` store, its scales, `channel_list` of an active set,
`scan_chan4_reference` scores, `bytes_chan4`, and (under TRITON_INTERPRET=1, power-of-two G: the
reference kernel's tl.arange(0, G) needs one) the scores of the reference Triton `scan_chan4_kernel`
through `Chan4Store.scan`.

Cases (prefix in the archive)
  c1  BH=2, n=700, G=4: active = the channels of a budget-48 plan
  c2  BH=1, n=1025, G=7: active = SparQ's top-16 of sum_g |q_g| (the reference benchmark's rule)
  c3  BH=2, n=130, G=4: all 128 channels (the full 4-bit scan), edge values (all-zero block,
      fp16 amax underflow and overflow)
  c4  BH=2, n=300, G=4, host run order (SUB = nblk): the 32 contiguous channels of a Loki/DS store
"""
import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def keys(gen, BH, n, D=128):
    scale = torch.randn(BH, 1, D, generator=gen).exp()
    return (torch.randn(BH, n, D, generator=gen) * scale).to(torch.bfloat16).float(), scale


def case(bp, out, name, K, q, active, sub=16):
    n = K.shape[1]
    bp.SUB, bp.SBT = sub, 64 * sub
    code, sc = bp.quantise_u4(K.float())
    chan_k = bp.pack_chan4(code)
    act, nact = bp.channel_list(active)
    out[f"{name}_K_bf16"] = K.to(torch.bfloat16).view(torch.int16).numpy()
    out[f"{name}_q"] = q.numpy()
    out[f"{name}_active"] = active.numpy()
    out[f"{name}_sub"] = np.int64(sub)
    out[f"{name}_code"] = code.numpy()
    out[f"{name}_chan_k"] = chan_k.numpy()
    out[f"{name}_act"] = act.numpy()
    out[f"{name}_nact"] = nact.numpy()
    out[f"{name}_scores"] = bp.scan_chan4_reference(q, code, sc, active).numpy()
    out[f"{name}_bytes"] = np.float64(bp.bytes_chan4(nact, n))
    st = bp.Chan4Store(K.float())
    assert torch.equal(st.chan_k, chan_k)
    out[f"{name}_scales_k"] = st.scales_k.view(torch.int16).numpy()
    G = q.shape[1]
    # the reference's Triton kernel needs a power-of-two G (tl.arange); G = 7 has the torch reference only
    if os.environ.get("TRITON_INTERPRET") == "1" and G & (G - 1) == 0:
        out[f"{name}_scores_triton"] = st.scan(q, act, nact).numpy()
    bp.SUB, bp.SBT = 16, 64 * 16
    print(f"{name}: n={n} BH={K.shape[0]} G={q.shape[1]} nact={nact.tolist()} sub={sub}")


def main(ref_root):
    sys.path.insert(0, os.path.join(ref_root, "kernels"))
    import bitplane as bp
    torch.set_grad_enabled(False)
    out = {}
    gen = torch.Generator().manual_seed(11)

    K, scale = keys(gen, 2, 700)
    q = torch.randn(2, 4, 128, generator=gen) * scale
    g = ((q ** 2) * K.var(1)[:, None]).sum(1)
    case(bp, out, "c1", K, q, bp.make_plan_torch(g, 48.0) > 0)

    K, scale = keys(gen, 1, 1025)
    q = torch.randn(1, 7, 128, generator=gen) * scale
    a = torch.zeros(1, 128, dtype=torch.bool)
    a.scatter_(1, q.abs().sum(1).topk(16, -1).indices, True)
    case(bp, out, "c2", K, q, a)

    K, scale = keys(gen, 2, 130)
    K[0, :64, 0:8] = 0.0                         # all-zero block
    K[0, 64:, 8] = 2e-8                           # amax below fp16's subnormal range
    K[0, :, 9] = 7.0e4                            # amax rounds to fp16 inf
    K = K.to(torch.bfloat16).float()
    q = torch.randn(2, 4, 128, generator=gen) * scale
    case(bp, out, "c3", K, q, torch.ones(2, 128, dtype=torch.bool))

    K, scale = keys(gen, 2, 300)
    q = torch.randn(2, 4, 128, generator=gen) * scale
    a = torch.zeros(2, 128, dtype=torch.bool)
    a[:, :32] = True
    case(bp, out, "c4", K, q, a, sub=math.ceil(300 / 64))

    np.savez_compressed(os.path.join(HERE, "chan4.npz"), **out)
    print("wrote chan4.npz")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("FATHOM_REFERENCE", "reference"))
