"""KLT-rotated bit-plane store (planesK) and per-layer scan budgets.

planesK (scripts/R_ruler.py:4, 63-64, 82-84) is the bit-plane scan over keys rotated into a per-head
Karhunen-Loeve basis -- the basis rule for models whose keys have no QK-norm, where a few rotated
channels carry most of the score variance:

  store   Kr = (K - mu) @ Vt, then the 4-bit block store of Kr (codes from the fp32 block absmax,
          codes_u4 of scripts/R_ruler.py:34-39)
  query   qr = q @ Vt, gains = sum_g qr^2 * lam, plan = make_plan(gains, budget)
  scores  the plane-prefix scan of qr over the store: q.(K - mu) up to quantisation, i.e. the scores up
          to the per-query constant q.mu, which no top-k depends on

The store build is one fused kernel (rotate + quantise + pack, fathom_klt_quantise_pack); the query
side is one kernel per layer (fathom_klt_query); the scan and selection are the plain plane-store
kernels.  The basis is calibration: `klt_basis` computes self_klt (scripts/R_agent.py:59-63) from the
session's own keys with library calls (a float64 covariance product and eigendecomposition), once per
layer before the store is built.

Per-layer budgets (scripts/l4_final_alloc.py:143-154): `allocate_layer_budgets` turns a calibration
table of per-layer errors into one scan budget per layer; each layer's make_plan then takes its own
budget (make_plan accepts a scalar or one budget per row).
"""
from typing import NamedTuple

import torch

from . import _lib, bitplane as bp
from ._lib import check, lib, ptr, require_cuda, stream_of

D = bp.D
SKIP = 16          # self_klt fits the basis on the keys after the first 4 * SINK tokens (SINK = 4)


class KLTBasis(NamedTuple):
    """Per-row KLT basis: mu [BH, D], Vt [BH, D, D] (column e = rotated channel e), lam [BH, D] >= 0; fp32."""
    mu: torch.Tensor
    Vt: torch.Tensor
    lam: torch.Tensor

    def ready(self, BH, device):
        """True if the basis is already contiguous fp32 on `device` with BH rows (no copy needed)."""
        return (self.Vt.device == torch.device(device) and self.mu.device == self.Vt.device and
                self.lam.device == self.Vt.device and
                all(x.dtype == torch.float32 and x.is_contiguous() for x in self) and
                self.mu.shape == (BH, D) and self.Vt.shape == (BH, D, D) and self.lam.shape == (BH, D))

    def checked(self, BH, device):
        """The basis as contiguous fp32 tensors on `device`, shapes checked against BH rows."""
        mu, Vt, lam = (x.to(device=device, dtype=torch.float32).contiguous() for x in (self.mu, self.Vt, self.lam))
        if mu.shape != (BH, D) or Vt.shape != (BH, D, D) or lam.shape != (BH, D):
            raise ValueError(f"KLTBasis: need mu [{BH},{D}], Vt [{BH},{D},{D}], lam [{BH},{D}]; got "
                             f"{tuple(mu.shape)}, {tuple(Vt.shape)}, {tuple(lam.shape)}")
        return KLTBasis(mu, Vt, lam)


def klt_basis(K, skip=SKIP):
    """self_klt (scripts/R_agent.py:59-63): K [BH, n, D] -> KLTBasis from the keys after the first `skip`
    tokens: mu = mean, (lam, Vt) = eigendecomposition of the centred covariance (eigenvalues ascending,
    clamped at 0).  Computed in float64 (cuBLAS / cuSOLVER), returned in fp32."""
    require_cuda(K)
    BH, n, d = K.shape
    if d != D or n <= skip:
        raise ValueError(f"klt_basis: need K [BH, n > {skip}, {D}], got {tuple(K.shape)}")
    X = K[:, skip:].double()
    mu = X.mean(1)
    Xc = X - mu[:, None]
    C = torch.bmm(Xc.transpose(1, 2), Xc) / X.shape[1]
    lam, V = torch.linalg.eigh(C)
    return KLTBasis(mu.float(), V.float().contiguous(), lam.clamp_min(0).float())


def klt_query(q, basis, gains=True, out=None):
    """scripts/R_ruler.py:82-83: q [BH, G, D] -> (qr = q @ Vt [BH, G, D] fp32, gains [BH, D] fp32 =
    sum_g qr^2 * lam, or None).  out=(qr, gains) writes into preallocated tensors."""
    require_cuda(q)
    BH, G, d = q.shape
    assert d == D
    b = basis if basis.ready(BH, q.device) else basis.checked(BH, q.device)
    qc = q if q.dtype == torch.float32 and q.is_contiguous() else q.contiguous().float()
    if out is not None:
        qr, g = out
        ok = (qr.shape == (BH, G, D) and qr.dtype == torch.float32 and qr.is_contiguous() and qr.device == q.device
              and (g is None or (g.shape == (BH, D) and g.dtype == torch.float32 and g.is_contiguous()
                                 and g.device == q.device)))
        if not ok:
            raise ValueError(f"klt_query: out must be (fp32 [{BH},{G},{D}], fp32 [{BH},{D}] or None) on {q.device}")
    else:
        qr = torch.empty(BH, G, D, device=q.device, dtype=torch.float32)
        g = torch.empty(BH, D, device=q.device, dtype=torch.float32) if gains else None
    check(lib().fathom_klt_query(ptr(qc), BH, G, ptr(b.Vt), ptr(b.lam), ptr(qr), ptr(g), stream_of(q.device)),
          "klt_query")
    return qr, g


def klt_rotate(K, basis):
    """(K - mu) @ Vt [BH, n, D] fp32 through the store-build kernel (the keys the store quantises)."""
    require_cuda(K)
    BH, n, d = K.shape
    assert d == D
    if K.dtype not in _lib.DTYPE_CODE:
        K = K.float()
    Kc = K if K.stride(-1) == 1 and K.stride(-2) == D else K.contiguous()
    b = basis.checked(BH, K.device)
    out = torch.empty(BH, n, D, device=K.device, dtype=torch.float32)
    check(lib().fathom_klt_quantise_pack(ptr(Kc), _lib.DTYPE_CODE[Kc.dtype], BH, n, Kc.stride(0), ptr(b.mu),
                                         ptr(b.Vt), 1, 0, None, None, 0, None, None, ptr(out),
                                         stream_of(K.device)), "klt_rotate")
    return out


class KLTPlaneStore(bp.PlaneStore):
    """The planesK store (scripts/R_ruler.py:63-64): a PlaneStore over (K - mu) @ Vt whose codes follow
    codes_u4 (fp32 block absmax; the stored scales are fp16 as in every PlaneStore).  scan() takes the
    rotated queries; `query(q)` gives them with the plan gains."""

    def __init__(self, K, basis, scale_dtype=torch.float32):
        super().__init__(K, scale_dtype, basis=basis)

    def query(self, q, gains=True):
        return klt_query(q, self.basis, gains)


def allocate_layer_budgets(err, budgets, mean_target):
    """allocate (scripts/l4_final_alloc.py:143-154): err {budget: {layer: error}} from calibration ->
    {layer: budget}.  Every layer starts at budgets[0]; while the mean budget is below mean_target the
    layer whose next budget step lowers its error most per budget unit moves up one step (the first
    such layer on ties; a step must lower the error by more than -1 per unit to be taken)."""
    budgets = list(budgets)
    layers = list(err[budgets[0]].keys())
    step = {L: 0 for L in layers}
    while sum(budgets[i] for i in step.values()) / len(layers) < mean_target:
        best, pick = -1, None
        for L in layers:
            i = step[L]
            if i + 1 >= len(budgets):
                continue
            gain = (err[budgets[i]][L] - err[budgets[i + 1]][L]) / (budgets[i + 1] - budgets[i])
            if gain > best:
                best, pick = gain, L
        if pick is None:
            break
        step[pick] += 1
    return {L: budgets[i] for L, i in step.items()}
