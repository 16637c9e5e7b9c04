"""Zero-copy row gather and decode attention against the oracle, from device memory and from pinned
mapped host memory, with and without device-resident recent rows."""
import numpy as np
import pytest
import torch

from oracle import bitplane_oracle as O

pytestmark = pytest.mark.gpu


def _kv(BH, cap, seed):
    g = torch.Generator().manual_seed(seed)
    sc = torch.randn(BH, 1, 128, generator=g).exp()
    K = (torch.randn(BH, cap, 128, generator=g) * sc).bfloat16()
    V = (torch.randn(BH, cap, 128, generator=g) * sc).bfloat16()
    return K, V


def test_gather_rows_device_and_host():
    from fathom_b200.offload import MappedBuffer, gather_rows
    BH, cap, R = 3, 5000, 777
    K, _ = _kv(BH, cap, 1)
    idx = torch.randint(-1, cap, (BH, R), dtype=torch.int32)
    ref = O.gather_rows(K.view(torch.int16).numpy(), idx.numpy())
    got = gather_rows(K.cuda(), cap, idx.cuda(), BH)
    assert np.array_equal(got.cpu().view(torch.int16).numpy(), ref)
    hb = MappedBuffer((BH, cap, 128), torch.bfloat16)
    hb.host.copy_(K)
    got = gather_rows(hb.dev, cap, idx.cuda(), BH)
    assert np.array_equal(got.cpu().view(torch.int16).numpy(), ref)
    hb.free()


@pytest.mark.parametrize("G,k", [(4, 580), (7, 2116), (1, 1), (8, 64)])
@pytest.mark.parametrize("where", ["device", "host"])
def test_decode_attention(G, k, where):
    from fathom_b200.offload import MappedBuffer, decode_attention
    BH, cap = 4, 30000
    K, V = _kv(BH, cap, G * 1000 + k)
    g = torch.Generator().manual_seed(k)
    q = torch.randn(BH, G, 128, generator=g)
    idx = torch.randint(0, cap, (BH, G, k), generator=g)
    idx[:, :, : k // 3] = idx[:, :1, : k // 3]                  # shared picks across the GQA group
    if where == "device":
        Ks, Vs = K.cuda(), V.cuda()
    else:
        kb, vb = MappedBuffer(K.shape, torch.bfloat16), MappedBuffer(V.shape, torch.bfloat16)
        kb.host.copy_(K)
        vb.host.copy_(V)
        Ks, Vs = kb.dev, vb.dev
    out = decode_attention(q.cuda(), idx.cuda(), Ks, Vs, cap).cpu().numpy()
    ref = O.decode_attention(q.numpy(), O.bf16_to_f32(K.view(torch.int16).numpy().view(np.uint16)),
                             O.bf16_to_f32(V.view(torch.int16).numpy().view(np.uint16)), idx.numpy())
    assert np.abs(out - ref).max() <= 1e-5 * np.abs(ref).max() + 1e-6
    outb = decode_attention(q.cuda(), idx.cuda(), Ks, Vs, cap, out_dtype=torch.bfloat16).float().cpu().numpy()
    assert np.abs(outb - ref).max() <= 1e-2 * np.abs(ref).max()


def test_decode_attention_recent_rows():
    """Indices >= n_host read the device-resident recent buffer (offload_attn :234-241)."""
    from fathom_b200.offload import decode_attention
    BH, G, k, cap, n_host, rc = 2, 4, 100, 2000, 1990, 16
    K, V = _kv(BH, cap, 5)
    Kr, Vr = _kv(BH, rc, 6)
    idx = torch.randint(0, n_host + rc, (BH, G, k))
    q = torch.randn(BH, G, 128)
    out = decode_attention(q.cuda(), idx.cuda(), K.cuda(), V.cuda(), cap, n_host, Kr.cuda(), Vr.cuda(), rc)
    f = lambda t: O.bf16_to_f32(t.view(torch.int16).numpy().view(np.uint16))
    ref = O.decode_attention(q.numpy(), f(K), f(V), idx.numpy(), f(Kr), f(Vr), n_host)
    assert np.abs(out.cpu().numpy() - ref).max() <= 1e-5 * np.abs(ref).max() + 1e-6


@pytest.mark.parametrize("parts", [1, 2, 3, 4])
def test_partial_attention_combine_equals_full(parts):
    """Context shards: partial attention over owned picks + log-sum-exp combine == full attention."""
    from fathom_b200 import shard
    from fathom_b200.offload import attention_combine, decode_attention, decode_attention_partial
    BH, G, k, n = 3, 4, 300, 9000
    K, V = _kv(BH, n, 40 + parts)
    g = torch.Generator().manual_seed(parts)
    q = torch.randn(BH, G, 128, generator=g).cuda()
    idx = torch.randint(0, n, (BH, G, k), generator=g).cuda()
    full = decode_attention(q, idx, K.cuda(), V.cuda(), n)
    packed = []
    for lo, hi in shard.chunk_bounds(n, parts):
        Kc, Vc = K[:, lo:hi].contiguous().cuda(), V[:, lo:hi].contiguous().cuda()
        packed.append(decode_attention_partial(q, idx, Kc, Vc, hi - lo, lo, hi))
    out = attention_combine(torch.stack(packed))
    assert torch.allclose(out, full, rtol=1e-5, atol=1e-6 * float(full.abs().max()))


def test_hugepage_buffers_gather_and_attention():
    """Huge-page-backed mapped buffers (cudaHostRegister) read like cudaHostAlloc ones."""
    from fathom_b200.offload import MappedBuffer, decode_attention, gather_rows
    BH, cap = 2, 50000
    K, V = _kv(BH, cap, 77)
    kb, vb = MappedBuffer(K.shape, torch.bfloat16, hugepages=True), MappedBuffer(V.shape, torch.bfloat16, hugepages=True)
    kb.host.copy_(K)
    vb.host.copy_(V)
    idx = torch.randint(0, cap, (BH, 300), dtype=torch.int32)
    got = gather_rows(kb.dev, cap, idx.cuda(), BH)
    assert np.array_equal(got.cpu().view(torch.int16).numpy(), O.gather_rows(K.view(torch.int16).numpy(), idx.numpy()))
    q = torch.randn(BH, 4, 128)
    pick = torch.randint(0, cap, (BH, 4, 200))
    a = decode_attention(q.cuda(), pick.cuda(), kb.dev, vb.dev, cap)
    b = decode_attention(q.cuda(), pick.cuda(), K.cuda(), V.cuda(), cap)
    assert torch.equal(a, b)
    kb.free()
    vb.free()


@pytest.mark.parametrize("where", ["device", "host"])
def test_interleaved_kv_rows(where):
    """A cache that interleaves each token's K and V rows ([BH][cap][2][128], row stride 256) gives
    the same attention as separate K and V buffers."""
    from fathom_b200.offload import MappedBuffer, decode_attention
    BH, G, k, cap = 3, 4, 400, 20000
    K, V = _kv(BH, cap, 11)
    KV = torch.stack([K, V], 2)                               # [BH, cap, 2, 128]
    if where == "device":
        kv = KV.cuda()
    else:
        buf = MappedBuffer(KV.shape, torch.bfloat16)
        buf.host.copy_(KV)
        kv = buf.dev
    q = torch.randn(BH, G, 128).cuda()
    idx = torch.randint(0, cap, (BH, G, k)).cuda()
    a = decode_attention(q, idx, kv[:, :, 0], kv[:, :, 1], cap)
    b = decode_attention(q, idx, K.cuda(), V.cuda(), cap)
    assert torch.equal(a, b)


@pytest.mark.parametrize("BH,G", [(2, 4), (40, 4), (32, 7), (90, 4)])
def test_in_place_attention_kernels_equal_staged(BH, G):
    """Device-resident rows are read in place (8 heads: 32 warps per head in 8-CTA clusters; 160 and
    config 3's 224 heads: 16 warps in 4-CTA clusters; 360: one 16-warp CTA per head); host-resident
    rows go through dedupe + staging.  Both sum in the same order: the outputs are bit-identical, and
    match the oracle."""
    from fathom_b200.offload import MappedBuffer, decode_attention
    cap, k = 3000, 300
    K, V = _kv(BH, cap, BH + G)
    g = torch.Generator().manual_seed(BH)
    q = torch.randn(BH, G, 128, generator=g)
    idx = torch.randint(0, cap, (BH, G, k), generator=g)
    kb, vb = MappedBuffer(K.shape, torch.bfloat16), MappedBuffer(V.shape, torch.bfloat16)
    kb.host.copy_(K)
    vb.host.copy_(V)
    dev_out = decode_attention(q.cuda(), idx.cuda(), K.cuda(), V.cuda(), cap)
    host_out = decode_attention(q.cuda(), idx.cuda(), kb.dev, vb.dev, cap)
    assert torch.equal(dev_out, host_out)
    ref = O.decode_attention(q.numpy(), O.bf16_to_f32(K.view(torch.int16).numpy().view(np.uint16)),
                             O.bf16_to_f32(V.view(torch.int16).numpy().view(np.uint16)), idx.numpy())
    out = dev_out.cpu().numpy()
    assert np.abs(out - ref).max() <= 1e-5 * np.abs(ref).max() + 1e-6
    kb.free()
    vb.free()


@pytest.mark.parametrize("nw", [16, 32])
def test_attention_bits_do_not_depend_on_the_cta_split(nw, monkeypatch):
    """The warps of a query head may sit in one CTA or in a cluster of 2, 4 or 8 CTAs (the tuning
    overrides pick the split); the merge runs in global warp order, so every split gives the same bits,
    from device rows and from staged host rows."""
    from fathom_b200.offload import MappedBuffer, decode_attention
    BH, G, k, cap = 3, 5, 1000, 20000
    K, V = _kv(BH, cap, 123)
    g = torch.Generator().manual_seed(9)
    q = torch.randn(BH, G, 128, generator=g).cuda()
    idx = torch.randint(0, cap, (BH, G, k), generator=g).cuda()
    kb, vb = MappedBuffer(K.shape, torch.bfloat16), MappedBuffer(V.shape, torch.bfloat16)
    kb.host.copy_(K)
    vb.host.copy_(V)
    monkeypatch.setenv("FATHOM_ATTN_NW", str(nw))
    outs = []
    for cs in (1, 2, 4, 8):
        monkeypatch.setenv("FATHOM_ATTN_CS", str(cs))
        outs.append(decode_attention(q, idx, K.cuda(), V.cuda(), cap))
        outs.append(decode_attention(q, idx, kb.dev, vb.dev, cap))
    torch.cuda.synchronize()
    for o in outs[1:]:
        assert torch.equal(o, outs[0])
    kb.free()
    vb.free()


@pytest.mark.parametrize("where", ["device", "host"])
def test_attention_skips_picks_outside_the_readable_rows(where):
    """Picks that are negative or at or past the readable rows (n_host source rows + recent_cap recent
    rows) are skipped: the output is the attention over the remaining picks, in place and staged."""
    from fathom_b200.offload import MappedBuffer, decode_attention
    BH, G, k, cap, n_host, rc = 3, 4, 300, 6000, 5900, 50
    K, V = _kv(BH, cap, 31)
    Kr, Vr = _kv(BH, rc, 32)
    g = torch.Generator().manual_seed(33)
    q = torch.randn(BH, G, 128, generator=g)
    idx = torch.randint(0, n_host + rc, (BH, G, k), generator=g)
    bad = torch.rand(BH, G, k, generator=g) < 0.2
    junk = torch.where(torch.rand(BH, G, k, generator=g) < 0.5, torch.full_like(idx, -1),
                       torch.randint(n_host + rc, 1 << 30, (BH, G, k), generator=g))
    idx = torch.where(bad, junk, idx)
    if where == "device":
        Ks, Vs = K.cuda(), V.cuda()
    else:
        kb, vb = MappedBuffer(K.shape, torch.bfloat16), MappedBuffer(V.shape, torch.bfloat16)
        kb.host.copy_(K)
        vb.host.copy_(V)
        Ks, Vs = kb.dev, vb.dev
    out = decode_attention(q.cuda(), idx.cuda(), Ks, Vs, cap, n_host, Kr.cuda(), Vr.cuda(), rc).cpu().numpy()
    f = lambda t: O.bf16_to_f32(t.view(torch.int16).numpy().view(np.uint16))
    ref = np.empty_like(out)
    for b in range(BH):
        for h in range(G):
            ok = idx[b, h][~bad[b, h]].numpy()[None, None, :]
            ref[b, h] = O.decode_attention(q[b:b + 1, h:h + 1].numpy(), f(K[b:b + 1]), f(V[b:b + 1]), ok,
                                           f(Kr[b:b + 1]), f(Vr[b:b + 1]), n_host)[0, 0]
    assert np.abs(out - ref).max() <= 1e-5 * np.abs(ref).max() + 1e-6
    if where == "host":
        kb.free()
        vb.free()
