"""Hugging Face decode integration: a Qwen3 / Qwen2-family model whose attention layers run the
offloaded key-scan decode path (scripts/B_e2e_offload_v2.py:163-259, `offload_attn` +
`patched_forward`).

Life cycle of a sequence batch:

  prefill   dense causal attention over device-resident K/V (torch SDPA, chunked), as the reference
            (`patched_forward` prefill branch :249-252)
  offload   per layer: the bit-plane index of the prefill keys (HostPlaneStore in pinned mapped host
            memory, or PlaneStore in HBM), the K/V rows in mapped host memory (K and V of a token
            interleaved in one 512-byte row) or in HBM, the per-channel key variance the plan gains
            use, and a device-resident buffer for the keys and values of generated tokens
            (:272-300); the device copy of the prefill K/V is released
  decode    per layer and generated token: q/k/v projections (+ QK-norm where the model has it) and
            RoPE; the new k/v appended to the recent buffer; plan on g = sum_g q^2 Var(K); one
            scan + selection call (sink and local windows masked, k - sink - local picks, sinks
            appended); the local window [m - local, m) appended (it reaches into the recent
            buffer); exact attention over the picks, host rows fetched once per KV head (:163-244)

With klt=True the index is the KLT-rotated store (planesK, for models without QK-norm): the basis
comes from the session's own prefill keys, the plan from the rotated gains.

The model's weights, norms, MLPs and sampling are untouched; the patch is per attention module
(`unpatch()` restores them).
"""
import sys
import types

import torch
import torch.nn.functional as F

from . import bitplane as bp, klt as klt_mod
from .offload import HostPlaneStore, MappedBuffer, decode_attention

SKIP = 16        # tokens left out of the key statistics (4 * SINK, scripts/sketch.py:44-46)


class _Layer:
    __slots__ = ("Kdev", "Vdev", "len", "n", "rows", "K_src", "V_src", "store", "var", "Krec", "Vrec", "nrec",
                 "owned")

    def __init__(self):
        self.Kdev = self.Vdev = self.rows = self.K_src = self.V_src = self.store = self.var = None
        self.Krec = self.Vrec = None
        self.len = self.n = self.nrec = 0
        self.owned = []


class OffloadedDecoder:
    """Patches every attention module of `model` (a transformers Qwen3/Qwen2 causal LM on a CUDA device)
    onto the offloaded decode path.

    k, sink, local  picks per query head (k includes sink and local, as sink_local_topk)
    budget          scan budget: a number, or a per-layer sequence / {layer: budget} (per-layer budgets)
    index, rows     "host" (pinned mapped host memory, zero-copy) or "hbm" for the bit-plane index and
                    for the K/V rows
    max_new         capacity of the recent-token buffer (generated tokens)
    klt             KLT-rotated index (planesK) instead of the plain one
    graphs          replay one CUDA graph of the whole model step per generated token once the local
                    window lies inside the recent-token buffer (from the local-th generated token on;
                    the steps before run eagerly): the slot of the new token, the window's first index
                    and the position are then device-resident inputs, so one capture serves every
                    later step
    """

    def __init__(self, model, k=580, sink=4, local=64, budget=48.0, index="host", rows="host", max_new=64,
                 klt=False, prefill_chunk=2048, graphs=False):
        cfg = model.config
        self.model = model
        self.Hq = cfg.num_attention_heads
        self.Hkv = cfg.num_key_value_heads
        self.D = getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads
        if self.D != bp.D:
            raise ValueError(f"OffloadedDecoder: head_dim must be {bp.D} (got {self.D})")
        self.G = self.Hq // self.Hkv
        self.k, self.sink, self.local = k, sink, local
        if index not in ("host", "hbm") or rows not in ("host", "hbm"):
            raise ValueError("OffloadedDecoder: index and rows must be 'host' or 'hbm'")
        self.index, self.rows, self.max_new, self.klt = index, rows, max_new, klt
        self.prefill_chunk = prefill_chunk
        self.attn = [layer.self_attn for layer in model.model.layers]
        nL = len(self.attn)
        if isinstance(budget, dict):
            self.budgets = [float(budget[L]) for L in range(nL)]
        elif isinstance(budget, (list, tuple)):
            if len(budget) != nL:
                raise ValueError(f"OffloadedDecoder: {len(budget)} budgets for {nL} layers")
            self.budgets = [float(b) for b in budget]
        else:
            self.budgets = [float(budget)] * nL
        self.mode = "idle"
        self.B = 0
        self.cache = [_Layer() for _ in range(nL)]
        self._orig = {}
        self._scores = self._idx = self._arange_local = None
        self.graphs = graphs
        self._graph = self._graph_logits = None
        self._graph_sig = None
        self._graph_mode = False
        self._ids_s = self._pos_s = self._slot_s = self._wbase_s = None
        for L, m in enumerate(self.attn):
            self._orig[L] = m.forward
            m.forward = types.MethodType(self._make_forward(L), m)

    # ---------------------------------------------------------------- patch
    def unpatch(self):
        for L, m in enumerate(self.attn):
            m.forward = self._orig[L]

    def _make_forward(self, L):
        eng = self

        def forward(attn, hidden_states, position_embeddings, attention_mask=None, past_key_values=None, **kw):
            B, Tq, _ = hidden_states.shape
            shape = (B, Tq, -1, eng.D)
            q = attn.q_proj(hidden_states).view(shape)
            k = attn.k_proj(hidden_states).view(shape)
            if hasattr(attn, "q_norm"):
                q, k = attn.q_norm(q), attn.k_norm(k)
            q, k = q.transpose(1, 2), k.transpose(1, 2)
            v = attn.v_proj(hidden_states).view(shape).transpose(1, 2)
            cos, sin = position_embeddings
            q, k = sys.modules[type(attn).__module__].apply_rotary_pos_emb(q, k, cos, sin)
            if eng.mode == "prefill":
                o = eng._prefill_attn(L, q, k, v)
            elif eng.mode == "decode":
                o = eng._decode_attn(L, q, k, v)
            else:
                raise RuntimeError("OffloadedDecoder: call prefill()/load_kv() and offload() before decoding")
            return attn.o_proj(o.transpose(1, 2).reshape(B, Tq, -1)), None

        return forward

    # ---------------------------------------------------------------- prefill
    def prefill(self, input_ids):
        """Dense prefill of input_ids [B, n] in chunks; returns the logits of the last position."""
        B, n = input_ids.shape
        dev = input_ids.device
        self._reset(B)
        for c in self.cache:
            c.Kdev = torch.empty(B, self.Hkv, n, self.D, dtype=torch.bfloat16, device=dev)
            c.Vdev = torch.empty_like(c.Kdev)
            c.len = 0
        self.mode = "prefill"
        logits = None
        with torch.no_grad():
            for c0 in range(0, n, self.prefill_chunk):
                c1 = min(n, c0 + self.prefill_chunk)
                pos = torch.arange(c0, c1, device=dev)[None].expand(B, -1)
                logits = self.model(input_ids[:, c0:c1], position_ids=pos, use_cache=False, logits_to_keep=1).logits
        self.mode = "idle"
        return logits[:, -1]

    def _prefill_attn(self, L, q, k, v):
        c = self.cache[L]
        m0, Tq = c.len, q.shape[2]
        c.Kdev[:, :, m0:m0 + Tq] = k
        c.Vdev[:, :, m0:m0 + Tq] = v
        c.len = m = m0 + Tq
        mask = torch.arange(m, device=q.device)[None] <= (m0 + torch.arange(Tq, device=q.device))[:, None]
        return F.scaled_dot_product_attention(q, c.Kdev[:, :, :m], c.Vdev[:, :, :m], attn_mask=mask, enable_gqa=True)

    def load_kv(self, L, K, V, offload=False, rows_of=None):
        """Install prefill keys/values [B, Hkv, n, D] for layer L without running the model (the
        reference's --synthetic-kv mode, :280-283); offload=True builds the layer's stores at once, so
        only one layer's prefill K/V is ever on the device.  rows_of=L0 (< L, already offloaded): the
        layer's index is built from K, but attention reads layer L0's row buffers (V unused) -- for
        timing runs whose host memory cannot hold every layer's rows."""
        if L == 0:
            self._reset(K.shape[0])
        c = self.cache[L]
        c.Kdev, c.Vdev, c.len = K, V, K.shape[2]
        if offload:
            self._offload_layer(L, rows_of)
            if L == len(self.cache) - 1:
                self._finish_offload()

    # ---------------------------------------------------------------- offload
    def offload(self):
        """Build each layer's index and row store from its prefill K/V and release the device copies."""
        for L in range(len(self.cache)):
            self._offload_layer(L)
        self._finish_offload()

    def _offload_layer(self, L, rows_of=None):
        B, Hkv, D = self.B, self.Hkv, self.D
        BH = B * Hkv
        c = self.cache[L]
        n = c.len
        if n < self.k + 1:
            raise ValueError(f"OffloadedDecoder: prefill of {n} tokens is shorter than k = {self.k}")
        if L > 0 and n != self.cache[0].n:
            raise ValueError("OffloadedDecoder: every layer needs the same prefill length")
        K = c.Kdev[:, :, :n].reshape(BH, n, D).to(torch.bfloat16)
        V = None if rows_of is not None else c.Vdev[:, :, :n].reshape(BH, n, D).to(torch.bfloat16)
        dev = K.device
        basis = klt_mod.klt_basis(K) if self.klt else None
        if self.index == "host":
            c.store = HostPlaneStore(K, torch.float32 if self.klt else torch.float16, basis=basis)
            c.owned.append(c.store)
        else:
            c.store = klt_mod.KLTPlaneStore(K, basis) if self.klt else bp.PlaneStore(K)
        c.var = None if self.klt else K[:, SKIP:].float().var(1)
        if rows_of is not None:
            src = self.cache[rows_of]
            if not (0 <= rows_of < L) or src.K_src is None or src.n != n:
                raise ValueError(f"OffloadedDecoder: rows_of={rows_of} must name an offloaded earlier layer")
            c.K_src, c.V_src = src.K_src, src.V_src
        elif self.rows == "host":
            buf = MappedBuffer((BH, n, 2 * D), torch.bfloat16, dev)
            buf.dev[..., :D].copy_(K)
            buf.dev[..., D:].copy_(V)
            c.rows = buf
            c.owned.append(buf)
            c.K_src, c.V_src = buf.dev[..., :D], buf.dev[..., D:]
        else:
            c.K_src, c.V_src = K.contiguous(), V.contiguous()
        c.Krec = torch.zeros(BH, self.max_new, D, dtype=torch.bfloat16, device=dev)
        c.Vrec = torch.zeros_like(c.Krec)
        c.n, c.nrec = n, 0
        c.Kdev = c.Vdev = None

    def _finish_offload(self):
        BH, n = self.B * self.Hkv, self.cache[0].n
        dev = self.cache[0].Krec.device
        self._scores = torch.empty(BH, self.G, n, dtype=torch.float32, device=dev)
        self._idx = torch.empty(BH, self.G, self.k, dtype=torch.int64, device=dev)
        self._arange_local = torch.arange(self.local, dtype=torch.int64, device=dev)
        # graph-mode inputs: token ids, positions, the recent-buffer slot, the local window's first index
        self._ids_s = torch.zeros(self.B, 1, dtype=torch.long, device=dev)
        self._pos_s = torch.zeros(self.B, 1, dtype=torch.long, device=dev)
        self._slot_s = torch.zeros(1, dtype=torch.long, device=dev)
        self._wbase_s = torch.zeros((), dtype=torch.long, device=dev)
        self._graph = self._graph_logits = None
        torch.cuda.synchronize(dev)
        self.mode = "decode"

    def _reset(self, B):
        self.free()
        self.B = B
        self.cache = [_Layer() for _ in self.attn]

    def free(self):
        """Release the host buffers of the current batch (and the captured graph)."""
        self._graph = self._graph_logits = None
        for c in self.cache:
            for o in c.owned:
                o.free()
            c.owned = []
            c.store = c.rows = c.K_src = c.V_src = None
        self.mode = "idle"

    # ---------------------------------------------------------------- decode
    @property
    def context(self):
        """Tokens visible to the next decode step's queries: prefill + generated so far."""
        c = self.cache[0]
        return c.n + c.nrec

    def decode(self, input_ids):
        """One generated token per sequence (input_ids [B, 1]); returns logits [B, vocab]."""
        B = input_ids.shape[0]
        if self.mode != "decode" or B != self.B:
            raise RuntimeError("OffloadedDecoder: decode() needs offload() of a batch of the same size")
        if self.cache[0].nrec >= self.max_new:
            raise RuntimeError(f"OffloadedDecoder: recent-token buffer full ({self.max_new} tokens)")
        if self.graphs and self.cache[0].nrec + 1 >= self.local:
            return self._decode_graph(input_ids)
        pos = torch.full((B, 1), self.context, device=input_ids.device, dtype=torch.long)
        with torch.no_grad():
            return self.model(input_ids, position_ids=pos, use_cache=False).logits[:, -1]

    def _decode_graph(self, input_ids):
        """One step by graph replay (captured on first use).  From here on the masked prefill tail is
        empty (min(n, m - local) = n), so the captured launches differ from step to step only in the
        device-resident inputs set below."""
        c0 = self.cache[0]
        r = c0.nrec
        self._ids_s.copy_(input_ids)
        self._pos_s.fill_(c0.n + r)
        self._slot_s.fill_(r)
        self._wbase_s.fill_(c0.n + r + 1 - self.local)
        sig = (self.k, tuple(self.budgets))          # baked into the capture: a change recaptures
        if self._graph is not None and self._graph_sig != sig:
            self._graph = self._graph_logits = None
        if self._graph is None:
            self._graph_sig = sig
            self._graph_mode = True
            try:
                with torch.no_grad():
                    side = torch.cuda.Stream(device=input_ids.device)
                    side.wait_stream(torch.cuda.current_stream(input_ids.device))
                    with torch.cuda.stream(side):       # warm-up run of this very step, then the capture
                        self.model(self._ids_s, position_ids=self._pos_s, use_cache=False)
                    torch.cuda.current_stream(input_ids.device).wait_stream(side)
                    g = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(g):
                        self._graph_logits = self.model(self._ids_s, position_ids=self._pos_s,
                                                        use_cache=False).logits[:, -1]
                self._graph = g
            finally:
                self._graph_mode = False
        self._graph.replay()
        for c in self.cache:
            c.nrec = r + 1
        return self._graph_logits.clone()

    def _decode_attn(self, L, q, k, v):
        c = self.cache[L]
        B, Hq, Tq, D = q.shape
        if Tq != 1:
            raise RuntimeError("OffloadedDecoder: decode takes one token per sequence")
        BH, G = B * self.Hkv, self.G
        sink, local = self.sink, self.local
        kk = self.k - sink - local
        n = c.n
        if self._graph_mode:                     # slot and window base are device inputs; nrec moves outside
            c.Krec.index_copy_(1, self._slot_s, k.reshape(BH, 1, D))
            c.Vrec.index_copy_(1, self._slot_s, v.reshape(BH, 1, D))
            m = n + c.nrec + 1
        else:
            r = c.nrec
            c.Krec[:, r] = k.reshape(BH, D)
            c.Vrec[:, r] = v.reshape(BH, D)
            c.nrec = r + 1
            m = n + c.nrec
        hi = min(n, m - local)
        if hi - sink < kk:
            raise ValueError(f"OffloadedDecoder: {hi - sink} selectable prefill tokens < k - sink - local = {kk}")
        qf = q.reshape(BH, G, D).float()
        if c.var is None:                                   # KLT index: rotated queries and gains
            qs, g = klt_mod.klt_query(qf, c.store.basis)
        else:
            qs, g = qf, (qf * qf * c.var[:, None]).sum(1)
        plan = bp.make_plan(g, self.budgets[L])
        if self._idx.shape[2] != self.k:
            self._idx = torch.empty(BH, G, self.k, dtype=torch.int64, device=q.device)
        idx = self._idx
        bp.scan_select(c.store, qs, plan, kk, mask_lo=sink, mask_hi=hi, append_sink=sink, scores=self._scores,
                       idx_out=idx)
        # the local window [m - local, m): one add into the strided tail of the index rows
        torch.add(self._arange_local.expand(BH, G, local), self._wbase_s if self._graph_mode else m - local,
                  out=idx[..., kk + sink:])
        out = decode_attention(qf, idx, c.K_src, c.V_src, n, n, c.Krec, c.Vrec, self.max_new,
                               out_dtype=torch.bfloat16)
        return out.view(B, Hq, 1, D)
