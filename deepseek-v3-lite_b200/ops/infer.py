"""Native inference path: prefill and decode over the latent KV cache.

``InferenceEngine(model)`` runs the reference model's inference forward on the
sm_100a kernels, reading the module parameters through cached bf16 copies:

* prefill at position 0 uses the materialised formulation (Q/K/V packing with
  RoPE + causal flash attention), exactly like the training step;
* every other call (decode, chunked prefill, speculative verification) uses
  the *absorbed* formulation over the latent cache: the query projection is
  pre-multiplied by ``W_k`` and the output projection by ``W_v`` (per head,
  once per weight version), so a step reads each cached latent row
  (``kv_lora_rank + rope_dim`` values) instead of materialising K and V for
  the whole context -- the reason MLA exists;
* the MoE FFN is the same routed/grouped kernel sequence as training
  (router GEMM, top-k, padded permutation, grouped SwiGLU and down GEMMs,
  weighted combine) plus the shared experts.

The cache lives in the attention modules (``kv_cache`` / ``pe_cache``, bf16)
so the module API (``reset_cache``, ``_ensure_cache``) keeps its meaning.
Positions may differ per row (``pos[b]``), which continuous batching and the
batched speculative decoder rely on.
"""
from __future__ import annotations

from typing import Dict, Optional, Tuple

import torch

from . import _ext
from ._ext import native
from .rope import rope_cos_sin

BF16 = torch.bfloat16
F32 = torch.float32


def _pad(n: int, m: int) -> int:
    return (n + m - 1) // m * m


class InferenceEngine:
    def __init__(self, model):
        self.model = model
        self.C = native()
        c = model.config
        self.c = c
        self.D, self.H = c["dim"], c["n_heads"]
        self.dn, self.dr, self.dv = c["qk_nope_head_dim"], c["qk_rope_head_dim"], c["v_head_dim"]
        self.R = c["kv_lora_rank"]
        self.V = c["vocab_size"]
        self.Vp = _pad(self.V, 64)
        self.DP = max(32, _pad(self.dn + self.dr, 16))
        self.device = next(model.parameters()).device
        self.cos, self.sin = rope_cos_sin(c["max_seq_len"], self.dr, float(c["rope_theta"]), self.device)
        self._cache: Dict[tuple, torch.Tensor] = {}
        self._graphs: Dict[tuple, tuple] = {}
        self.q_lora = int(c.get("q_lora_rank", 0) or 0)

    # ------------------------------------------------------------ weights
    def _key(self, tag, *params):
        return (tag,) + tuple((id(p), p._version, p.data_ptr()) for p in params)

    def bf16(self, p) -> torch.Tensor:
        k = self._key("w", p)
        t = self._cache.get(k)
        if t is None:
            self._drop("w", p)
            t = p.detach().to(BF16).contiguous()
            self._cache[k] = t
        return t

    def _drop(self, tag, p):
        for k in [k for k in self._cache if k[0] == tag and k[1][0] == id(p)]:
            del self._cache[k]

    @staticmethod
    def _wq(attn):
        """The projection that yields q from its input: ``wq`` (input: normalised x)
        or ``wq_b`` of the LoRA chain (input: ``q_norm(wq_a x)``)."""
        return attn.wq_b.weight if getattr(attn, "q_lora_rank", 0) > 0 else attn.wq.weight

    def _q_input(self, attn, xn):
        """What the query projection multiplies: ``xn`` or ``q_norm(wq_a xn)``."""
        if not self.q_lora:
            return xn
        qa = self._lin(xn, self.bf16(attn.wq_a.weight))
        qn = torch.empty_like(qa)
        self.C.rmsnorm_fwd(qa, attn.q_norm.weight.detach().float().contiguous(), 1e-6, qn,
                           torch.empty(0, device=self.device))
        return qn

    def _absorbed(self, attn):
        """(Wq_lat [H*R, Din], Wq_pe [H*dr, Din], W_out [D, H*R]) for ``attn`` (bf16);
        ``Din`` is the query projection's input width (D, or q_lora_rank)."""
        wq_p = self._wq(attn)
        k = self._key("abs", wq_p, attn.wkv_b.weight, attn.wo.weight)
        got = self._cache.get(k)
        if got is not None:
            return got
        self._drop("abs", wq_p)
        H, dn, dr, dv, R, D = self.H, self.dn, self.dr, self.dv, self.R, self.D
        with torch.no_grad():
            Din = wq_p.shape[1]
            wq = wq_p.float().view(H, dn + dr, Din)
            wkvb = attn.wkv_b.weight.float().view(H, dn + dv, R)
            w_k, w_v = wkvb[:, :dn], wkvb[:, dn:]
            q_lat = torch.einsum("hdr,hdk->hrk", w_k, wq[:, :dn]).reshape(H * R, Din)   # rows: W_k[h]^T Wq_nope[h]
            q_pe = wq[:, dn:].reshape(H * dr, Din)
            wo = attn.wo.weight.float().view(D, H, dv)
            w_out = torch.einsum("khd,hdr->khr", wo, w_v).reshape(D, H * R)          # Wo_h W_v[h]
            got = (q_lat.to(BF16).contiguous(), q_pe.to(BF16).contiguous(), w_out.to(BF16).contiguous())
        self._cache[k] = got
        return got

    def _experts(self, moe):
        ws = [w for e in moe.experts for w in (e.w1.weight, e.w3.weight, e.w2.weight)]
        k = self._key("exp", *ws)
        got = self._cache.get(k)
        if got is None:
            for kk in [kk for kk in self._cache if kk[0] == "exp" and kk[1][0] == id(ws[0])]:
                del self._cache[kk]
            E = len(moe.experts)
            w13 = torch.stack([torch.stack([e.w1.weight, e.w3.weight]) for e in moe.experts]).to(BF16).contiguous()
            w2 = torch.stack([e.w2.weight for e in moe.experts]).to(BF16).contiguous()
            got = (w13.view(E, 2, *moe.experts[0].w1.weight.shape), w2)
            self._cache[k] = got
        return got

    def _swiglu_pair(self, w1, w3):
        k = self._key("sw", w1, w3)
        got = self._cache.get(k)
        if got is None:
            self._drop("sw", w1)
            got = torch.stack([w1, w3]).to(BF16).unsqueeze(0).contiguous()
            self._cache[k] = got
        return got

    # --------------------------------------------------------------- layers
    def _norm(self, x, w):
        y = torch.empty(x.shape[0], x.shape[1], dtype=BF16, device=self.device)
        self.C.rmsnorm_fwd(x, w.detach().float().contiguous(), 1e-6, y, torch.empty(0, device=self.device))
        return y

    def _lin(self, x, p_bf16, out=None, accumulate=False):
        if out is None:
            out = torch.empty(x.shape[0], p_bf16.shape[0], dtype=BF16, device=self.device)
            self.C.linear_fwd(x, p_bf16, out)
        else:
            self.C.linear_fwd(x, p_bf16, out, accumulate)
        return out

    def _dense_ffn(self, w1, w3, w2, xn, out):
        T, I = xn.shape[0], w1.shape[0]
        h = torch.empty(T, I, dtype=BF16, device=self.device)
        gu = torch.empty(T, 2 * I, dtype=BF16, device=self.device)
        self.C.swiglu_fwd(xn, self._swiglu_pair(w1, w3), torch.empty(0, dtype=torch.int32, device=self.device), h, gu)
        self.C.linear_fwd(h, self.bf16(w2), out, True)

    def _moe(self, moe, xn, out):
        C = self.C
        T = xn.shape[0]
        E, k, I = moe.n_routed_experts, moe.topk, moe.moe_inter_dim
        Ep = _pad(E, 8)
        logits = torch.empty(T, Ep, dtype=F32, device=self.device)
        C.linear_fwd(xn, self.bf16(moe.gate.weight), logits[:, :E], False)
        idx = torch.empty(T, k, dtype=torch.int32, device=self.device)
        wts = torch.empty(T, k, dtype=F32, device=self.device)
        ssel = torch.empty(T, k, dtype=F32, device=self.device)
        counts = torch.zeros(E, dtype=torch.int32, device=self.device)
        C.router_topk(logits, moe.gate.bias, E, k, float(moe.gate.route_scale), idx, wts, ssel, counts)
        P = _pad(T * k + E * 255, 256)       # 256-row expert ranges (CTA-pair GEMM tiles)
        row_off = torch.empty(E + 1, dtype=torch.int32, device=self.device)
        tg = torch.empty(P // 128, dtype=torch.int32, device=self.device)
        cursor = torch.empty(E, dtype=torch.int32, device=self.device)
        src = torch.empty(P, dtype=torch.int32, device=self.device)
        dst = torch.empty(T, k, dtype=torch.int32, device=self.device)
        C.permute_plan(counts, row_off, tg, cursor, src, src_tail_only=True)
        xs = torch.empty(P, self.D, dtype=BF16, device=self.device)
        C.permute_gather(idx, counts, row_off, cursor, xn, src, dst, xs)
        w13, w2 = self._experts(moe)
        h = torch.empty(P, I, dtype=BF16, device=self.device)
        gu = torch.empty(P, 2 * I, dtype=BF16, device=self.device)
        C.swiglu_fwd(xs, w13, tg, h, gu, group_rows=256)
        ys = torch.empty(P, self.D, dtype=BF16, device=self.device)
        C.grouped_fwd(h, w2, tg, ys, group_rows=256)
        C.combine_fwd(ys, dst, wts, out)
        for e in moe.shared_experts:
            self._dense_ffn(e.w1.weight, e.w3.weight, e.w2.weight, xn, out)
        moe._last_indices, moe._last_weights, moe._last_counts = idx, wts, counts

    def _attn_prefill0(self, attn, xn, B, S, out):
        """Materialised causal attention for a prompt starting at position 0."""
        C, H, dn, dr, dv, R = self.C, self.H, self.dn, self.dr, self.dv, self.R
        T = B * S
        q = self._lin(self._q_input(attn, xn), self.bf16(self._wq(attn)))
        kv_a = self._lin(xn, self.bf16(attn.wkv_a.weight))
        lat = torch.empty(T, R, dtype=BF16, device=self.device)
        C.rmsnorm_fwd(kv_a[:, :R], attn.kv_norm.weight.detach().float().contiguous(), 1e-6, lat,
                      torch.empty(0, device=self.device))
        kvb = self._lin(lat, self.bf16(attn.wkv_b.weight))
        Q = torch.empty(B * H, S, self.DP, dtype=BF16, device=self.device)
        K = torch.empty_like(Q)
        Vt = torch.empty(B * H, S, dv, dtype=BF16, device=self.device)
        C.mla_pack(q, kvb, kv_a[:, R:], Q, K, Vt, B, S, H, dn, dr, dv, self.cos, self.sin, 0)
        O = torch.empty(T, H * dv, dtype=BF16, device=self.device)
        L = torch.empty(B * H, S, dtype=F32, device=self.device)
        C.flash_fwd(Q, K, Vt, O, L, 0, attn.softmax_scale, True, H)
        C.linear_fwd(O, self.bf16(attn.wo.weight), out, True)
        # cache: post-norm latent and post-RoPE k_pe
        kpe = kv_a[:, R:].contiguous().view(T, 1, dr)
        C.rope_inplace(kpe, 0, dr // 2, self.cos, self.sin, None, S, 0, False)
        attn.kv_cache[:B, :S] = lat.view(B, S, R)
        attn.pe_cache[:B, :S] = kpe.view(B, S, dr)

    def _attn_latent(self, attn, xn, B, S, pos, out):
        """Absorbed attention for queries at positions ``pos`` [B*S] over the cache."""
        C, H, dr, R = self.C, self.H, self.dr, self.R
        T = B * S
        wq_lat, wq_pe, w_out = self._absorbed(attn)
        kv_a = self._lin(xn, self.bf16(attn.wkv_a.weight))
        lat = torch.empty(T, R, dtype=BF16, device=self.device)
        C.rmsnorm_fwd(kv_a[:, :R], attn.kv_norm.weight.detach().float().contiguous(), 1e-6, lat,
                      torch.empty(0, device=self.device))
        kpe = kv_a[:, R:].contiguous().view(T, 1, dr)
        C.rope_inplace(kpe, 0, dr // 2, self.cos, self.sin, pos, 1, 0, False)
        rows = torch.arange(B, device=self.device).repeat_interleave(S)
        attn.kv_cache[rows, pos.long()] = lat
        attn.pe_cache[rows, pos.long()] = kpe.view(T, dr)
        q_src = self._q_input(attn, xn)
        q_lat = self._lin(q_src, wq_lat).view(T, H, R)
        q_pe = self._lin(q_src, wq_pe).view(T, H, dr)
        C.rope_inplace(q_pe, 0, dr // 2, self.cos, self.sin, pos, 1, 0, False)
        max_len = int(self.c["max_seq_len"])
        nsplit = (max_len + 255) // 256
        scratch = torch.empty(T * H * nsplit * (2 + R), dtype=F32, device=self.device)
        o_lat = torch.empty(T, H, R, dtype=BF16, device=self.device)
        lens = (pos + 1).to(torch.int32)
        C.latent_decode(q_lat, q_pe, attn.kv_cache, attn.pe_cache, lens, attn.softmax_scale, max_len, scratch, o_lat, S)
        C.linear_fwd(o_lat.view(T, H * R), w_out, out, True)

    # -------------------------------------------------------------- forward
    @torch.no_grad()
    def forward(self, tokens: torch.Tensor, start_pos: int = 0, pos: Optional[torch.Tensor] = None,
                want_hidden: bool = False) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
        """Logits ``[B, S, V]`` (bf16) for ``tokens [B, S]`` written into the cache.

        ``pos`` ([B] int) gives each row's position (S must then be 1);
        otherwise row b's tokens sit at ``start_pos .. start_pos + S - 1``.
        """
        m, C = self.model, self.C
        B, S = tokens.shape
        T = B * S
        if pos is None:
            pos_t = (torch.arange(S, device=self.device) + start_pos).repeat(B).to(torch.int32)
        else:
            assert S == 1, "per-row positions take one token per row"
            pos_t = pos.to(torch.int32)
        for layer in m.layers:
            layer.attn._ensure_cache(B, self.device, BF16)
        x = torch.empty(T, self.D, dtype=F32, device=self.device)
        C.embedding_fwd(tokens.reshape(-1).long().contiguous(), m.embed.weight.detach().float().contiguous(), x)
        prefill0 = pos is None and start_pos == 0 and S > 1
        for layer in m.layers:
            xn = self._norm(x, layer.attn_norm.weight)
            if prefill0:
                self._attn_prefill0(layer.attn, xn, B, S, x)
            else:
                self._attn_latent(layer.attn, xn, B, S, pos_t, x)
            xn2 = self._norm(x, layer.ffn_norm.weight)
            if hasattr(layer.ffn, "experts"):
                self._moe(layer.ffn, xn2, x)
            else:
                self._dense_ffn(layer.ffn.w1.weight, layer.ffn.w3.weight, layer.ffn.w2.weight, xn2, x)
        xf = self._norm(x, m.norm.weight)
        logits = torch.empty(T, self.Vp, dtype=BF16, device=self.device)
        C.linear_fwd(xf, self.bf16(m.head.weight), logits[:, :self.V])
        out = logits[:, :self.V].view(B, S, self.V)
        return out, (x.view(B, S, self.D) if want_hidden else None)

    # ------------------------------------------------------- graph decode
    def _graph_key(self, B: int) -> tuple:
        m = self.model
        caches = tuple(layer.attn.kv_cache.data_ptr() for layer in m.layers)
        probe = (m.embed.weight, self._wq(m.layers[0].attn), m.layers[-1].attn.wo.weight, m.head.weight)
        return (B, caches, tuple((p.data_ptr(), p._version) for p in probe))

    @torch.no_grad()
    def decode(self, tokens: torch.Tensor, pos: torch.Tensor):
        """One decode step for ``tokens [B]`` at positions ``pos [B]``, replayed
        from a CUDA graph (captured on first use per batch size / cache
        buffers / weight version).  Returns ``(logits [B, V] bf16, hidden [B, D])``."""
        B = tokens.shape[0]
        for layer in self.model.layers:
            layer.attn._ensure_cache(B, self.device, BF16)
        key = self._graph_key(B)
        entry = self._graphs.get(key)
        if entry is None:
            for k in [k for k in self._graphs if k[0] == B]:
                del self._graphs[k]
            st = tokens.reshape(B, 1).long().clone()
            sp = pos.to(torch.int32).clone()
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):   # warm-up fills the weight caches outside the capture
                self.forward(st, pos=sp, want_hidden=True)
            torch.cuda.current_stream().wait_stream(side)
            graph = torch.cuda.CUDAGraph()
            # thread-local capture: a CUDA call from another thread (the data
            # loader's pin-memory thread allocating pinned buffers) must not
            # invalidate this capture
            with _ext.launch_scope() as scope, torch.cuda.graph(graph, capture_error_mode="thread_local"):
                out = self.forward(st, pos=sp, want_hidden=True)
            entry = (graph, st, sp, out, scope.count)
            self._graphs[key] = entry
        graph, st, sp, (logits, hidden), n_kernels = entry
        st.copy_(tokens.reshape(B, 1))
        sp.copy_(pos)
        graph.replay()
        _ext.add_launches(n_kernels)
        return logits[:, 0], hidden[:, 0]
