"""Static-shape decode runtime for Llama / Qwen2-family models with CSAQLinear layers.

The per-token work of a decoder layer runs as a fixed sequence of sm_100a
kernels over preallocated buffers, so a whole decode step (or a whole
self-speculative block: K draft steps, one verify pass over K+1 tokens and
the on-device acceptance) is captured once as a CUDA graph and replayed:

    RMSNorm -> fused q/k/v quantised GEMV -> RoPE + KV-cache write ->
    split-K decode attention -> o_proj GEMV (+ residual) -> RMSNorm ->
    fused gate/up GEMV -> SiLU gate -> down GEMV (+ residual)

The unquantised lm_head runs as an fp16 tier of the same GEMV kernel (every
token's logits are independent of the launch's token count, so speculative
and one-token decoding agree exactly); the embedding gather and the
vocabulary argmax use torch (ATen) kernels.

Weights: the draft pass reads only the quantised tiers; the verify pass
reads the tiers without their protected rows plus the fp16 copies of those
rows, in the same launch (see CSAQLinear.gemv_descriptors).
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Dict, List, Optional

import torch
import torch.nn as nn

from . import _lib
from ._lib import check, dtype_code, lib, ptr
from .kernels import CSAQLinear


def _layers_of(model: nn.Module):
    inner = getattr(model, "model", None)
    layers = getattr(inner, "layers", None) if inner is not None else None
    return inner, layers


def supports(model: nn.Module) -> bool:
    """True for Llama/Qwen2-style decoders whose attention/MLP linears are CSAQLinear."""
    inner, layers = _layers_of(model)
    if layers is None or len(layers) == 0:
        return False
    l0 = layers[0]
    attn = getattr(l0, "self_attn", None)
    mlp = getattr(l0, "mlp", None)
    if attn is None or mlp is None:
        return False
    names = [(attn, "q_proj"), (attn, "k_proj"), (attn, "v_proj"), (attn, "o_proj"),
             (mlp, "gate_proj"), (mlp, "up_proj"), (mlp, "down_proj")]
    if not all(isinstance(getattr(m, n, None), CSAQLinear) for m, n in names):
        return False
    cfg = getattr(model, "config", None)
    head_dim = getattr(cfg, "head_dim", None) or (cfg.hidden_size // cfg.num_attention_heads)
    return head_dim == 128 and getattr(model, "lm_head", None) is not None


@dataclass
class _Shape:
    S: int          # tokens per sequence in the step
    M: int          # B * S rows
    x: torch.Tensor
    xn: torch.Tensor
    qkv: torch.Tensor
    q_rot: torch.Tensor
    attn: torch.Tensor
    gu: torch.Tensor
    h: torch.Tensor
    logits: torch.Tensor
    part: torch.Tensor
    descs: Dict  # (layer, name, verify) -> ctypes array + count


class DecodeRuntime:
    """Decode / self-speculative generation for a quantised Llama/Qwen2 model."""

    def __init__(self, model: nn.Module, max_batch: int, max_len: int, lookahead: int = 4,
                 prefill_chunk: int = 64):
        if not supports(model):
            raise ValueError("model is not a Llama/Qwen2 decoder with CSAQLinear layers")
        cfg = model.config
        inner, layers = _layers_of(model)
        self.model = model
        self.cfg = cfg
        self.layers = layers
        self.B = max_batch
        self.K = lookahead
        self.Lmax = max_len
        self.prefill_chunk = prefill_chunk
        self.H = cfg.hidden_size
        self.Hq = cfg.num_attention_heads
        self.Hkv = getattr(cfg, "num_key_value_heads", None) or self.Hq
        self.D = getattr(cfg, "head_dim", None) or self.H // self.Hq
        self.I = cfg.intermediate_size
        self.V = model.lm_head.weight.shape[0]
        self.eps = float(getattr(cfg, "rms_norm_eps", 1e-6))
        self.embed = inner.embed_tokens.weight.detach()
        self.dev = self.embed.device
        self.dtype = self.embed.dtype
        self.dt = dtype_code(self.dtype)
        self.final_norm = inner.norm.weight.detach()
        self.lm_w = model.lm_head.weight.detach()
        # lm_head as one fp16 tier of the quantised-linear kernel: every
        # token's logits are computed independently of how many tokens share
        # the launch, so the verify pass over K+1 tokens and one-token steps
        # give identical logits (and identical argmax)
        head = nn.Linear(self.H, self.V, bias=False, device="meta")
        head.weight = nn.Parameter(self.lm_w.detach(), requires_grad=False)
        self.lm_head = CSAQLinear.from_tiers(head, {16: torch.arange(self.V)}, group_size=self.H)
        self.n_layers = len(layers)
        L, B, Hkv, D = self.n_layers, self.B, self.Hkv, self.D
        self.k_cache = torch.zeros(L, B, Hkv, max_len, D, dtype=self.dtype, device=self.dev)
        self.v_cache = torch.zeros(L, B, Hkv, max_len, D, dtype=self.dtype, device=self.dev)
        self.tickets = torch.zeros(L, B * Hkv, dtype=torch.int32, device=self.dev)
        self._rope_tables(inner)
        # generation state
        i32, i64 = torch.int32, torch.int64
        self.pos0 = torch.zeros(B, dtype=i32, device=self.dev)
        self.cur_pos = torch.zeros(B, dtype=i32, device=self.dev)
        self.next_tok = torch.zeros(B, dtype=i64, device=self.dev)
        self.draft = torch.zeros(B, max(lookahead, 1), dtype=i64, device=self.dev)
        self.vin = torch.zeros(B, lookahead + 1, dtype=i64, device=self.dev)
        self.vt = torch.zeros(B, lookahead + 1, dtype=i64, device=self.dev)
        self.n_new = torch.zeros(B, dtype=i32, device=self.dev)
        self.stats = torch.zeros(3, dtype=i64, device=self.dev)
        self.remaining = torch.zeros(B, dtype=i32, device=self.dev)
        self.cap = max_len
        self.out_tokens = torch.zeros(B, self.cap, dtype=i64, device=self.dev)
        self.n_out = torch.zeros(B, dtype=i32, device=self.dev)
        self.argmax_buf = torch.zeros(B * (lookahead + 1), dtype=i64, device=self.dev)
        self.shapes: Dict[int, _Shape] = {}
        self.graphs: Dict[str, torch.cuda.CUDAGraph] = {}
        self.launches_per_step: Dict[str, int] = {}

    # ── setup ────────────────────────────────────────────────────────────────
    def _rope_tables(self, inner):
        rot = getattr(inner, "rotary_emb", None)
        pos = torch.arange(self.Lmax, device=self.dev).unsqueeze(0)
        dummy = torch.zeros(1, 1, self.D, dtype=self.dtype, device=self.dev)
        if rot is not None:
            cos, sin = rot(dummy, pos)
        else:
            inv = 1.0 / (getattr(self.cfg, "rope_theta", 10000.0) **
                         (torch.arange(0, self.D, 2, device=self.dev).float() / self.D))
            f = pos[0].float()[:, None] * inv[None, :]
            emb = torch.cat([f, f], dim=-1)
            cos, sin = emb.cos().to(self.dtype), emb.sin().to(self.dtype)
        self.cos = cos.reshape(self.Lmax, self.D).float().contiguous()
        self.sin = sin.reshape(self.Lmax, self.D).float().contiguous()

    def _shape(self, S: int) -> _Shape:
        sh = self.shapes.get(S)
        if sh is not None:
            return sh
        B, H, D, Hq, Hkv, I = self.B, self.H, self.D, self.Hq, self.Hkv, self.I
        M = B * S
        mk = lambda *s: torch.zeros(*s, dtype=self.dtype, device=self.dev)
        nq, nkv = Hq * D, Hkv * D
        part_n = lib().csaq_attention_workspace_floats(B, S, Hq, Hkv, D, self.Lmax)
        sh = _Shape(S=S, M=M, x=mk(M, H), xn=mk(M, H), qkv=mk(M, nq + 2 * nkv), q_rot=mk(M, nq),
                    attn=mk(M, nq), gu=mk(M, 2 * I), h=mk(M, I), logits=mk(M, self.V),
                    part=torch.zeros(max(part_n, 1), dtype=torch.float32, device=self.dev),
                    descs={})
        for li, layer in enumerate(self.layers):
            a, m = layer.self_attn, layer.mlp
            for verify in (False, True):
                qkv = (a.q_proj.gemv_descriptors(sh.qkv[:, :nq], verify)
                       + a.k_proj.gemv_descriptors(sh.qkv[:, nq:nq + nkv], verify)
                       + a.v_proj.gemv_descriptors(sh.qkv[:, nq + nkv:], verify))
                o = a.o_proj.gemv_descriptors(sh.x, verify, residual=sh.x)
                gu = (m.gate_proj.gemv_descriptors(sh.gu[:, :I], verify)
                      + m.up_proj.gemv_descriptors(sh.gu[:, I:], verify))
                dn = m.down_proj.gemv_descriptors(sh.x, verify, residual=sh.x)
                for name, d in (("qkv", qkv), ("o", o), ("gu", gu), ("down", dn)):
                    sh.descs[(li, name, verify)] = (_lib.tier_array(d), len(d))
        d = self.lm_head.gemv_descriptors(sh.logits)
        sh.descs[("lm", "all")] = (_lib.tier_array(d), len(d))
        d = self.lm_head.gemv_descriptors(sh.logits[: self.B])
        sh.descs[("lm", "last")] = (_lib.tier_array(d), len(d))
        self.shapes[S] = sh
        return sh

    # ── one step of S tokens per sequence ───────────────────────────────────
    def _gemv(self, arr_n, K: int, x: torch.Tensor, M: int, st: int) -> None:
        arr, n = arr_n
        check(lib().csaq_qgemv(arr, n, K, x.data_ptr(), self.dt, M, x.stride(0), st), "qgemv")

    @torch.no_grad()
    def step(self, S: int, ids: torch.Tensor, pos: torch.Tensor, verify: bool,
             last_only: bool = False) -> torch.Tensor:
        """Run all layers for B*S tokens (ids: B*S int64, pos: per-sequence
        start positions) and return the logits buffer (M, V) (or (B, V) rows
        of the last token of each sequence when last_only)."""
        sh = self._shape(S)
        L = lib()
        st = torch.cuda.current_stream(self.dev).cuda_stream
        M, H, D, Hq, Hkv, I = sh.M, self.H, self.D, self.Hq, self.Hkv, self.I
        nq, nkv = Hq * D, Hkv * D
        torch.index_select(self.embed, 0, ids.view(-1), out=sh.x)
        scale = 1.0 / math.sqrt(D)
        for li, layer in enumerate(self.layers):
            a, m = layer.self_attn, layer.mlp
            check(L.csaq_rmsnorm(sh.x.data_ptr(), H, layer.input_layernorm.weight.data_ptr(),
                                 sh.xn.data_ptr(), H, M, H, self.eps, self.dt, st), "rmsnorm")
            self._gemv(sh.descs[(li, "qkv", verify)], H, sh.xn, M, st)
            qkv = sh.qkv
            check(L.csaq_rope_kv(qkv.data_ptr(), qkv.stride(0), qkv[:, nq:].data_ptr(), qkv.stride(0),
                                 qkv[:, nq + nkv:].data_ptr(), qkv.stride(0), pos.data_ptr(), self.B, S,
                                 Hq, Hkv, D, self.cos.data_ptr(), self.sin.data_ptr(),
                                 sh.q_rot.data_ptr(), self.k_cache[li].data_ptr(),
                                 self.v_cache[li].data_ptr(), self.Lmax, self.dt, st), "rope_kv")
            check(L.csaq_decode_attention(sh.q_rot.data_ptr(), self.k_cache[li].data_ptr(),
                                          self.v_cache[li].data_ptr(), pos.data_ptr(), self.B, S, Hq,
                                          Hkv, D, self.Lmax, scale, sh.part.data_ptr(),
                                          self.tickets[li].data_ptr(), sh.attn.data_ptr(), self.dt,
                                          st), "attention")
            self._gemv(sh.descs[(li, "o", verify)], nq, sh.attn, M, st)
            check(L.csaq_rmsnorm(sh.x.data_ptr(), H, layer.post_attention_layernorm.weight.data_ptr(),
                                 sh.xn.data_ptr(), H, M, H, self.eps, self.dt, st), "rmsnorm")
            self._gemv(sh.descs[(li, "gu", verify)], H, sh.xn, M, st)
            check(L.csaq_silu_mul(sh.gu.data_ptr(), sh.gu.stride(0), sh.gu[:, I:].data_ptr(),
                                  sh.gu.stride(0), sh.h.data_ptr(), I, M, I, self.dt, st), "silu_mul")
            self._gemv(sh.descs[(li, "down", verify)], I, sh.h, M, st)
        check(L.csaq_rmsnorm(sh.x.data_ptr(), H, self.final_norm.data_ptr(), sh.xn.data_ptr(), H, M, H,
                             self.eps, self.dt, st), "rmsnorm")
        if last_only and S > 1:
            arr, n = sh.descs[("lm", "last")]
            last = sh.xn[S - 1:]  # rows S-1, 2S-1, ...: the last token of each sequence
            check(L.csaq_qgemv(arr, n, H, last.data_ptr(), self.dt, self.B, S * H, st), "lm_head")
            return sh.logits[: self.B]
        self._gemv(sh.descs[("lm", "all")], H, sh.xn, M, st)
        return sh.logits

    def kernels_per_step(self, S: int) -> int:
        """Own (libcsaq) kernel launches in one step of up to 16 tokens per
        GEMV launch: per layer 2 RMSNorm, 4 GEMV, RoPE, attention, SiLU; plus
        the final RMSNorm and the lm_head GEMV."""
        return self.n_layers * 9 + 2

    # ── generation ──────────────────────────────────────────────────────────
    @torch.no_grad()
    def reset(self, prompts: torch.Tensor, max_new: int, verify: bool = True) -> None:
        """Prefill `prompts` (B, P) (verify or draft weights) and set the state
        for generating `max_new` tokens (the first comes from the prefill)."""
        B, P = prompts.shape
        if B != self.B:
            raise ValueError(f"runtime built for batch {self.B}, got {B}")
        if P + max_new + 2 * self.K + 2 > self.Lmax:
            raise ValueError("prompt + max_new + 2*lookahead + 2 exceeds max_len")
        self.k_cache.zero_()
        self.v_cache.zero_()
        self.n_out.zero_()
        self.stats.zero_()
        prompts = prompts.to(self.dev)
        C = self.prefill_chunk
        for s0 in range(0, P, C):
            chunk = prompts[:, s0:s0 + C]
            S = chunk.shape[1]
            self.pos0.fill_(s0)
            logits = self.step(S, chunk.contiguous().view(-1), self.pos0, verify=verify, last_only=True)
        self.prefill_logits = logits[: self.B].clone()
        first = torch.argmax(logits[: self.B], dim=-1)
        self.out_tokens[:, 0] = first
        self.n_out.fill_(1)
        self.next_tok.copy_(first)
        self.pos0.fill_(P)
        self.remaining.fill_(max_new - 1)

    @torch.no_grad()
    def _spec_iteration(self) -> None:
        K, B = self.K, self.B
        L = lib()
        st = torch.cuda.current_stream(self.dev).cuda_stream
        self.vin[:, 0].copy_(self.next_tok)
        self.cur_pos.copy_(self.pos0)
        for k in range(K):
            logits = self.step(1, self.next_tok, self.cur_pos, verify=False)
            torch.argmax(logits[:B], dim=-1, out=self.next_tok)
            self.draft[:, k].copy_(self.next_tok)
            self.vin[:, k + 1].copy_(self.next_tok)
            self.cur_pos.add_(1)
        logits = self.step(K + 1, self.vin, self.pos0, verify=True)
        torch.argmax(logits, dim=-1, out=self.argmax_buf)
        self.vt.copy_(self.argmax_buf.view(B, K + 1))
        check(L.csaq_spec_accept(self.draft.data_ptr(), self.vt.data_ptr(), B, K, self.pos0.data_ptr(),
                                 self.out_tokens.data_ptr(), self.n_out.data_ptr(), self.cap,
                                 self.next_tok.data_ptr(), self.n_new.data_ptr(), self.stats.data_ptr(),
                                 self.remaining.data_ptr(), st), "spec_accept")

    @torch.no_grad()
    def _greedy_step(self, verify: bool) -> None:
        L = lib()
        st = torch.cuda.current_stream(self.dev).cuda_stream
        logits = self.step(1, self.next_tok, self.pos0, verify=verify)
        torch.argmax(logits[: self.B], dim=-1, out=self.argmax_buf[: self.B])
        check(L.csaq_greedy_commit(self.argmax_buf.data_ptr(), self.B, self.pos0.data_ptr(),
                                   self.out_tokens.data_ptr(), self.n_out.data_ptr(), self.cap,
                                   self.next_tok.data_ptr(), self.remaining.data_ptr(), st), "commit")

    def _graph(self, name: str, fn) -> torch.cuda.CUDAGraph:
        g = self.graphs.get(name)
        if g is None:
            # warm up outside capture (allocations, descriptors, lazy init)
            s = torch.cuda.Stream(self.dev)
            s.wait_stream(torch.cuda.current_stream(self.dev))
            saved = [t.clone() for t in self._state()]
            with torch.cuda.stream(s):
                fn()
            torch.cuda.current_stream(self.dev).wait_stream(s)
            for t, v in zip(self._state(), saved):
                t.copy_(v)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                fn()
            for t, v in zip(self._state(), saved):
                t.copy_(v)
            self.graphs[name] = g
        return g

    def _state(self) -> List[torch.Tensor]:
        return [self.pos0, self.cur_pos, self.next_tok, self.draft, self.vin, self.vt, self.n_new,
                self.stats, self.remaining, self.out_tokens, self.n_out, self.k_cache, self.v_cache]

    def generate_speculative(self, max_new: int) -> int:
        """Self-speculative greedy decode after reset(); returns iterations."""
        g = self._graph("spec", self._spec_iteration)
        iters = 0
        rem_host = torch.empty(1, dtype=torch.int32, pin_memory=True)
        while True:
            g.replay()
            iters += 1
            rem_host.copy_(self.remaining.max().view(1), non_blocking=True)
            torch.cuda.current_stream(self.dev).synchronize()
            if int(rem_host[0]) <= 0:
                break
        return iters

    def generate_greedy(self, max_new: int, verify: bool = True) -> int:
        """Plain greedy decode (one token per step) after reset()."""
        g = self._graph("greedy_v" if verify else "greedy_d", lambda: self._greedy_step(verify))
        for _ in range(max_new - 1):
            g.replay()
        return max_new - 1

    def outputs(self) -> torch.Tensor:
        n = int(self.n_out.max())
        return self.out_tokens[:, :n]

    def spec_stats(self) -> Dict[str, int]:
        a, r, blocks = (int(v) for v in self.stats.tolist())
        return {"accepted": a, "rejected": r, "blocks": blocks}
