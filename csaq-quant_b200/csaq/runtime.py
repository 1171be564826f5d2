"""Static-shape decode runtime for Llama / Qwen2-family models with CSAQLinear layers.

The per-token work of a decoder layer runs as a fixed sequence of sm_100a
kernels over preallocated buffers, so a whole decode step (or a whole
self-speculative block: K draft steps, one verify pass over K+1 tokens and
the on-device acceptance) is captured once as a CUDA graph and replayed:

    RMSNorm -> fused q/k/v quantised GEMV -> RoPE + KV-cache write +
    split-K decode attention (one launch) -> o_proj GEMV (+ residual) -> RMSNorm ->
    fused gate/up GEMV -> SiLU gate -> down GEMV (+ residual)

The unquantised lm_head runs as an fp16 tier of the same GEMV kernel (every
token's logits are independent of the launch's token count, so speculative
and one-token decoding agree exactly); the embedding gather uses torch.

Tensor parallel (tp_group of W ranks): each rank holds column shards of
q/k/v/gate/up (its heads and its slice of the MLP width), row shards of
o/down (the matching input slice) and a vocabulary slice of the lm_head.
After o and down every rank all-gathers the partial outputs and adds them to
the residual stream in rank order (csaq_rank_sum), so a token's result does
not depend on how many tokens share the step; the greedy token is the argmax
over the gathered vocabulary slices.

Weights: the draft pass reads only the quantised tiers; the verify pass
reads the tiers without their protected rows plus the fp16 copies of those
rows, in the same launch (see CSAQLinear.gemv_descriptors).
"""

from __future__ import annotations

import ctypes
import math
import os
from dataclasses import dataclass
from typing import Dict, List, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _lib
from ._lib import check, dtype_code, lib, ptr
from .kernels import CSAQLinear

# Prefill chunks of at least this many tokens use the tcgen05 GEMM; smaller
# steps (decode, verify, short prompts) use the GEMV, which is faster there.
RUNTIME_GEMM_MIN_TOKENS = 256
# Prefill chunks of at least this many tokens use torch's fused attention
# (the decode attention kernel splits keys, not queries, and suits few rows).
PREFILL_SDPA_TOKENS = 32


def _layers_of(model: nn.Module):
    inner = getattr(model, "model", None)
    layers = getattr(inner, "layers", None) if inner is not None else None
    return inner, layers


def supports(model: nn.Module) -> bool:
    """True for Llama/Qwen2-style decoders whose attention/MLP linears are
    CSAQLinear, with 64- or 128-wide heads (the decode attention kernel's)."""
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
    return head_dim in (64, 128) and getattr(model, "lm_head", None) is not None


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
    gate_mask: Dict = None  # (layer, verify) -> bit mask of the gate tiers of the fused gate/up launch
    fuse_gate: bool = False  # the SiLU gate runs inside the gate/up and down GEMVs (csaq_qgemv_ext)
    y_part: Optional[torch.Tensor] = None    # TP: this rank's partial o/down output (M, H)
    y_all: Optional[torch.Tensor] = None     # TP: all ranks' partials (W, M, H)
    logits_all: Optional[torch.Tensor] = None  # TP: all ranks' vocabulary slices (W, M, V/W)


class _P2PExchange:
    """Peer-memory buffers for the tensor-parallel combine (csaq_tp_exchange_sum).

    Each rank allocates two partial buffers (rows x H each: parity 0 for the o
    projection, 1 for down) and a control block (flags, exchange count, CTA
    ticket, error counter) with csaq_p2p_alloc, sends the IPC handles over the
    process group, and maps every peer's buffers into its own address space."""

    def __init__(self, group, rank: int, world: int, rows: int, H: int, elem_bytes: int, dev):
        import torch.distributed as dist
        if world > _lib.MAX_RANKS:
            raise ValueError(f"peer-memory combine supports up to {_lib.MAX_RANKS} ranks")
        L = lib()
        self.rows, self.H, self.elem = rows, H, elem_bytes
        self.world, self.rank = world, rank
        self._own = []
        self._opened = []
        parts, ctl = c_void_p_(), c_void_p_()
        check(L.csaq_p2p_alloc(2 * rows * H * elem_bytes, ctypes.byref(parts)), "p2p_alloc")
        self._own.append(parts.value)
        check(L.csaq_p2p_alloc(256, ctypes.byref(ctl)), "p2p_alloc")
        self._own.append(ctl.value)
        h0 = (ctypes.c_uint8 * _lib.IPC_HANDLE_BYTES)()
        h1 = (ctypes.c_uint8 * _lib.IPC_HANDLE_BYTES)()
        check(L.csaq_ipc_handle(parts.value, h0), "ipc_handle")
        check(L.csaq_ipc_handle(ctl.value, h1), "ipc_handle")
        mine = torch.tensor(bytearray(bytes(h0) + bytes(h1)), dtype=torch.uint8, device=dev)
        allh = torch.empty(world, mine.numel(), dtype=torch.uint8, device=dev)
        dist.all_gather_into_tensor(allh, mine, group=group)
        allh = allh.cpu()
        g = _lib.CsaqP2PGroup()
        g.n_ranks, g.rank = world, rank
        for p in range(world):
            if p == rank:
                g.parts[p], g.flags[p] = parts.value, ctl.value
                continue
            hb = bytes(allh[p].tolist())
            ptrs = []
            for k in range(2):
                buf = (ctypes.c_uint8 * _lib.IPC_HANDLE_BYTES).from_buffer_copy(
                    hb[k * _lib.IPC_HANDLE_BYTES:(k + 1) * _lib.IPC_HANDLE_BYTES])
                out = c_void_p_()
                check(L.csaq_ipc_open(buf, ctypes.byref(out)), "ipc_open")
                self._opened.append(out.value)
                ptrs.append(out.value)
            g.parts[p], g.flags[p] = ptrs[0], ptrs[1]
        g.seq, g.ticket, g.err = ctl.value + 128, ctl.value + 136, ctl.value + 140
        self.group = g
        self.parts_ptr = parts.value
        dist.barrier(group=group)  # every rank has mapped every peer before any exchange

    def part_ptr(self, parity: int) -> int:
        return self.parts_ptr + parity * self.rows * self.H * self.elem

    def errors(self) -> int:
        n = ctypes.c_int64(0)
        check(lib().csaq_p2p_errors(ctypes.byref(self.group), ctypes.byref(n)), "p2p_errors")
        return int(n.value)

    def close(self, group=None) -> None:
        """Unmap the peers' buffers, then (after a barrier over `group`, when
        given, so that no peer still maps them) free this rank's own."""
        L = lib()
        torch.cuda.synchronize()
        for ptr in self._opened:
            L.csaq_ipc_close(ptr)
        self._opened = []
        if group is not None and self._own:
            import torch.distributed as dist
            dist.barrier(group=group)
        for ptr in self._own:
            L.csaq_p2p_free(ptr)
        self._own = []

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def c_void_p_():
    return ctypes.c_void_p(0)


class DecodeRuntime:
    """Decode / self-speculative generation for a quantised Llama/Qwen2 model."""

    def __init__(self, model: nn.Module, max_batch: int, max_len: int, lookahead: int = 4,
                 prefill_chunk: int = 512, tp_group=None):
        if not supports(model):
            raise ValueError("model is not a Llama/Qwen2 decoder with CSAQLinear layers")
        import torch.distributed as dist
        self.tp_group = tp_group
        self.tp = dist.get_world_size(tp_group) if tp_group is not None else 1
        self.tp_rank = dist.get_rank(tp_group) if tp_group is not None else 0
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
        W, r = self.tp, self.tp_rank
        for what, n in (("query heads", self.Hq), ("KV heads", self.Hkv), ("intermediate", self.I),
                        ("vocabulary", self.V)):
            if n % W:
                raise ValueError(f"{what} ({n}) do not split over {W} ranks")
        self.Vl = self.V // W  # this rank's vocabulary slice (tensor parallel)
        head = nn.Linear(self.H, self.Vl, bias=False, device="meta")
        head.weight = nn.Parameter(self.lm_w[r * self.Vl:(r + 1) * self.Vl].detach(), requires_grad=False)
        self.lm_head = CSAQLinear.from_tiers(head, {16: torch.arange(self.Vl)}, group_size=self.H)
        self.n_layers = len(layers)
        # this rank's linears: the model's own at TP 1; column shards of
        # q/k/v/gate/up and row shards of o/down otherwise
        self.lin = []
        for layer in layers:
            a, m = layer.self_attn, layer.mlp
            mods = {"q": a.q_proj, "k": a.k_proj, "v": a.v_proj, "o": a.o_proj, "gate": m.gate_proj,
                    "up": m.up_proj, "down": m.down_proj}
            if W > 1:
                mods = {k: v.tp_shard("row" if k in ("o", "down") else "col", r, W) for k, v in mods.items()}
            self.lin.append(mods)
        self.Hq_l, self.Hkv_l, self.I_l = self.Hq // W, self.Hkv // W, self.I // W
        L, B, Hkv, D = self.n_layers, self.B, self.Hkv_l, self.D
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
        # sampling at temperature > 0: Philox call counter (+ CTA ticket), the
        # draft steps' full-vocabulary logits (allocated on first use)
        self.rng = torch.zeros(2, dtype=i64, device=self.dev)
        self.dlog: Optional[torch.Tensor] = None
        self.shapes: Dict[int, _Shape] = {}
        # TP combine through peer memory (NVLink), unless CSAQ_TP_EXCHANGE=nccl
        self.p2p: Optional[_P2PExchange] = None
        if W > 1 and os.environ.get("CSAQ_TP_EXCHANGE", "p2p") != "nccl":
            rows = B * max(prefill_chunk, lookahead + 1)
            self.p2p = _P2PExchange(tp_group, self.tp_rank, W, rows, self.H, self.embed.element_size(), self.dev)
        self.graphs: Dict[str, torch.cuda.CUDAGraph] = {}
        self.launches_per_step: Dict[str, int] = {}
        # the peer-memory combines also run the RMSNorm that follows them
        # (CSAQ_TP_FUSE_NORM=0 keeps a separate csaq_rmsnorm launch)
        self.fuse_tp_norm = os.environ.get("CSAQ_TP_FUSE_NORM", "1") != "0"

    def release(self) -> None:
        """Drop the captured graphs and, under TP, the peer-memory buffers
        (a collective: every rank calls it)."""
        self.graphs.clear()
        if self.p2p is not None:
            self.p2p.close(self.tp_group)
            self.p2p = None

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
        B, H, D, Hq, Hkv, I = self.B, self.H, self.D, self.Hq_l, self.Hkv_l, self.I_l
        W = self.tp
        M = B * S
        mk = lambda *s: torch.zeros(*s, dtype=self.dtype, device=self.dev)
        nq, nkv = Hq * D, Hkv * D
        part_n = lib().csaq_attention_workspace_floats(B, S, Hq, Hkv, D, self.Lmax)
        sh = _Shape(S=S, M=M, x=mk(M, H), xn=mk(M, H), qkv=mk(M, nq + 2 * nkv), q_rot=mk(M, nq),
                    attn=mk(M, nq), gu=mk(M, 2 * I), h=mk(M, I), logits=mk(M, self.Vl),
                    part=torch.zeros(max(part_n, 1), dtype=torch.float32, device=self.dev),
                    descs={}, gate_mask={})
        # the SiLU gate fused into the gate/up and down GEMVs when both run the
        # tensor-core kernel (CSAQ_FUSE_GATE=0 keeps the separate csaq_silu_mul)
        fuse = (os.environ.get("CSAQ_FUSE_GATE", "1") != "0" and H % 128 == 0 and I % 128 == 0
                and self.dtype in (torch.bfloat16, torch.float16))
        if W > 1:
            sh.y_part, sh.y_all, sh.logits_all = mk(M, H), mk(W, M, H), mk(W, M, self.Vl)
        # at TP 1 the o/down GEMVs add the residual in their epilogue; with
        # TP each rank writes its partial and the combine adds them to x
        res_out = sh.x if W == 1 else sh.y_part
        res = sh.x if W == 1 else None
        for li, mods in enumerate(self.lin):
            for verify in (False, True):
                qkv = (mods["q"].gemv_descriptors(sh.qkv[:, :nq], verify)
                       + mods["k"].gemv_descriptors(sh.qkv[:, nq:nq + nkv], verify)
                       + mods["v"].gemv_descriptors(sh.qkv[:, nq + nkv:], verify))
                o = mods["o"].gemv_descriptors(res_out, verify, residual=res)
                gu = (mods["gate"].gemv_descriptors(sh.gu[:, :I], verify)
                      + mods["up"].gemv_descriptors(sh.gu[:, I:], verify))
                dn = mods["down"].gemv_descriptors(res_out, verify, residual=res)
                if self._p2p_for(M):  # partials straight into the peer-visible buffers
                    for parity, ds in ((0, o), (1, dn)):
                        for d in ds:
                            d.y, d.ldy = self.p2p.part_ptr(parity), H
                for name, d in (("qkv", qkv), ("o", o), ("gu", gu), ("down", dn)):
                    sh.descs[(li, name, verify)] = (_lib.tier_array(d), len(d))
                n_gate = len(mods["gate"].gemv_descriptors(sh.gu[:, :I], verify))
                sh.gate_mask[(li, verify)] = (1 << n_gate) - 1
                fuse = fuse and all(t.blocks or t.n_rows == 0 for t in gu + dn)
        sh.fuse_gate = fuse
        d = self.lm_head.gemv_descriptors(sh.logits)
        sh.descs[("lm", "all")] = (_lib.tier_array(d), len(d))
        d = self.lm_head.gemv_descriptors(sh.logits[: self.B])
        sh.descs[("lm", "last")] = (_lib.tier_array(d), len(d))
        self.shapes[S] = sh
        return sh

    # ── one step of S tokens per sequence ───────────────────────────────────
    def _gemv(self, arr_n, K: int, x: torch.Tensor, M: int, st: int) -> None:
        """One quantised linear launch: the decode GEMV for a few tokens, the
        tcgen05 GEMM for prefill chunks of RUNTIME_GEMM_MIN_TOKENS tokens or more."""
        arr, n = arr_n
        if M >= RUNTIME_GEMM_MIN_TOKENS and K % 64 == 0:
            check(lib().csaq_qgemm(arr, n, K, x.data_ptr(), self.dt, M, x.stride(0), st), "qgemm")
        else:
            check(lib().csaq_qgemv(arr, n, K, x.data_ptr(), self.dt, M, x.stride(0), st), "qgemv")

    @staticmethod
    def _fused_gate(sh: "_Shape") -> bool:
        return sh.fuse_gate and sh.M < RUNTIME_GEMM_MIN_TOKENS

    def _gemv_ext(self, arr_n, K: int, x: torch.Tensor, M: int, st: int, silu_tiers: int = 0,
                  x_mul: Optional[torch.Tensor] = None) -> None:
        """The GEMV with the SiLU gate fused in: silu_tiers stores silu(y) for
        the gate tiers; x_mul makes the input dtype(x * x_mul) (g' * u)."""
        arr, n = arr_n
        ext = _lib.CsaqGemvExt(silu_tiers, x_mul.data_ptr() if x_mul is not None else None)
        check(lib().csaq_qgemv_ext(arr, n, K, x.data_ptr(), self.dt, M, x.stride(0), ctypes.byref(ext), st),
              "qgemv_ext")

    def _p2p_for(self, M: int) -> bool:
        return self.p2p is not None and M <= self.p2p.rows

    def _combine(self, sh: _Shape, M: int, st: int, parity: int, norm_w: Optional[torch.Tensor] = None) -> bool:
        """TP: add every rank's partial o (parity 0) or down (parity 1) output
        to x in rank order: through peer memory when the step fits the
        exchange buffers, else an NCCL all-gather and csaq_rank_sum. Through
        peer memory with norm_w given, the same launch also writes
        xn = RMSNorm(x) with those weights; returns whether it did."""
        if self._p2p_for(M) and norm_w is not None and self.fuse_tp_norm:
            check(lib().csaq_tp_exchange_sum_rmsnorm(ctypes.byref(self.p2p.group), parity * self.p2p.rows * self.H,
                                                     self.H, sh.x.data_ptr(), self.H, M, self.H, norm_w.data_ptr(),
                                                     sh.xn.data_ptr(), self.H, self.eps, self.dt, st),
                  "tp_exchange_rmsnorm")
            return True
        if self._p2p_for(M):
            check(lib().csaq_tp_exchange_sum(ctypes.byref(self.p2p.group), parity * self.p2p.rows * self.H, self.H,
                                             sh.x.data_ptr(), self.H, M, self.H, self.dt, st), "tp_exchange")
            return False
        import torch.distributed as dist
        dist.all_gather_into_tensor(sh.y_all[:, :M], sh.y_part[:M], group=self.tp_group)
        H = self.H
        check(lib().csaq_rank_sum(sh.y_all.data_ptr(), self.tp, sh.y_all.stride(0), H, sh.x.data_ptr(), H, M, H, 1,
                                  self.dt, st), "rank_sum")
        return False

    def _attention(self, li: int, sh: "_Shape", S: int, pos: torch.Tensor, pos_host: Optional[int],
                   scale: float, st: int) -> None:
        """RoPE, the KV-cache write and attention of the step's queries over the
        cache. Prefill chunks of PREFILL_SDPA_TOKENS tokens or more (all
        sequences at the same host-known start) go to csaq_rope_kv and torch's
        fused scaled-dot-product attention; decode and verify steps to the
        split-key decode kernel with the rotation fused in."""
        qkv, nq, nkv = sh.qkv, self.Hq_l * self.D, self.Hkv_l * self.D
        if pos_host is not None and S >= PREFILL_SDPA_TOKENS:
            check(lib().csaq_rope_kv(qkv.data_ptr(), qkv.stride(0), qkv[:, nq:].data_ptr(), qkv.stride(0),
                                     qkv[:, nq + nkv:].data_ptr(), qkv.stride(0), pos.data_ptr(), self.B, S,
                                     self.Hq_l, self.Hkv_l, self.D, self.cos.data_ptr(), self.sin.data_ptr(),
                                     sh.q_rot.data_ptr(), self.k_cache[li].data_ptr(),
                                     self.v_cache[li].data_ptr(), self.Lmax, self.dt, st), "rope_kv")
            B, Hq, Hkv, D = self.B, self.Hq_l, self.Hkv_l, self.D
            n = pos_host + S
            q = sh.q_rot.view(B, S, Hq, D).transpose(1, 2)
            k = self.k_cache[li][:, :, :n]
            v = self.v_cache[li][:, :, :n]
            if pos_host == 0:
                o = F.scaled_dot_product_attention(q, k, v, is_causal=True, scale=scale, enable_gqa=Hq != Hkv)
            else:  # query i sits at position pos_host + i
                qi = torch.arange(S, device=self.dev).unsqueeze(1) + pos_host
                mask = torch.arange(n, device=self.dev).unsqueeze(0) <= qi
                o = F.scaled_dot_product_attention(q, k, v, attn_mask=mask, scale=scale, enable_gqa=Hq != Hkv)
            sh.attn.view(B, S, Hq, D).copy_(o.transpose(1, 2))
            return
        # decode / verify / short chunks: RoPE, the cache write and attention in one launch
        check(lib().csaq_decode_attention_rope(qkv.data_ptr(), qkv[:, nq:].data_ptr(), qkv[:, nq + nkv:].data_ptr(),
                                               qkv.stride(0), pos.data_ptr(), self.B, S, self.Hq_l, self.Hkv_l,
                                               self.D, self.cos.data_ptr(), self.sin.data_ptr(),
                                               self.k_cache[li].data_ptr(), self.v_cache[li].data_ptr(), self.Lmax,
                                               scale, sh.part.data_ptr(), self.tickets[li].data_ptr(),
                                               sh.attn.data_ptr(), self.dt, st), "attention")

    @torch.no_grad()
    def step(self, S: int, ids: torch.Tensor, pos: torch.Tensor, verify: bool,
             last_only: bool = False, pos_host: Optional[int] = None) -> torch.Tensor:
        """Run all layers for B*S tokens (ids: B*S int64, pos: per-sequence
        start positions; pos_host: the same start for every sequence, when the
        host knows it, as in prefill) and leave the logits of this rank's
        vocabulary slice in the shape's logits buffer (M rows, or the B rows of
        the last token of each sequence when last_only); returns the number of
        logit rows."""
        sh = self._shape(S)
        L = lib()
        st = torch.cuda.current_stream(self.dev).cuda_stream
        M, H, D, Hq, Hkv, I = sh.M, self.H, self.D, self.Hq_l, self.Hkv_l, self.I_l
        nq, nkv = Hq * D, Hkv * D
        torch.index_select(self.embed, 0, ids.view(-1), out=sh.x)
        scale = 1.0 / math.sqrt(D)
        fgate = self._fused_gate(sh)
        n_layers = len(self.layers)
        xn_ready = False  # the previous combine already wrote this layer's input norm into xn
        for li, layer in enumerate(self.layers):
            if not xn_ready:
                check(L.csaq_rmsnorm(sh.x.data_ptr(), H, layer.input_layernorm.weight.data_ptr(),
                                     sh.xn.data_ptr(), H, M, H, self.eps, self.dt, st), "rmsnorm")
            self._gemv(sh.descs[(li, "qkv", verify)], H, sh.xn, M, st)
            self._attention(li, sh, S, pos, pos_host, scale, st)
            self._gemv(sh.descs[(li, "o", verify)], nq, sh.attn, M, st)
            post = layer.post_attention_layernorm.weight
            if not (self.tp > 1 and self._combine(sh, M, st, 0, norm_w=post)):
                check(L.csaq_rmsnorm(sh.x.data_ptr(), H, post.data_ptr(),
                                     sh.xn.data_ptr(), H, M, H, self.eps, self.dt, st), "rmsnorm")
            if fgate:  # gate tiers store silu(y); the down GEMV multiplies g' and u in its record build
                self._gemv_ext(sh.descs[(li, "gu", verify)], H, sh.xn, M, st, silu_tiers=sh.gate_mask[(li, verify)])
                self._gemv_ext(sh.descs[(li, "down", verify)], I, sh.gu, M, st, x_mul=sh.gu[:, I:])
            else:
                self._gemv(sh.descs[(li, "gu", verify)], H, sh.xn, M, st)
                check(L.csaq_silu_mul(sh.gu.data_ptr(), sh.gu.stride(0), sh.gu[:, I:].data_ptr(),
                                      sh.gu.stride(0), sh.h.data_ptr(), I, M, I, self.dt, st), "silu_mul")
                self._gemv(sh.descs[(li, "down", verify)], I, sh.h, M, st)
            nxt = self.layers[li + 1].input_layernorm.weight if li + 1 < n_layers else self.final_norm
            xn_ready = self.tp > 1 and self._combine(sh, M, st, 1, norm_w=nxt)
        if not xn_ready:
            check(L.csaq_rmsnorm(sh.x.data_ptr(), H, self.final_norm.data_ptr(), sh.xn.data_ptr(), H, M, H,
                                 self.eps, self.dt, st), "rmsnorm")
        if last_only and S > 1:
            arr, n = sh.descs[("lm", "last")]
            last = sh.xn[S - 1:]  # rows S-1, 2S-1, ...: the last token of each sequence
            check(L.csaq_qgemv(arr, n, H, last.data_ptr(), self.dt, self.B, S * H, st), "lm_head")
            return self.B
        self._gemv(sh.descs[("lm", "all")], H, sh.xn, M, st)
        return M

    def argmax(self, S: int, rows: int, out: torch.Tensor) -> None:
        """Greedy tokens of the first `rows` logit rows of the last step over
        the whole vocabulary (gathering every rank's slice under TP)."""
        sh = self.shapes[S]
        st = torch.cuda.current_stream(self.dev).cuda_stream
        Vl = self.Vl
        if self.tp > 1:
            src = self._gather_logits(sh, rows)
            n_parts, pstride = self.tp, rows * Vl
        else:
            src, n_parts, pstride = sh.logits, 1, 0
        check(lib().csaq_argmax_parts(src.data_ptr(), n_parts, pstride, Vl, Vl, rows, out.data_ptr(), self.dt, st),
              "argmax")

    def logits_full(self, S: int, rows: int) -> torch.Tensor:
        """The full-vocabulary logits of the last step (a copy; gathers under TP)."""
        sh = self.shapes[S]
        if self.tp == 1:
            return sh.logits[:rows].clone()
        return self._gather_logits(sh, rows).permute(1, 0, 2).reshape(rows, self.V).clone()

    def _gather_logits(self, sh: _Shape, rows: int) -> torch.Tensor:
        """Every rank's vocabulary slice of the first `rows` logit rows, as a
        contiguous (W, rows, V/W) view of the shape's gather buffer."""
        import torch.distributed as dist
        out = sh.logits_all.view(-1)[: self.tp * rows * self.Vl].view(self.tp, rows, self.Vl)
        dist.all_gather_into_tensor(out, sh.logits[:rows], group=self.tp_group)
        return out

    def kernels_per_step(self, S: int) -> int:
        """Own (libcsaq) kernel launches in one step of up to 16 tokens per
        GEMV launch: per layer 2 RMSNorm, 4 GEMV, RoPE with attention (one
        launch), SiLU unless the GEMVs run it (and 2 rank-order combines under
        TP, which through peer memory also run the RMSNorm that follows
        them); plus the final RMSNorm, the lm_head GEMV and the argmax."""
        sh = self._shape(S)
        silu = 0 if self._fused_gate(sh) else 1
        norms = self._norm_launches(sh.M)
        return self.n_layers * (5 + silu + (2 if self.tp > 1 else 0)) + norms + 2

    def _norm_launches(self, M: int) -> int:
        """Separate RMSNorm launches of one step of M tokens: 2 per layer and
        the final one, or only the first layer's input norm when the peer
        memory combines run the others."""
        return 1 if (self.tp > 1 and self._p2p_for(M) and self.fuse_tp_norm) else 2 * self.n_layers + 1

    def prefill_kernels(self, P: int, verify: bool = True) -> int:
        """Own kernel launches of reset() for a P-token prompt: per chunk and
        layer 2 RMSNorm, RoPE, SiLU (unless inside the GEMVs), the decode attention kernel for chunks
        below PREFILL_SDPA_TOKENS (torch's fused attention above), the
        combines under TP, and the linears (one tcgen05 GEMM launch per tier
        from RUNTIME_GEMM_MIN_TOKENS tokens, else one GEMV launch per 16 tokens
        or fewer); then the final RMSNorm, the lm_head GEMV and the argmax."""
        n, C = 0, self.prefill_chunk
        for s0 in range(0, P, C):
            S = min(C, P - s0)
            M = self.B * S
            sh = self._shape(S)
            for li in range(self.n_layers):
                for name in ("qkv", "o", "gu", "down"):
                    arr, nd = sh.descs[(li, name, verify)]
                    if M >= RUNTIME_GEMM_MIN_TOKENS:
                        n += sum(1 for i in range(nd) if arr[i].n_rows > 0)
                    else:
                        n += -(-M // 16)
                silu = 0 if self._fused_gate(sh) else 1  # SiLU, unless inside the GEMVs
                n += 1 + silu + (2 if self.tp > 1 else 0)  # RoPE (+ SDPA) or fused RoPE + attention
            n += self._norm_launches(M) + 1  # the RMSNorms and the lm_head
        return n + 1

    # ── generation ──────────────────────────────────────────────────────────
    @torch.no_grad()
    def reset(self, prompts: torch.Tensor, max_new: int, verify: bool = True, temperature: float = 0.0,
              top_p: float = 1.0, seed: int = 0) -> None:
        """Prefill `prompts` (B, P) (verify or draft weights) and set the state
        for generating `max_new` tokens (the first comes from the prefill:
        greedy at temperature 0, else sampled)."""
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
            self.step(S, chunk.contiguous().view(-1), self.pos0, verify=verify, last_only=True, pos_host=s0)
        self.prefill_logits = self.logits_full(S, self.B)
        self.rng.zero_()
        if temperature > 0.0:
            self.sample(S, self.B, self.next_tok, temperature, top_p, seed)
        else:
            self.argmax(S, self.B, self.next_tok)
        self.out_tokens[:, 0] = self.next_tok
        self.n_out.fill_(1)
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
            self.step(1, self.next_tok, self.cur_pos, verify=False)
            self.argmax(1, B, self.next_tok)
            self.draft[:, k].copy_(self.next_tok)
            self.vin[:, k + 1].copy_(self.next_tok)
            self.cur_pos.add_(1)
        self.step(K + 1, self.vin, self.pos0, verify=True)
        self.argmax(K + 1, B * (K + 1), self.argmax_buf)
        self.vt.copy_(self.argmax_buf.view(B, K + 1))
        check(L.csaq_spec_accept(self.draft.data_ptr(), self.vt.data_ptr(), B, K, self.pos0.data_ptr(),
                                 self.out_tokens.data_ptr(), self.n_out.data_ptr(), self.cap,
                                 self.next_tok.data_ptr(), self.n_new.data_ptr(), self.stats.data_ptr(),
                                 self.remaining.data_ptr(), st), "spec_accept")

    def _logit_parts(self, S: int, rows: int):
        """(pointer, n_parts, part_stride, ld, part_len) of the first `rows`
        full-vocabulary logit rows of the last step (gathered under TP)."""
        sh = self.shapes[S]
        if self.tp > 1:
            src = self._gather_logits(sh, rows)
            return src.data_ptr(), self.tp, rows * self.Vl, self.Vl, self.Vl
        return sh.logits.data_ptr(), 1, 0, self.Vl, self.Vl

    def sample(self, S: int, rows: int, out: torch.Tensor, temperature: float, top_p: float, seed: int) -> None:
        """Draw one token per logit row of the last step (csaq_sample_rows)."""
        st = torch.cuda.current_stream(self.dev).cuda_stream
        ptr, n_parts, pstride, ld, plen = self._logit_parts(S, rows)
        check(lib().csaq_sample_rows(ptr, n_parts, pstride, ld, plen, rows, float(temperature), float(top_p),
                                     int(seed) & 0xFFFFFFFFFFFFFFFF, self.rng.data_ptr(), out.data_ptr(), self.dt,
                                     st), "sample")

    def _spec_iteration_sample(self, temperature: float, top_p: float, seed: int) -> None:
        """One self-speculative iteration with sampled drafts and on-device
        rejection sampling (no host synchronisation)."""
        K, B, V = self.K, self.B, self.V
        L = lib()
        st = torch.cuda.current_stream(self.dev).cuda_stream
        if self.dlog is None or self.dlog.shape != (K, B, V):
            self.dlog = torch.zeros(K, B, V, dtype=self.dtype, device=self.dev)
        self.vin[:, 0].copy_(self.next_tok)
        self.cur_pos.copy_(self.pos0)
        for k in range(K):
            self.step(1, self.next_tok, self.cur_pos, verify=False)
            self.dlog[k].copy_(self.logits_view(1, B))
            check(L.csaq_sample_rows(self.dlog[k].data_ptr(), 1, 0, V, V, B, float(temperature), float(top_p),
                                     int(seed) & 0xFFFFFFFFFFFFFFFF, self.rng.data_ptr(), self.next_tok.data_ptr(),
                                     self.dt, st), "sample")
            self.draft[:, k].copy_(self.next_tok)
            self.vin[:, k + 1].copy_(self.next_tok)
            self.cur_pos.add_(1)
        self.step(K + 1, self.vin, self.pos0, verify=True)
        ptr, n_parts, pstride, ld, plen = self._logit_parts(K + 1, B * (K + 1))
        check(L.csaq_spec_sample_verify(self.draft.data_ptr(), self.dlog.data_ptr(), ptr, n_parts, pstride, ld, plen,
                                        B, K, float(temperature), float(top_p), int(seed) & 0xFFFFFFFFFFFFFFFF,
                                        self.rng.data_ptr(), self.vt.data_ptr(), self.dt, st), "spec_sample")
        check(L.csaq_spec_accept(self.draft.data_ptr(), self.vt.data_ptr(), B, K, self.pos0.data_ptr(),
                                 self.out_tokens.data_ptr(), self.n_out.data_ptr(), self.cap,
                                 self.next_tok.data_ptr(), self.n_new.data_ptr(), self.stats.data_ptr(),
                                 self.remaining.data_ptr(), st), "spec_accept")

    def logits_view(self, S: int, rows: int) -> torch.Tensor:
        """The first `rows` full-vocabulary logit rows of the last step as a
        (rows, V) tensor (a view at TP 1; gathered and rearranged under TP)."""
        sh = self.shapes[S]
        if self.tp == 1:
            return sh.logits[:rows]
        return self._gather_logits(sh, rows).permute(1, 0, 2).reshape(rows, self.V)

    @torch.no_grad()
    def _greedy_step(self, verify: bool) -> None:
        L = lib()
        st = torch.cuda.current_stream(self.dev).cuda_stream
        self.step(1, self.next_tok, self.pos0, verify=verify)
        self.argmax(1, self.B, self.argmax_buf[: self.B])
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
                self.stats, self.remaining, self.out_tokens, self.n_out, self.k_cache, self.v_cache, self.rng]

    def generate_speculative(self, max_new: int, temperature: float = 0.0, top_p: float = 1.0,
                             seed: int = 0) -> int:
        """Self-speculative decode after reset(); greedy at temperature 0, else
        sampled drafts with on-device rejection sampling; returns iterations."""
        if temperature > 0.0:
            key = f"spec_sample_{temperature!r}_{top_p!r}_{seed}"
            g = self._graph(key, lambda: self._spec_iteration_sample(temperature, top_p, seed))
        else:
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
