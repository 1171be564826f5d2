"""csaq.inference — self-speculative decoding on B200.

Drop-in for csaq-quant's ``csaq/inference.py``: ``SpeculativeReport`` and
``CSAQInferenceEngine`` with the same constructor, ``generate`` signature and
report fields.

Two paths:
* Llama/Qwen2 decoders with greedy decoding (temperature 0) run on
  ``csaq.runtime.DecodeRuntime``: static KV cache, fused sm_100a kernels, one
  CUDA graph per speculative block (K draft steps reading only quantised
  weights, one verify pass whose protected rows come from their fp16 copies
  in the same GEMV launches, on-device acceptance).
* Other models, and sampling, run the HF forward (whose linears are
  CSAQLinear) in a Python loop with a DynamicCache.

Semantics fixed relative to the reference (csaq/inference.py:396-574): the
verify pass really uses the verify weights (the reference sets an override
its forward never reads, :225), draft token k is compared with the
verifier's prediction at position k (the reference uses k+1, :486), and the
prompt is prefilled (the reference starts from the last prompt token with an
empty cache, :423-440). Greedy speculative output therefore equals greedy
decoding with the verify weights.
"""

from __future__ import annotations

import time
import warnings
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional, Tuple

import numpy as np
import torch
import torch.nn as nn
import torch.nn.functional as F

from .kernels import CSAQLinear


@dataclass
class SpeculativeReport:
    """Performance record of one generation (csaq/inference.py:37-111)."""

    tokens_generated: int = 0
    tokens_accepted: int = 0
    tokens_rejected: int = 0
    draft_calls: int = 0
    verify_calls: int = 0
    total_wallclock_s: float = 0.0
    mode: str = "speculative"
    error_log: str = ""
    _token_times: List[float] = field(default_factory=list)

    @property
    def acceptance_rate(self) -> float:
        total = self.tokens_accepted + self.tokens_rejected
        return self.tokens_accepted / max(total, 1)

    @property
    def speedup_factor(self) -> float:
        return self.tokens_generated / max(self.draft_calls + self.verify_calls, 1)

    @property
    def inter_token_latency_ms(self) -> float:
        return (self.total_wallclock_s * 1e3) / max(self.tokens_generated, 1)

    @property
    def block_efficiency(self) -> float:
        return self.tokens_accepted / max(self.verify_calls, 1)

    @property
    def p95_latency_ms(self) -> float:
        if not self._token_times:
            return float("nan")
        return float(np.percentile(self._token_times, 95)) * 1000.0

    @property
    def tokens_per_second(self) -> float:
        if self.total_wallclock_s <= 0:
            return 0.0
        return self.tokens_generated / self.total_wallclock_s

    def summary(self) -> Dict[str, Any]:
        return {
            "mode": self.mode,
            "tokens_generated": self.tokens_generated,
            "acceptance_rate": round(self.acceptance_rate, 4),
            "speedup_factor": round(self.speedup_factor, 2),
            "inter_token_latency_ms": round(self.inter_token_latency_ms, 2),
            "p95_latency_ms": round(self.p95_latency_ms, 2) if not np.isnan(self.p95_latency_ms) else "nan",
            "tokens_per_second": round(self.tokens_per_second, 2),
            "block_efficiency": round(self.block_efficiency, 2),
            "draft_calls": self.draft_calls,
            "verify_calls": self.verify_calls,
            "wallclock_s": round(self.total_wallclock_s, 3),
            "error_log": self.error_log,
        }

    def __repr__(self) -> str:  # pragma: no cover
        return (f"SpeculativeReport(tokens={self.tokens_generated}, acceptance={self.acceptance_rate:.2%}, "
                f"speedup={self.speedup_factor:.2f}x, latency={self.inter_token_latency_ms:.1f}ms/tok)")


_HookEntry = Tuple[CSAQLinear, torch.Tensor, torch.Tensor, Optional[torch.Tensor]]


class CSAQInferenceEngine:
    """Self-speculative decoding engine (csaq/inference.py:125-574)."""

    def __init__(self, model: nn.Module, causal_map: Dict[str, List[int]], tokenizer: Optional[Any] = None,
                 verbose: bool = True, tp_group: Any = None) -> None:
        self.model = model
        self.tp_group = tp_group  # torch.distributed group: tensor-parallel decode runtime
        self.causal_map = causal_map
        self.tokenizer = tokenizer
        self.verbose = verbose
        self.device = next(model.parameters(), next(model.buffers())).device
        self._in_verify = False
        self._warmup_complete = False
        self.telemetry: Dict[str, int] = {"total_tokens": 0, "accepted_tokens": 0, "backpressure_events": 0}
        self._hooks: List[_HookEntry] = []
        self._runtime = None
        self._runtime_key = None
        self._build_hooks()
        if not self._hooks:
            warnings.warn(
                "[CSAQ] CSAQInferenceEngine found 0 hooked layers.  Speculative decoding will fall back "
                "to standard generation.  Make sure the model was quantised with csaq.quantize().",
                stacklevel=2)

    # ── hook discovery (csaq/inference.py:184-215) ──────────────────────────
    def _build_hooks(self) -> None:
        self._hooks.clear()
        for name in self.causal_map:
            module = self._resolve_module(name)
            if not isinstance(module, CSAQLinear):
                continue
            if not (hasattr(module, "_csaq_fp16_backup") and hasattr(module, "_csaq_hi_rows")):
                continue
            self._hooks.append((module, module._csaq_hi_rows, module._csaq_fp16_backup,
                                getattr(module, "_csaq_quant_stash", None)))

    def _resolve_module(self, name: str) -> Optional[nn.Module]:
        parts = name.split(".")
        if parts and parts[-1] == "weight":
            parts = parts[:-1]
        mod: nn.Module = self.model
        for p in parts:
            child = getattr(mod, p, None)
            if child is None:
                return None
            mod = child
        return mod if isinstance(mod, nn.Module) else None

    # ── verify / draft weights (csaq/inference.py:219-237) ──────────────────
    def _swap_to_verify(self) -> None:
        for module, _, _, _ in self._hooks:
            module.verify_mode = True
        self._in_verify = True

    def _swap_to_draft(self) -> None:
        for module, _, _, _ in self._hooks:
            module.verify_mode = False
        self._in_verify = False

    def _ensure_draft_state(self) -> None:
        if self._in_verify:
            self._swap_to_draft()

    # ── KV cache utilities (the roles of csaq/inference.py:241-265) ─────────
    @staticmethod
    def _kv_len(cache: Optional[Any]) -> int:
        """Positions a cache holds: 0 for none; a transformers Cache reports
        its own length, a legacy ((k, v), ...) tuple is read off the first key
        (batch, heads, positions, head_dim)."""
        if cache is None:
            return 0
        length = getattr(cache, "get_seq_length", None)
        if length is not None:
            return int(length())
        return int(cache[0][0].shape[-2])

    @staticmethod
    def _truncate_kv(cache: Optional[Any], length: int) -> Optional[Any]:
        """Drop every position from `length` on: in place for a transformers
        Cache (its crop), as a new tuple for the legacy layout."""
        if cache is None:
            return None
        crop = getattr(cache, "crop", None)
        if crop is not None:
            crop(length)
            return cache
        return tuple(tuple(t[..., :length, :] for t in layer) for layer in cache)

    # ── sampling (the rule of csaq/inference.py:269-304) ────────────────────
    @staticmethod
    def _sample(logits: torch.Tensor, temperature: float, top_p: float,
                greedy: bool) -> Tuple[torch.Tensor, torch.Tensor]:
        """One token per row, shape (rows, 1), and the probabilities drawn from.

        NaN logits read as 0 and all are clamped to [-50, 50]. Greedy takes the
        argmax. Otherwise the logits are divided by the temperature and, for
        top_p < 1, token j stays in the draw only while the probability mass of
        the tokens ranked above it is at most top_p (the smallest set whose mass
        exceeds top_p, ties broken by the sort). Rows whose probabilities are
        not a usable distribution fall back to the argmax. This is the same rule
        csaq_sample_rows applies on the device."""
        z = torch.nan_to_num(logits.float(), nan=0.0).clamp(-50.0, 50.0)
        if greedy:
            return z.argmax(-1, keepdim=True), torch.softmax(z, -1)
        p = torch.softmax(z / max(temperature, 1e-8), -1)
        if top_p < 1.0:
            ranked, order = p.sort(-1, descending=True)
            above = ranked.cumsum(-1) - ranked
            keep = torch.zeros_like(p, dtype=torch.bool).scatter_(-1, order, above <= top_p)
            p = torch.where(keep, p, torch.zeros_like(p))
            p = p / p.sum(-1, keepdim=True)
        if not (torch.isfinite(p).all() and bool((p.sum(-1) > 1e-8).all())):
            return z.argmax(-1, keepdim=True), p
        return torch.multinomial(p, 1), p

    def warmup(self, n: int = 3) -> None:
        if self._warmup_complete:
            return
        dummy = torch.tensor([[1]], device=self.device)
        with torch.no_grad():
            for _ in range(n):
                self.generate(dummy, max_new_tokens=2, speculative=bool(self._hooks), temperature=0.0)
        self._warmup_complete = True
        if self.verbose:
            print("[CSAQ] Inference engine warmup complete.")

    # ── fast path ───────────────────────────────────────────────────────────
    def _fast_ok(self, input_ids: torch.Tensor, temperature: float, speculative: bool = False) -> bool:
        """The static runtime serves greedy decoding and, at temperature > 0,
        self-speculative sampling (on-device rejection sampling)."""
        from . import runtime
        return ((temperature == 0.0 or (speculative and bool(self._hooks))) and torch.cuda.is_available()
                and input_ids is not None and input_ids.dim() == 2 and runtime.supports(self.model))

    def runtime(self, batch: int, max_len: int, lookahead: int):
        """The (cached) static decode runtime for this batch / length / lookahead."""
        from .runtime import DecodeRuntime
        key = (batch, lookahead)
        rt = self._runtime
        if rt is None or self._runtime_key != key or rt.Lmax < max_len:
            self._runtime = None
            torch.cuda.empty_cache()
            L = max(max_len, 64)
            L = (L + 63) // 64 * 64
            rt = DecodeRuntime(self.model, max_batch=batch, max_len=L, lookahead=lookahead,
                               tp_group=self.tp_group)
            self._runtime, self._runtime_key = rt, key
        return rt

    def _generate_fast(self, input_ids: torch.Tensor, speculative: bool, lookahead: int,
                       max_new_tokens: int, temperature: float = 0.0, top_p: float = 1.0,
                       seed: Optional[int] = None) -> Tuple[torch.Tensor, SpeculativeReport]:
        B, P = input_ids.shape
        K = max(1, lookahead)
        rt = self.runtime(B, P + max_new_tokens + 2 * K + 2, K)
        ids_dev = input_ids.to(self.device, non_blocking=True)
        t0 = time.time()
        if seed is None:
            seed = int(torch.randint(0, 2 ** 62, (1,)).item()) if temperature > 0.0 else 0
        rt.reset(ids_dev, max_new_tokens, verify=speculative, temperature=temperature, top_p=top_p, seed=seed)
        report = SpeculativeReport(mode="speculative" if speculative else "standard")
        if max_new_tokens > 1:
            if speculative:
                iters = rt.generate_speculative(max_new_tokens, temperature=temperature, top_p=top_p, seed=seed)
                st = rt.spec_stats()
                report.draft_calls = iters * K
                report.verify_calls = iters
                report.tokens_accepted = st["accepted"]
                report.tokens_rejected = st["rejected"]
            else:
                rt.generate_greedy(max_new_tokens, verify=False)
                report.draft_calls = max_new_tokens - 1
        out = rt.outputs()[:, :max_new_tokens]
        result = torch.cat([ids_dev, out], dim=1)
        torch.cuda.synchronize()
        report.total_wallclock_s = time.time() - t0
        report.tokens_generated = int(out.shape[1]) * B if B > 1 else int(out.shape[1])
        if not speculative:
            report.tokens_accepted = report.tokens_generated
        self.telemetry["total_tokens"] += report.tokens_generated
        self.telemetry["accepted_tokens"] += report.tokens_accepted
        return result.to(input_ids.device), report

    # ── public API (csaq/inference.py:325-392) ──────────────────────────────
    def generate(self, input_ids: Optional[torch.Tensor] = None, *, speculative: bool = False,
                 lookahead: int = 4, temperature: float = 1.0, top_p: float = 1.0,
                 max_new_tokens: int = 128, **kwargs: Any) -> Tuple[torch.Tensor, SpeculativeReport]:
        if input_ids is not None and self._fast_ok(input_ids, temperature, speculative):
            with torch.no_grad():
                return self._generate_fast(input_ids, speculative and bool(self._hooks), lookahead,
                                           max_new_tokens, temperature=temperature, top_p=top_p,
                                           seed=kwargs.get("seed"))
        if speculative and self._hooks:
            return self._generate_speculative(input_ids, max_new_tokens, lookahead, temperature, top_p)
        self._ensure_draft_state()
        t0 = time.time()
        gen_kwargs: Dict[str, Any] = {"input_ids": input_ids, "max_new_tokens": max_new_tokens,
                                      "do_sample": temperature > 0, **kwargs}
        if temperature > 0:
            gen_kwargs["temperature"] = temperature
        if top_p < 1.0:
            gen_kwargs["top_p"] = top_p
        pad_id = ((self.tokenizer.pad_token_id if self.tokenizer else None)
                  or getattr(getattr(self.model, "config", None), "eos_token_id", None))
        if pad_id is not None:
            gen_kwargs.setdefault("pad_token_id", pad_id)
        output = self.model.generate(**gen_kwargs)
        elapsed = time.time() - t0
        p_len = input_ids.shape[-1] if input_ids is not None else 0
        n_new = max(0, output.shape[-1] - p_len)
        return output, SpeculativeReport(tokens_generated=n_new, tokens_accepted=n_new,
                                         total_wallclock_s=elapsed, mode="standard")

    # ── general speculative loop (HF forward) ───────────────────────────────
    @torch.no_grad()
    def _generate_speculative(self, input_ids: torch.Tensor, max_new_tokens: int, lookahead: int,
                              temperature: float, top_p: float) -> Tuple[torch.Tensor, SpeculativeReport]:
        report = SpeculativeReport()
        t0 = time.time()
        greedy = temperature == 0.0
        self.model.eval()
        generated = input_ids.clone().to(self.device)
        eos_id = ((self.tokenizer.eos_token_id if self.tokenizer else None)
                  or getattr(getattr(self.model, "config", None), "eos_token_id", None))
        produced = 0
        last_time = time.time()
        try:
            # prefill with the verify weights: cache holds all but the last token
            self._swap_to_verify()
            past = None
            if generated.shape[1] > 1:
                out = self.model(input_ids=generated[:, :-1], past_key_values=None, use_cache=True)
                past = out.past_key_values
            self._swap_to_draft()
            while produced < max_new_tokens:
                K = min(lookahead, max_new_tokens - produced)
                kv_before = self._kv_len(past)
                d_tokens, d_logits = [], []
                nxt = generated[:, -1:]
                for _ in range(K):
                    out = self.model(input_ids=nxt, past_key_values=past, use_cache=True)
                    past = out.past_key_values
                    logits = out.logits[:, -1, :]
                    report.draft_calls += 1
                    tok, _ = self._sample(logits, temperature, top_p, greedy)
                    d_tokens.append(tok)
                    d_logits.append(logits)
                    nxt = tok
                draft_ids = torch.cat(d_tokens, dim=-1)
                past = self._truncate_kv(past, kv_before)
                vin = torch.cat([generated[:, -1:], draft_ids], dim=-1)
                try:
                    self._swap_to_verify()
                    v_out = self.model(input_ids=vin, past_key_values=past, use_cache=True)
                    report.verify_calls += 1
                finally:
                    self._swap_to_draft()
                v_logits = v_out.logits
                past = v_out.past_key_values
                new: List[int] = []
                n_acc = 0
                for k in range(K):
                    d_tok = int(draft_ids[0, k])
                    if greedy:
                        v_tok = int(v_logits[0, k].argmax())
                        if v_tok == d_tok:
                            n_acc += 1
                            new.append(d_tok)
                            continue
                        new.append(v_tok)
                        break
                    p = F.softmax(v_logits[:, k].float() / max(temperature, 1e-8), dim=-1)
                    q = F.softmax(d_logits[k].float() / max(temperature, 1e-8), dim=-1)
                    ratio = p[0, d_tok] / q[0, d_tok].clamp(min=1e-10)
                    if float(torch.rand(1, device=p.device)) < min(1.0, float(ratio)):
                        n_acc += 1
                        new.append(d_tok)
                        continue
                    resid = (p - q).clamp(min=0.0)
                    s = resid.sum()
                    new.append(int(torch.multinomial(resid / s, 1)) if s > 1e-8 else int(p.argmax()))
                    break
                if n_acc == K:  # every draft accepted: the verifier's next token is free
                    tok, _ = self._sample(v_logits[:, K], temperature, top_p, greedy)
                    new.append(int(tok))
                new = new[: max_new_tokens - produced]
                generated = torch.cat([generated, torch.tensor([new], device=self.device,
                                                               dtype=generated.dtype)], dim=-1)
                produced += len(new)
                report.tokens_accepted += min(n_acc, len(new))
                report.tokens_rejected += K - min(n_acc, len(new))
                report.tokens_generated += len(new)
                now = time.time()
                report._token_times.extend([(now - last_time) / len(new)] * len(new))
                last_time = now
                self.telemetry["total_tokens"] += len(new)
                self.telemetry["accepted_tokens"] += n_acc
                if n_acc / max(K, 1) < 0.20:
                    self.telemetry["backpressure_events"] += 1
                past = self._truncate_kv(past, kv_before + len(new))
                if eos_id is not None and new and new[-1] == eos_id:
                    break
        except RuntimeError as exc:
            msg = f"RuntimeError during speculative decoding: {exc}"
            warnings.warn(f"[CSAQ] {msg}  Falling back to standard generation.")
            report.error_log = msg
            self._ensure_draft_state()
            rem = max(0, max_new_tokens - produced)
            if rem > 0:
                generated, fb = self.generate(input_ids=generated, speculative=False, max_new_tokens=rem)
                report.tokens_generated += fb.tokens_generated
        report.total_wallclock_s = time.time() - t0
        return generated, report
