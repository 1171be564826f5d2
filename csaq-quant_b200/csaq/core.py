"""csaq.core — the three-phase pipeline on B200.

Drop-in for csaq-quant's ``csaq/core.py`` (same names, arguments, return
values): calibration profiling (salience and co-activation cliques), the
bit-budget solver, and application of the quantised layers.

Device work runs in libcsaq_b200.so:
* forward hooks turn each linear's output into a bit-packed top-k
  co-activation mask (csaq_act_mask) that stays on the GPU;
* |grad * W| salience accumulates in fp32 on the GPU (csaq_salience_accum);
* cliques come from popcount intersection counts (csaq_coact_counts), fp32
  Jaccard threshold bits (csaq_jaccard_bits) and the seed-order greedy
  partition (csaq_greedy_cliques).
The solver and the layer bookkeeping are host orchestration, as in the
reference.

Layer layout: with ``config.group_size == -1`` (the default) every layer is
the reference's uniform CSAQLinear built by ``CSAQLinear.from_cliques``;
with ``group_size > 0`` (e.g. 128) each layer becomes a mixed-row layer whose
rows carry the bit-width the solver gave their clique.
"""

from __future__ import annotations

import contextlib
import gc
import math
import time
import warnings
from collections import defaultdict
from typing import Any, Dict, Iterator, List, Optional, Tuple, Union

import numpy as np
import torch
import torch.nn as nn

from . import _lib
from ._lib import check, dtype_code, lib, ptr, stream_of
from .config import CSAQConfig
from .kernels import CSAQLinear, _get_submodule, inject_csaq_linear

BudgetMap = Dict[str, List[Dict[str, Any]]]
SalienceMap = Dict[str, torch.Tensor]
CliqueMap = Dict[str, List[List[int]]]


def _prepare_calib_data(calib_data: Union[List[Dict[str, torch.Tensor]], List[str]], model: nn.Module,
                        device: str = "cpu", tokenizer: Any = None,
                        seq_len: int = 128) -> List[Dict[str, torch.Tensor]]:
    """Normalise calibration data to tokenised batches (csaq/core.py:40-89)."""
    if not calib_data:
        raise ValueError("[CSAQ] calib_data is empty.")
    if isinstance(calib_data[0], dict):
        out = []
        for batch in calib_data:
            if "attention_mask" not in batch:
                batch = dict(batch)
                batch["attention_mask"] = torch.ones_like(batch["input_ids"])
            out.append({k: v.to(device) for k, v in batch.items()})
        return out
    if isinstance(calib_data[0], str):
        if tokenizer is None:
            raise ValueError(
                "[CSAQ] calib_data contains raw strings but no tokenizer was provided.  Pass "
                "tokenizer= to quantize(), or pre-tokenise your texts using "
                "build_calibration_data() before calling quantize().")
        batches = []
        for text in calib_data:
            enc = tokenizer(str(text), return_tensors="pt", max_length=seq_len, truncation=True,
                            padding="max_length")
            batches.append({k: v.to(device) for k, v in enc.items()})
        return batches
    raise TypeError("[CSAQ] Unsupported calib_data type.  Expected List[Dict] or List[str].")


def _linear_modules(model: nn.Module) -> Iterator[Tuple[str, nn.Linear]]:
    """Quantisable nn.Linear layers (csaq/core.py:92-102)."""
    skip = ("lm_head", "embed_tokens", "embed_positions", "wte", "wpe")
    for name, module in model.named_modules():
        if not isinstance(module, nn.Linear) or module.weight is None:
            continue
        if any(p in name for p in skip):
            continue
        yield name, module


# ─────────────────────────────────────────────────────────────────────────────
# GPU calibration primitives
# ─────────────────────────────────────────────────────────────────────────────

class MaskHistory:
    """Bit-packed co-activation masks of one layer, channel-major, on the GPU.

    Grows by doubling; bit t of channel c is token t of the calibration run.
    """

    def __init__(self, channels: int, device: torch.device, capacity_tokens: int = 4096):
        self.C = channels
        self.dev = device
        self.n_tok = 0
        self.words = max(1, (capacity_tokens + 31) // 32)
        self.bits = torch.zeros(channels, self.words, dtype=torch.int32, device=device)
        self.tok_thr = torch.zeros(1, dtype=torch.int32, device=device)

    def _reserve(self, n_tok: int) -> None:
        need = (self.n_tok + n_tok + 31) // 32 + 1
        if need <= self.words:
            return
        words = max(need, 2 * self.words)
        nb = torch.zeros(self.C, words, dtype=torch.int32, device=self.dev)
        nb[:, : self.words] = self.bits
        self.bits, self.words = nb, words

    def append(self, act: torch.Tensor, mode: int, thr: float = 0.0, k: int = 1) -> None:
        a = act.detach().reshape(-1, act.shape[-1])
        if not a.is_cuda:
            a = a.to(self.dev)
        if a.dtype not in (torch.float32, torch.float16, torch.bfloat16):
            a = a.float()
        if a.stride(1) != 1:
            a = a.contiguous()
        n = a.shape[0]
        if n == 0:
            return
        # keep every append on a 32-token boundary: pad the running count
        self.n_tok = (self.n_tok + 31) // 32 * 32 if self.n_tok % 32 else self.n_tok
        self._reserve(n)
        if mode == 1 and self.tok_thr.numel() < n:
            self.tok_thr = torch.zeros(n, dtype=torch.int32, device=self.dev)
        check(lib().csaq_act_mask(a.data_ptr(), dtype_code(a.dtype), n, self.C, a.stride(0), mode,
                                  float(thr), int(k), self.tok_thr.data_ptr(), self.bits.data_ptr(),
                                  self.words, self.n_tok, stream_of(a)), "act_mask")
        self.n_tok += n

    def words_used(self) -> int:
        return (self.n_tok + 31) // 32


def coactivation_counts(bits: torch.Tensor, n_words: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """Exact intersection counts I (C, C) int32 and activation counts f (C,) int32."""
    C = bits.shape[0]
    inter = torch.empty(C, C, dtype=torch.int32, device=bits.device)
    f = torch.empty(C, dtype=torch.int32, device=bits.device)
    check(lib().csaq_coact_counts(bits.data_ptr(), C, n_words, bits.stride(0), inter.data_ptr(), C,
                                  f.data_ptr(), stream_of(bits)), "coact_counts")
    return inter, f


def jaccard_cliques(inter: torch.Tensor, f: torch.Tensor, threshold: float) -> List[List[int]]:
    """Seed-order greedy cliques over Jaccard >= threshold (csaq/core.py:263-285)."""
    C = inter.shape[0]
    words = (C + 31) // 32
    adj = torch.empty(C, words, dtype=torch.int32, device=inter.device)
    thr32 = float(torch.tensor(threshold, dtype=torch.float32))
    st = stream_of(inter)
    check(lib().csaq_jaccard_bits(inter.data_ptr(), inter.stride(0), f.data_ptr(), C, thr32,
                                  adj.data_ptr(), words, st), "jaccard_bits")
    labels = torch.empty(C, dtype=torch.int32, device=inter.device)
    n = torch.zeros(1, dtype=torch.int32, device=inter.device)
    check(lib().csaq_greedy_cliques(adj.data_ptr(), words, C, labels.data_ptr(), n.data_ptr(), st),
          "greedy_cliques")
    return cliques_from_labels(labels)


def spearman_rho(ranks: torch.Tensor, prev_ranks: torch.Tensor) -> float:
    """Spearman's rho of two rank vectors without ties: 1 - 6 sum(d^2) / (n (n^2 - 1))
    (csaq/core.py:218-222)."""
    n_r = float(ranks.numel())
    d = ranks - prev_ranks
    return 1.0 - (6.0 * (d ** 2).sum().item()) / (n_r * (n_r ** 2 - 1))


def cliques_from_labels(labels: torch.Tensor) -> List[List[int]]:
    """Clique lists (ascending members, seed first) from per-channel labels."""
    lab = labels.to(torch.int64).cpu()
    order = torch.argsort(lab, stable=True)
    counts = torch.bincount(lab)
    return [g.tolist() for g in torch.split(order, counts.tolist())]


def salience_accumulate(acc: torch.Tensor, grad: torch.Tensor, weight: torch.Tensor) -> None:
    """acc += |grad * weight| in fp32 (csaq/core.py:204-210)."""
    g = grad.contiguous()
    w = weight.contiguous()
    if g.dtype != w.dtype:
        g = g.to(w.dtype)
    if w.dtype not in (torch.float32, torch.float16, torch.bfloat16):
        g, w = g.float(), w.float()
    check(lib().csaq_salience_accum(g.data_ptr(), w.data_ptr(), dtype_code(w.dtype), w.numel(),
                                    acc.data_ptr(), stream_of(acc)), "salience_accum")


# ─────────────────────────────────────────────────────────────────────────────
# Phase 1 & 2: CausalProfiler (csaq/core.py:109-287)
# ─────────────────────────────────────────────────────────────────────────────

class CausalProfiler:
    """Causal salience (|dL/dw * w|) and Jaccard co-activation cliques.

    Same interface as csaq/core.py:109-287. Masks and salience accumulators
    live on the GPU of each layer; the Spearman early stop follows
    csaq/core.py:212-230.
    """

    _EARLY_STOP_RHO: float = 0.99
    _EARLY_STOP_MIN_BATCHES: int = 16
    _EVAL_STRIDE: int = 8
    _SPEARMAN_SAMPLE: int = 50_000

    def __init__(self, model: nn.Module, config: CSAQConfig, dp_group: Any = None) -> None:
        self.model = model
        self.config = config
        # data parallel over calibration batches: rank r profiles batches r, r+W, ...;
        # salience (fp32) and co-activation counts (int32) are summed over the ranks
        self.dp_group = dp_group
        self.salience: SalienceMap = {}
        self._masks: Dict[str, MaskHistory] = {}
        self._hooks: List[Any] = []
        self._modules: Dict[str, nn.Linear] = {}
        dev = _lib.cuda_device()
        for name, module in _linear_modules(model):
            self._modules[name] = module
            mdev = module.weight.device if module.weight.is_cuda else dev
            self.salience[name] = torch.zeros(module.weight.shape, dtype=torch.float32, device=mdev)
            self._masks[name] = MaskHistory(module.weight.shape[0], mdev)
            self._register_hook(name, module)
            self._register_salience_hook(name, module)

    def _register_hook(self, name: str, module: nn.Linear) -> None:
        alpha = self.config.salience_alpha

        def forward_hook(m: nn.Module, inp, out: torch.Tensor) -> None:
            with torch.no_grad():
                C = out.shape[-1]
                frac = min(1.0, 0.1 * alpha)
                k = max(1, int(frac * C))
                self._masks[name].append(out, mode=1, k=k)

        self._hooks.append(module.register_forward_hook(forward_hook))

    def _register_salience_hook(self, name: str, module: nn.Linear) -> None:
        """|grad * W| (csaq/core.py:204-210) accumulated as soon as the weight's
        gradient is complete, during the backward pass, and the gradient freed
        right away: the salience kernels overlap the rest of the backward and
        the gradients of all layers never coexist (16 GB of bf16 gradients at
        the Llama-3-8B shape). A batch whose backward fails part-way keeps
        the salience of the layers whose gradients had completed (the
        reference, which accumulates after the backward, drops the batch)."""
        w = module.weight
        if not hasattr(w, "register_post_accumulate_grad_hook"):
            return

        def hook(param: torch.Tensor) -> None:
            if param.grad is None:
                return
            acc = self.salience[name]
            g, data = param.grad, param.data
            if not g.is_cuda:
                g, data = g.to(acc.device), data.to(acc.device)
            with torch.no_grad():
                salience_accumulate(acc, g, data)
            param.grad = None

        self._hooks.append(w.register_post_accumulate_grad_hook(hook))

    def add_activation_masks(self, name: str, act: torch.Tensor, threshold: Optional[float] = None) -> None:
        """Append co-activation masks from activations directly: act > threshold
        when given (in act's dtype), else the hook's top-k rule."""
        mh = self._masks[name]
        if threshold is None:
            k = max(1, int(min(1.0, 0.1 * self.config.salience_alpha) * act.shape[-1]))
            mh.append(act, mode=1, k=k)
        else:
            thr = float(torch.tensor(threshold, dtype=act.dtype)) if act.is_floating_point() else threshold
            mh.append(act, mode=0, thr=thr)

    def _dp(self):
        if self.dp_group is None:
            return None, 0, 1
        import torch.distributed as dist
        return dist, dist.get_rank(self.dp_group), dist.get_world_size(self.dp_group)

    def profile(self, calib_data: List[Dict[str, torch.Tensor]],
                verbose: bool = True) -> Tuple[SalienceMap, CliqueMap]:
        dist, rank, world = self._dp()
        if world > 1:
            calib_data = list(calib_data)[rank::world]
        self.model.train()
        n_samples = len(calib_data)
        actual_batches = 0
        prev_ranks = None
        eval_idx = None
        first_device = next(self.model.parameters()).device
        for i, batch in enumerate(calib_data):
            actual_batches += 1
            batch = {k: v.to(first_device) if isinstance(v, torch.Tensor) else v for k, v in batch.items()}
            labels = batch.get("labels", batch.get("input_ids"))
            try:
                out = self.model(**batch, labels=labels)
                out.loss.backward()
            except Exception as exc:  # the reference skips a failing batch (csaq/core.py:199-202)
                warnings.warn(f"[CSAQ] Skipping calibration batch {i}: {exc}")
                self.model.zero_grad()
                continue
            with torch.no_grad():  # weights without the gradient hook (accumulated there otherwise)
                for name, module in self._modules.items():
                    if module.weight.grad is not None:
                        acc = self.salience[name]
                        g, w = module.weight.grad, module.weight.data
                        if not g.is_cuda:
                            g, w = g.to(acc.device), w.to(acc.device)
                        salience_accumulate(acc, g, w)
            self.model.zero_grad()
            if (i + 1) % self._EVAL_STRIDE == 0 and (i + 1) >= self._EARLY_STOP_MIN_BATCHES:
                if eval_idx is None:
                    eval_idx = self._spearman_indices(first_device, dist, world)
                sample = self._salience_sample(eval_idx, first_device)
                if world > 1:  # every rank ranks the same (all-reduced) sample, so all stop together
                    dist.all_reduce(sample, group=self.dp_group)
                ranks = sample.argsort().argsort().float()
                if prev_ranks is not None:
                    rho = spearman_rho(ranks, prev_ranks)
                    if rho >= self._EARLY_STOP_RHO:
                        if verbose:
                            print(f"[CSAQ] Early stop at batch {i + 1}/{n_samples} (ρ={rho:.4f})")
                        break
                prev_ranks = ranks.clone()
        if world > 1:
            n_b = torch.tensor([actual_batches], dtype=torch.int64, device=first_device)
            dist.all_reduce(n_b, group=self.dp_group)
            actual_batches = int(n_b)
            for name in self.salience:
                dist.all_reduce(self.salience[name], group=self.dp_group)
        for name in self.salience:
            acc = self.salience[name]
            check(lib().csaq_salience_finalize(acc.data_ptr(), acc.numel(), max(actual_batches, 1),
                                               stream_of(acc)), "salience_finalize")
        for h in self._hooks:
            h.remove()
        self.model.eval()
        return self.salience, self._build_cliques()

    # Sampling without replacement by torch.randperm(N) allocates N indices;
    # above this many salience entries a chunked sampler is used instead.
    _RANDPERM_MAX: int = 1 << 26

    def _spearman_indices(self, device, dist, world: int) -> torch.Tensor:
        """Flat indices (into the layers' salience in module order) of the
        early-stop sample: torch.randperm(N)[:50000] on the host generator as
        in csaq/core.py:214-216 while N <= _RANDPERM_MAX; above it, 50000
        distinct indices drawn uniformly with the host generator (the
        reference's randperm would allocate N int64 values: 56 GB at the 8B
        shape). Under data parallelism rank 0 draws and broadcasts."""
        N = sum(self.salience[n].numel() for n in self._modules)
        size = min(self._SPEARMAN_SAMPLE, N)
        if world > 1 and dist.get_rank(self.dp_group) != 0:
            idx = torch.empty(size, dtype=torch.int64)
        elif N <= self._RANDPERM_MAX:
            idx = torch.randperm(N)[:size]
        else:
            picked = torch.empty(0, dtype=torch.int64)
            while picked.numel() < size:
                cand = torch.randint(0, N, (2 * size,), dtype=torch.int64)
                picked = torch.cat([picked, cand])
                # keep the first occurrence of every index, in draw order
                uniq, inv = torch.unique(picked, return_inverse=True)
                first = torch.full((uniq.numel(),), picked.numel(), dtype=torch.int64)
                first.scatter_reduce_(0, inv, torch.arange(picked.numel()), reduce="amin")
                picked = picked[torch.sort(first).values]
            idx = picked[:size]
        if world > 1:
            idx = idx.to(device)
            dist.broadcast(idx, 0, group=self.dp_group)
        return idx.to(device)

    def _salience_sample(self, idx: torch.Tensor, device) -> torch.Tensor:
        """all_s[idx] for all_s = cat(salience[n].flatten() for n in modules),
        gathered layer by layer without building all_s."""
        out = torch.empty(idx.numel(), dtype=torch.float32, device=device)
        off = 0
        for n in self._modules:
            t = self.salience[n]
            sel = (idx >= off) & (idx < off + t.numel())
            if bool(sel.any()):
                loc = (idx[sel] - off).to(t.device)
                out[sel] = t.reshape(-1)[loc].to(device=device, dtype=torch.float32)
            off += t.numel()
        return out

    def _build_cliques(self) -> CliqueMap:
        """Partition each layer's output channels (csaq/core.py:240-287)."""
        if self.config.clique_mode == "per_channel":
            return {name: [[i] for i in range(m.weight.shape[0])] for name, m in self._modules.items()}
        out: CliqueMap = {}
        for name, module in self._modules.items():
            mh = self._masks[name]
            C = module.weight.shape[0]
            if mh.n_tok == 0 and self.dp_group is None:
                out[name] = [[i] for i in range(C)]
                continue
            inter, f = coactivation_counts(mh.bits, mh.words_used())
            dist, _, world = self._dp()
            if world > 1:  # integer sums: every rank gets the same counts, hence the same cliques
                dist.all_reduce(inter, group=self.dp_group)
                dist.all_reduce(f, group=self.dp_group)
            out[name] = jaccard_cliques(inter, f, self.config.clique_threshold)
            del inter
            self._masks[name] = MaskHistory(C, mh.dev)
        return out


# ─────────────────────────────────────────────────────────────────────────────
# Phase 3: solver (csaq/core.py:294-361)
# ─────────────────────────────────────────────────────────────────────────────

_SCAN_WINDOW = 65536  # cliques per cumulative-sum window of the upgrade scan


@contextlib.contextmanager
def _gc_paused() -> Iterator[None]:
    """Pause Python's cyclic garbage collector while a large acyclic result
    (millions of small dicts and lists) is built; its collections would
    otherwise rescan the growing result several times over."""
    was = gc.isenabled()
    gc.disable()
    try:
        yield
    finally:
        if was:
            gc.enable()


def solve_clique_budget(salience: SalienceMap, cliques: CliqueMap,
                        config: CSAQConfig) -> Tuple[BudgetMap, Dict[str, int], float]:
    """Assign bit-widths to cliques to hit config.target_bits on average.

    Same greedy as csaq/core.py:294-361: cliques start at the lowest option,
    are ordered by salience density (stable, descending), the top
    max(1, floor(protection_floor * n)) are lifted to >= 8 bits when 8 is an
    option, then each clique in order takes upgrades while the running total
    stays within target_bits * elements. Per-clique sums are taken on the
    device in one pass per layer.

    The upgrade pass is a scan, not a loop over cliques. In order, clique i
    reaches the largest option o with (o - b_i) * e_i <= R_i, where R_i is
    the budget left (the reference's step-by-step upgrades accept exactly
    that prefix of options). A run of cliques that all reach their top
    option while the budget lasts is one cumulative sum; only the clique that
    ends a run is resolved on its own, and each such clique takes part of
    what is left. All budget arithmetic is in integers: an integer total fits
    under target_bits * elements iff it fits under its floor.
    """
    with _gc_paused():
        return _solve_clique_budget(salience, cliques, config)


def _solve_clique_budget(salience: SalienceMap, cliques: CliqueMap,
                         config: CSAQConfig) -> Tuple[BudgetMap, Dict[str, int], float]:
    options = sorted(config.bit_options)
    min_bits, max_bits = options[0], options[-1]
    layer_names: List[str] = []
    layer_counts: List[int] = []
    rows_all: List[List[int]] = []
    sal_all: List[float] = []
    elems_all: List[int] = []
    lead_all: List[int] = []
    for name, layer_cliques in cliques.items():
        s = salience[name]
        if not layer_cliques:
            continue
        if s.dtype != torch.float32:
            s = s.float()
        C, K = s.shape
        row_sal = s.sum(dim=1)
        sizes = [len(c) for c in layer_cliques]
        idx = torch.tensor([r for c in layer_cliques for r in c], dtype=torch.int64, device=s.device)
        seg = torch.repeat_interleave(torch.arange(len(layer_cliques), device=s.device),
                                      torch.tensor(sizes, device=s.device))
        rs = row_sal[idx]
        c_sal = torch.zeros(len(layer_cliques), dtype=torch.float32, device=s.device).index_add_(0, seg, rs)
        # leader: first row of maximal row salience inside the clique
        big = torch.full((len(layer_cliques),), -float("inf"), dtype=torch.float32, device=s.device)
        big = big.scatter_reduce(0, seg, rs, reduce="amax")
        is_max = rs == big[seg]
        pos_in = torch.arange(idx.numel(), device=s.device)
        first = torch.full((len(layer_cliques),), idx.numel(), dtype=torch.int64, device=s.device)
        first = first.scatter_reduce(0, seg, torch.where(is_max, pos_in, torch.full_like(pos_in, idx.numel())),
                                     reduce="amin")
        lead_all.extend(idx[first.clamp(max=idx.numel() - 1)].cpu().tolist())
        sal_all.extend(c_sal.cpu().tolist())
        layer_names.append(name)
        layer_counts.append(len(layer_cliques))
        rows_all.extend(layer_cliques)
        elems_all.extend(n * K for n in sizes)
    n = len(rows_all)
    if n == 0:
        return {}, {}, float(config.target_bits)
    elems = np.asarray(elems_all, dtype=np.int64)
    dens = np.asarray(sal_all, dtype=np.float64) / np.maximum(elems, 1)
    total = int(elems.sum())
    target_total = config.target_bits * total
    if np.isnan(dens).any():  # NaN keys: keep the reference's comparison sort
        order = np.asarray(sorted(range(n), key=lambda i: dens[i], reverse=True), dtype=np.int64)
    else:
        order = np.argsort(-dens, kind="stable")
    e = elems[order]
    b = np.full(n, min_bits, dtype=np.int64)  # bits in `order`
    current = min_bits * total
    n_protect = max(1, int(config.protection_floor * n))
    floor_target = min(8, max_bits)
    if floor_target in options and floor_target > min_bits:
        k = min(n_protect, n)
        current += (floor_target - min_bits) * int(e[:k].sum())
        b[:k] = floor_target
    # upgrades: increments to the top option and to the next option
    opts = np.asarray(options, dtype=np.int64)
    nxt = opts[np.minimum(np.searchsorted(opts, b, side="right"), len(opts) - 1)]
    inc_max = (max_bits - b) * e
    inc_min = np.where(b < max_bits, (nxt - b) * e, np.iinfo(np.int64).max)
    suffix_min = np.minimum.accumulate(inc_min[::-1])[::-1]
    final = b.copy()
    R = (math.floor(target_total) if math.isfinite(target_total) else 0) - current
    i, window = 0, _SCAN_WINDOW
    while i < n and R >= suffix_min[i]:
        j_end = min(n, i + window)
        cand = inc_min[i:j_end] <= R
        cons = np.where(cand, inc_max[i:j_end], 0)
        cs = np.cumsum(cons)
        over = np.flatnonzero(cs > R)
        q = int(over[0]) if over.size else j_end - i
        final[i:i + q][cand[:q]] = max_bits
        if q:
            R -= int(cs[q - 1])
        if not over.size:
            i = j_end
            continue
        j = i + q  # its top option no longer fits: the largest that does
        for o in options[::-1]:
            if o > b[j] and (o - int(b[j])) * int(e[j]) <= R:
                final[j] = o
                R -= (o - int(b[j])) * int(e[j])
                break
        i = j + 1
    # dict keys in first-use order along `order`, as the reference's loop inserts them
    used_bits = [(int(np.argmax(final == o)), o) for o in options if (final == o).any()]
    stats = {f"int{o}": int(e[final == o].sum()) for _, o in sorted(used_bits)}
    # per layer, its cliques in the global order (a stable sort keeps that order inside a layer,
    # so a layer's first entry is where it first appears along `order`)
    layer_of = np.repeat(np.arange(len(layer_names)), layer_counts)[order]
    grouped = np.argsort(layer_of, kind="stable")
    g_order, g_final = order[grouped].tolist(), final[grouped].tolist()
    starts = np.concatenate([[0], np.cumsum(layer_counts)]).tolist()
    first_pos = grouped[np.asarray(starts[:-1], dtype=np.int64)]
    budget: BudgetMap = {}
    for li in np.argsort(first_pos, kind="stable").tolist():
        nm, a, z = layer_names[li], starts[li], starts[li + 1]
        budget[nm] = [{"layer": nm, "rows": rows_all[oi], "salience": sal_all[oi], "elems": elems_all[oi],
                       "bits": bt, "leader": lead_all[oi]}
                      for oi, bt in zip(g_order[a:z], g_final[a:z])]
    used = int((final * e).sum())
    return budget, stats, used / max(total, 1)


# ─────────────────────────────────────────────────────────────────────────────
# Phase 3b: apply (csaq/core.py:368-418)
# ─────────────────────────────────────────────────────────────────────────────

def _protect_rows(salience_rows: torch.Tensor, floor: float) -> torch.Tensor:
    n = salience_rows.shape[0]
    n_protect = max(1, int(floor * n))
    return salience_rows.topk(n_protect).indices.sort().values


def apply_csaq(model: nn.Module, budget: BudgetMap, salience: SalienceMap, config: CSAQConfig,
               verbose: bool = True) -> Dict[str, List[int]]:
    """Replace linears by CSAQLinear and register the verify-pass rows.

    Uniform layers (group_size -1) follow csaq/core.py:368-418 exactly,
    except that the fp16 copies of the protected rows hold the original
    weights (the reference copies the dequantised rows, which makes its
    verify pass equal to its draft pass). Mixed layers (group_size > 0) give
    each row its clique's bit-width.
    """
    causal_map: Dict[str, List[int]] = {}
    mixed = config.group_size is not None and config.group_size > 0
    originals: Dict[str, torch.Tensor] = {}
    for name in budget:
        mod = _get_submodule(model, name)
        if isinstance(mod, nn.Linear) and name in salience:
            row_sal = salience[name].float().sum(dim=1)
            top = _protect_rows(row_sal, config.protection_floor)
            originals[name] = mod.weight.data[top.to(mod.weight.device)].to(torch.float16).clone()
    if mixed:
        replaced = 0
        for name, clique_list in budget.items():
            parent_name, _, child_name = name.rpartition(".")
            parent = model if not parent_name else _get_submodule(model, parent_name)
            child = getattr(parent, child_name, None) if parent is not None else None
            if not isinstance(child, nn.Linear):
                continue
            tier_rows: Dict[int, List[int]] = defaultdict(list)
            for c in clique_list:
                tier_rows[int(c["bits"])].extend(c["rows"])
            covered = set(r for rows in tier_rows.values() for r in rows)
            missing = [r for r in range(child.out_features) if r not in covered]
            if missing:
                tier_rows[max(config.bit_options)].extend(missing)
            tr = {b: torch.tensor(sorted(set(r)), dtype=torch.int64) for b, r in tier_rows.items()}
            prot = None
            if name in salience:
                prot = _protect_rows(salience[name].float().sum(dim=1), config.protection_floor)
            layer = CSAQLinear.from_tiers(child, tr, group_size=config.group_size, protected_rows=prot)
            setattr(parent, child_name, layer)
            replaced += 1
        if verbose:
            print(f"[CSAQ] Replaced {replaced} nn.Linear layers with mixed-row CSAQLinear.")
    else:
        inject_csaq_linear(model, budget, verbose=verbose)
    for mod_name in budget:
        module = _get_submodule(model, mod_name)
        if not isinstance(module, CSAQLinear) or mod_name not in salience:
            continue
        top = _protect_rows(salience[mod_name].float().sum(dim=1), config.protection_floor)
        if not mixed:
            module.set_protected_rows(top.to(module._buf_device()), originals[mod_name])
        causal_map[mod_name] = top.tolist()
    if verbose:
        n_protected = sum(len(v) for v in causal_map.values())
        print(f"[CSAQ] Protected {n_protected} rows across {len(causal_map)} layers for speculative decoding.")
    return causal_map


def quantize(model: nn.Module, calib_data, config: Optional[CSAQConfig] = None, verbose: bool = True,
             tokenizer: Any = None, seq_len: int = 128,
             calibration_domain: str = "user_provided", dp_group: Any = None) -> Tuple[nn.Module, Dict[str, Any]]:
    """Full pipeline (csaq/core.py:425-553): profile -> solve -> apply."""
    if config is None:
        config = CSAQConfig()
    t0 = time.time()
    if verbose:
        print(f"\n{'=' * 60}\n  CSAQ Quantization Pipeline (B200)\n  Target       : {config.target_bits} "
              f"bits/weight\n  Bit options  : {config.bit_options}\n  Clique thresh: "
              f"{config.clique_threshold}\n  Domain       : {calibration_domain}\n{'=' * 60}\n")
    if getattr(getattr(model, "config", None), "tie_word_embeddings", False):
        warnings.warn("[CSAQ] tie_word_embeddings=True detected. Untying for safe quantisation.",
                      stacklevel=2)
        model.config.tie_word_embeddings = False
        try:
            if model.get_input_embeddings().weight is model.get_output_embeddings().weight:
                model.get_output_embeddings().weight = nn.Parameter(
                    model.get_output_embeddings().weight.detach().clone().contiguous())
        except Exception:
            pass
    device = next(model.parameters()).device
    calib = _prepare_calib_data(calib_data, model, str(device), tokenizer=tokenizer, seq_len=seq_len)

    def _mem():
        if torch.cuda.is_available():
            torch.cuda.synchronize()
            return torch.cuda.memory_allocated() / 1024 ** 3
        import os
        import psutil
        return psutil.Process(os.getpid()).memory_info().rss / 1024 ** 3

    mem_before = _mem()
    profiler = CausalProfiler(model, config, dp_group=dp_group)
    salience, cliques = profiler.profile(calib, verbose=verbose)
    cliques_count = sum(len(v) for v in cliques.values())
    budget, tier_stats, actual_bits = solve_clique_budget(salience, cliques, config)
    if verbose:
        print(f"[CSAQ] Actual avg bits: {actual_bits:.3f} (target: {config.target_bits})")
    causal_map = apply_csaq(model, budget, salience, config, verbose=verbose)
    mem_after = _mem()
    saved = max(0, mem_before - mem_after)
    pct = max(0, (mem_before - mem_after) / max(mem_before, 1e-6)) * 100
    elapsed = time.time() - t0
    return model, {
        "tier_stats": tier_stats, "budget": budget, "causal_map": causal_map,
        "actual_bits": actual_bits, "cliques_count": cliques_count, "elapsed_s": elapsed,
        "calibration_domain": calibration_domain, "memory_before_gb": round(mem_before, 3),
        "memory_after_gb": round(mem_after, 3), "memory_saved_gb": round(saved, 3),
        "memory_saved_pct": round(pct, 1),
    }
