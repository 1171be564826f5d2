"""Seeded synthetic workloads for the quantised hot path.

No checkpoints or datasets are available offline, so every workload is drawn
from ``torch.Generator().manual_seed(seed)`` on the host in fp32 and then cast.
The draw order below is part of the definition: the golden fixtures, the GPU
parity tests and ``bench.py`` all regenerate the same tensors from it.

Workloads:

* ``mixed_linear``: a single mixed-precision linear. W (N, K) ~ N(0, 0.02^2)
  with a seeded 1 % of rows scaled x10 as outliers; G ~ N(0, 1e-3^2); row
  salience = sum_k |G*W|; rows ranked by descending salience get 16-bit
  (top 10 %), 8-bit (next 20 %) and 4-bit (rest). X ~ N(0, 1).
  At N = K = 4096 this is the 4096x4096 single-linear workload.
* ``calibration``: MLP pre-activations (S*T, C) fp16 built as
  sqrt(rho)*z_block + sqrt(1-rho)*eps with channel blocks of 32 sharing z,
  rho = 0.9; the co-activation mask is act > 0.5. Salience inputs are
  W (C, K) ~ N(0, 0.02^2) and per-sample grads ~ N(0, 1e-3^2).
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import List

import torch


@dataclass
class MixedLinearCase:
    W: torch.Tensor            # (N, K) fp16 (or the requested dtype)
    salience: torch.Tensor     # (N,) fp32 row salience
    order: torch.Tensor        # (N,) int64, rows by descending salience
    tier_rows: dict            # bits -> sorted int64 row indices
    X: torch.Tensor            # (M, K) activations


def tier_split(n_rows: int, fracs=(0.1, 0.2)) -> List[int]:
    """Row counts per tier: floor(f * N) for each fraction, the rest last
    (default 16/8/4: floor(0.1N), floor(0.2N), rest)."""
    counts = [int(math.floor(f * n_rows)) for f in fracs]
    return counts + [n_rows - sum(counts)]


def mixed_linear(n: int = 4096, k: int = 4096, m: int = 1, seed: int = 0,
                 dtype: torch.dtype = torch.float16, outlier_frac: float = 0.01,
                 bits=(16, 8, 4), fracs=(0.1, 0.2)) -> MixedLinearCase:
    """`bits` lists the tiers from most to least salient; `fracs` gives the
    fraction of rows of every tier but the last."""
    if len(bits) != len(fracs) + 1 or len(set(bits)) != len(bits):
        raise ValueError("need len(bits) == len(fracs) + 1 and distinct bit-widths")
    gen = torch.Generator().manual_seed(seed)
    W = torch.randn(n, k, generator=gen) * 0.02
    n_out = max(1, int(outlier_frac * n))
    out_rows = torch.randperm(n, generator=gen)[:n_out]
    W[out_rows] *= 10.0
    W = W.to(dtype)
    G = (torch.randn(n, k, generator=gen) * 1e-3).to(dtype)
    sal = (G.float() * W.float()).abs().sum(dim=1)
    order = torch.argsort(sal, descending=True, stable=True)
    counts = tier_split(n, fracs)
    tier_rows = {}
    start = 0
    for b, c in zip(bits, counts):
        tier_rows[b] = torch.sort(order[start:start + c]).values
        start += c
    X = torch.randn(m, k, generator=gen).to(dtype)
    return MixedLinearCase(W=W, salience=sal, order=order, tier_rows=tier_rows, X=X)


def activations(n_tokens: int, channels: int, seed: int = 0, rho: float = 0.9,
                block: int = 32) -> torch.Tensor:
    """Correlated pre-activations (n_tokens, channels) fp16; blocks of `block`
    channels share one latent factor with correlation rho."""
    gen = torch.Generator().manual_seed(seed)
    n_blocks = (channels + block - 1) // block
    z = torch.randn(n_tokens, n_blocks, generator=gen)
    eps = torch.randn(n_tokens, channels, generator=gen)
    zc = z.repeat_interleave(block, dim=1)[:, :channels]
    act = math.sqrt(rho) * zc + math.sqrt(1.0 - rho) * eps
    return act.to(torch.float16)


def salience_inputs(channels: int, k: int, n_samples: int, seed: int = 0,
                    dtype: torch.dtype = torch.float16):
    """W (channels, k) ~ N(0, 0.02^2) and a list of per-sample grads ~ N(0, 1e-3^2)."""
    gen = torch.Generator().manual_seed(seed)
    W = (torch.randn(channels, k, generator=gen) * 0.02).to(dtype)
    grads = [(torch.randn(channels, k, generator=gen) * 1e-3).to(dtype)
             for _ in range(n_samples)]
    return W, grads


# ── decoder-shaped models (random init, no checkpoint needed) ────────────────
DECODERS = {
    # name: (architecture, hidden, intermediate, layers, heads, kv heads, vocab)
    "qwen1.5-0.5b": ("qwen2", 1024, 2816, 24, 16, 16, 151936),
    "llama3-8b": ("llama", 4096, 14336, 32, 32, 8, 128256),
    "llama3-70b": ("llama", 8192, 28672, 80, 64, 8, 128256),
    "tiny-llama": ("llama", 512, 1536, 2, 4, 2, 2048),
    "tiny-qwen2": ("qwen2", 512, 1408, 2, 4, 4, 2048),
    "tiny-qwen2-d64": ("qwen2", 256, 768, 2, 4, 4, 2048),  # 64-wide heads, like Qwen1.5-0.5B
}


def decoder_config(name: str, n_layers: int = None):
    """HF config of a decoder shape (head_dim hidden/heads: 64 or 128; default rope)."""
    from transformers import LlamaConfig, Qwen2Config
    arch, h, inter, layers, heads, kv, vocab = DECODERS[name]
    kw = dict(hidden_size=h, intermediate_size=inter, num_hidden_layers=n_layers or layers,
              num_attention_heads=heads, num_key_value_heads=kv, vocab_size=vocab,
              max_position_embeddings=4096, initializer_range=0.02, tie_word_embeddings=False)
    return LlamaConfig(**kw) if arch == "llama" else Qwen2Config(**kw)


def build_decoder(name: str, device="cuda", dtype: torch.dtype = torch.bfloat16, seed: int = 0,
                  n_layers: int = None):
    """Random-init decoder: every weight ~ N(0, 0.02^2), norms = 1, biases 0."""
    from transformers import AutoModelForCausalLM
    cfg = decoder_config(name, n_layers)
    torch.manual_seed(seed)
    with torch.device(device):
        model = AutoModelForCausalLM.from_config(cfg, dtype=dtype)
    gen = torch.Generator(device=device).manual_seed(seed)
    with torch.no_grad():
        for n, p in model.named_parameters():
            if p.dim() >= 2:
                p.copy_(torch.randn(p.shape, generator=gen, device=device, dtype=torch.float32) * 0.02)
            elif "norm" in n:
                p.fill_(1.0)
            else:
                p.zero_()
    model.eval()
    return model


def synthetic_salience(model, seed: int = 0):
    """Row salience sum_k |G*W| with G ~ N(0, 1e-3^2) for every quantisable
    linear, returned as (C, K) expanded views of the per-row value / K (the
    solver and apply_csaq only reduce over K)."""
    import torch.nn as nn
    out = {}
    gen = torch.Generator(device=next(model.parameters()).device).manual_seed(seed)
    skip = ("lm_head", "embed_tokens")
    for name, m in model.named_modules():
        if not isinstance(m, nn.Linear) or any(s in name for s in skip):
            continue
        W = m.weight.data
        C, K = W.shape
        rs = torch.empty(C, dtype=torch.float32, device=W.device)
        step = max(1, (1 << 26) // K)
        for r0 in range(0, C, step):
            w = W[r0:r0 + step].float()
            g = torch.randn(w.shape, generator=gen, device=W.device) * 1e-3
            rs[r0:r0 + step] = (g * w).abs().sum(dim=1)
        out[name] = (rs / K)[:, None].expand(C, K)
    return out
