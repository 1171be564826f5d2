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
