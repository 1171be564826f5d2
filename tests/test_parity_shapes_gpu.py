"""Parity of the quantised linear at the workloads' own layer shapes.

* The tcgen05 dequantise-GEMM (prefill) at the Llama-3-70B-shaped layer's
  linears with 8/4/2-bit tiers: K = 8192 (q, k, gate) and K = 28672 (down)
  at 8192 tokens, and the tensor-parallel-8 slices (gate rows / 8, down
  columns / 8) at 32768 tokens.
* The decode GEMV at the Llama-3-8B-shaped down projection (14336 -> 4096,
  16/8/4-bit tiers) at M = 1 and 5, the fused gate/up launch (28672 rows),
  and the 16-bit 128256 x 4096 lm_head.

Outputs are compared with the oracle's dequantise-then-matmul
(csaq/kernels.py:450-475) within the 1e-2 relative bound of _tol.py. The
largest shapes are compared on a seeded sample of tokens and rows: the
oracle quantises only the sampled rows, which gives the same codes, scales
and zero points as quantising the whole tier because quantisation is per
row (csaq/kernels.py:128-158).
"""

import numpy as np
import pytest
import torch

from _tol import assert_linear_close
from oracle import csaq_oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _weights(n, k, seed, dtype=torch.bfloat16):
    """W (n, k) ~ N(0, 0.02^2) with a seeded 1 % of rows x10, drawn on the device."""
    g = torch.Generator(device=DEV).manual_seed(seed)
    W = torch.randn(n, k, generator=g, device=DEV) * 0.02
    W[torch.randperm(n, generator=g, device=DEV)[:max(1, n // 100)]] *= 10.0
    return W.to(dtype)


def _tiers(n, mix, seed):
    """Rows split at random into tiers: mix = ((bits, fraction), ...), the last takes the rest."""
    perm = torch.randperm(n, generator=torch.Generator().manual_seed(seed))
    out, start = {}, 0
    for i, (b, f) in enumerate(mix):
        cnt = n - start if i == len(mix) - 1 else int(f * n)
        out[b] = torch.sort(perm[start:start + cnt]).values
        start += cnt
    return out


def _layer(W, tier_rows):
    from csaq.kernels import CSAQLinear
    n, k = W.shape
    lin = torch.nn.Linear(k, n, bias=False, device="meta")
    lin.weight = torch.nn.Parameter(W, requires_grad=False)
    return CSAQLinear.from_tiers(lin, tier_rows, group_size=128)


def _oracle_rows(W, tier_rows, rows):
    """Dequantised oracle weights (len(rows), K) of the sampled rows."""
    Wh = W[rows.to(DEV)].float().cpu().numpy()
    out = np.zeros(Wh.shape, np.float32)
    for b, tr in tier_rows.items():
        sel = np.isin(rows.numpy(), tr.numpy())
        if not sel.any():
            continue
        qw = O.quantize_per_channel(Wh[sel], b, 128)
        out[sel] = qw.dequantize() if b == 16 else O.dequantize_grouped(
            qw.qdata, qw.scales, qw.zero_points, b, qw.rows, qw.cols, qw.group_size)
    return out


def _sample(n, count, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.sort(torch.randperm(n, generator=g)[:count]).values


MIX_70B = ((8, 0.10), (4, 0.25), (2, 0.65))   # about 3.1 bits, the {2, 4, 8} mix at average 3.0
MIX_8B = ((16, 0.10), (8, 0.20), (4, 0.70))   # the {4, 8, 16} mix with the 10 % protection floor


@pytest.mark.parametrize("name,n,k,m", [
    ("q_proj", 8192, 8192, 8192),
    ("k_proj", 1024, 8192, 8192),
    ("gate_proj", 28672, 8192, 8192),
    ("down_proj", 8192, 28672, 8192),
    ("gate_proj/8", 3584, 8192, 32768),
    ("down_proj/8", 8192, 3584, 32768),
])
def test_qgemm_llama70b_shapes(name, n, k, m):
    """Prefill GEMM (CSAQLinear.forward at m tokens) on sampled tokens and rows."""
    seed = n + k + m
    W = _weights(n, k, seed)
    tiers = _tiers(n, MIX_70B, seed)
    layer = _layer(W, tiers)
    x = (torch.randn(m, k, generator=torch.Generator(device=DEV).manual_seed(seed + 1), device=DEV)
         .to(torch.bfloat16))
    y = layer(x)
    assert y.shape == (m, n)
    toks = _sample(m, 48, seed + 2)
    rows = torch.cat([_sample(n, 512, seed + 3), torch.tensor([0, n - 1])]).unique()
    Wref = _oracle_rows(W, tiers, rows)
    xs = x[toks.to(DEV)].float().cpu().numpy()
    got = y[toks.to(DEV)][:, rows.to(DEV)].float().cpu().numpy()
    assert_linear_close(got, O.linear_ref(xs, Wref), what=f"{name} {m}x{n}x{k}")
    # within the bf16 output's own rounding of the reference's numerics (weights rounded to x.dtype)
    Wx = torch.from_numpy(Wref).to(torch.bfloat16).float().numpy()
    assert_linear_close(got, O.linear_ref(xs, Wx), rtol=4e-3, what=f"{name} x-dtype weights")
    assert torch.isfinite(y).all()


@pytest.mark.parametrize("m", [1, 5])
def test_qgemv_llama8b_down_proj(m):
    """Decode GEMV, 14336 -> 4096 with 16/8/4-bit tiers, every row against the oracle."""
    n, k = 4096, 14336
    W = _weights(n, k, 21)
    tiers = _tiers(n, MIX_8B, 21)
    layer = _layer(W, tiers)
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(m)).to(torch.bfloat16)
    y = layer(x.to(DEV)).float().cpu().numpy()
    Wref = O.mixed_weight(W.float().cpu().numpy(), {b: r.numpy() for b, r in tiers.items()}, 128)
    assert_linear_close(y, O.linear_ref(x.float().numpy(), Wref), what=f"down m={m}")


@pytest.mark.parametrize("m", [1, 5])
def test_qgemv_llama8b_gate_up_fused(m):
    """The runtime's fused gate/up launch: 28672 rows over K = 4096, sampled rows."""
    n, k = 28672, 4096
    W = _weights(n, k, 22)
    tiers = _tiers(n, MIX_8B, 22)
    layer = _layer(W, tiers)
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(10 + m)).to(torch.bfloat16)
    y = layer(x.to(DEV))
    rows = _sample(n, 2048, 23)
    Wref = _oracle_rows(W, tiers, rows)
    got = y[:, rows.to(DEV)].float().cpu().numpy()
    assert_linear_close(got, O.linear_ref(x.float().numpy(), Wref), what=f"gate/up m={m}")


@pytest.mark.parametrize("m", [1, 5])
def test_qgemv_llama8b_lm_head_16bit(m):
    """The 16-bit lm_head (128256 x 4096): every row against the fp16-cast weights."""
    n, k = 128256, 4096
    W = _weights(n, k, 24)
    layer = _layer(W, {16: torch.arange(n)})
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(20 + m)).to(torch.bfloat16)
    y = layer(x.to(DEV)).float().cpu().numpy()
    ref = np.empty((m, n), np.float32)
    xs = x.float().numpy()
    step = 16384
    for r0 in range(0, n, step):  # the oracle's 16-bit rows: the fp16 cast (csaq/kernels.py:94-107)
        W16 = O.quantize_per_channel(W[r0:r0 + step].float().cpu().numpy(), 16).dequantize()
        ref[:, r0:r0 + step] = O.linear_ref(xs, W16)
    assert_linear_close(y, ref, what=f"lm_head m={m}")
