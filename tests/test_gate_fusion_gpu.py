"""The SiLU gate fused into the GEMVs (csaq_qgemv_ext) against the separate
launches it replaces in the decode runtime: the gate/up GEMV, csaq_silu_mul
(h = dtype(silu(g)) * u, HF LlamaMLP) and the down GEMV. The fused path must
give the same bits: the gate tiers store dtype(silu(y)), the down GEMV
builds its records from dtype(g' * u).
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _layer(n, k, seed, dtype):
    from csaq import _synthetic as syn
    from csaq.kernels import CSAQLinear
    case = syn.mixed_linear(n=n, k=k, m=1, seed=seed, dtype=dtype, bits=(16, 8, 4), fracs=(0.1, 0.2))
    lin = torch.nn.Linear(k, n, bias=False, dtype=dtype).to(DEV)
    lin.weight.data = case.W.to(DEV)
    return CSAQLinear.from_tiers(lin, case.tier_rows, group_size=128)


def _ext(descs, K, x, M, silu_tiers, x_mul):
    from csaq import _lib
    from csaq._lib import check, dtype_code, lib, stream_of
    ext = _lib.CsaqGemvExt(silu_tiers, x_mul.data_ptr() if x_mul is not None else None)
    return check(lib().csaq_qgemv_ext(_lib.tier_array(descs), len(descs), K, x.data_ptr(), dtype_code(x.dtype), M,
                                      x.stride(0), ctypes.byref(ext), stream_of(x)), "qgemv_ext")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("H,I,M", [(512, 1024, 1), (512, 1024, 5), (512, 1024, 16), (256, 14336, 5),
                                   (256, 14336, 16)])
def test_fused_gate_matches_separate_launches(dtype, H, I, M):
    from csaq import _lib
    from csaq._lib import check, dtype_code, lib, stream_of
    gate, up, down = _layer(I, H, 1, dtype), _layer(I, H, 2, dtype), _layer(H, I, 3, dtype)
    g = torch.Generator().manual_seed(M)
    x = torch.randn(M, H, generator=g).to(dtype).to(DEV)
    r = (torch.randn(M, H, generator=g) * 0.5).to(dtype).to(DEV)

    # separate launches, as the runtime ran them
    gu = torch.zeros(M, 2 * I, dtype=dtype, device=DEV)
    _lib.qgemv(gate.gemv_descriptors(gu[:, :I]) + up.gemv_descriptors(gu[:, I:]), H, x, M)
    h = torch.zeros(M, I, dtype=dtype, device=DEV)
    st = stream_of(x)
    check(lib().csaq_silu_mul(gu.data_ptr(), gu.stride(0), gu[:, I:].data_ptr(), gu.stride(0), h.data_ptr(), I, M,
                              I, dtype_code(dtype), st), "silu_mul")
    ones = torch.ones(M, I, dtype=dtype, device=DEV)
    g_act = torch.zeros(M, I, dtype=dtype, device=DEV)  # dtype(silu(g)) * 1 = dtype(silu(g))
    check(lib().csaq_silu_mul(gu.data_ptr(), gu.stride(0), ones.data_ptr(), I, g_act.data_ptr(), I, M, I,
                              dtype_code(dtype), st), "silu_mul")
    y_ref = r.clone()
    _lib.qgemv(down.gemv_descriptors(y_ref, residual=y_ref), I, h, M)

    # fused
    gu2 = torch.zeros(M, 2 * I, dtype=dtype, device=DEV)
    d_gate = gate.gemv_descriptors(gu2[:, :I])
    _ext(d_gate + up.gemv_descriptors(gu2[:, I:]), H, x, M, (1 << len(d_gate)) - 1, None)
    y = r.clone()
    _ext(down.gemv_descriptors(y, residual=y), I, gu2, M, 0, gu2[:, I:])
    torch.cuda.synchronize()

    assert torch.equal(gu2[:, I:], gu[:, I:]), "up half"
    assert torch.equal(gu2[:, :I], g_act), "gate half: dtype(silu(y))"
    assert torch.equal(y, y_ref), "down output"
    assert torch.isfinite(y.float()).all()


def test_fused_gate_rejects_what_it_cannot_serve():
    """F32 input and tier bits beyond n_tiers are refused before any launch."""
    from csaq import _lib
    from csaq._lib import dtype_code, lib, stream_of
    up = _layer(256, 256, 4, torch.bfloat16)
    x = torch.randn(2, 256).to(DEV)
    y = torch.zeros(2, 256, dtype=torch.bfloat16, device=DEV)
    d = up.gemv_descriptors(y)
    ext = _lib.CsaqGemvExt(0, None)
    rc = lib().csaq_qgemv_ext(_lib.tier_array(d), len(d), 256, x.data_ptr(), dtype_code(x.dtype), 2, 256,
                              ctypes.byref(ext), stream_of(x))
    assert rc == -5  # CSAQ_ERR_UNSUPPORTED
    ext = _lib.CsaqGemvExt(1 << len(d), None)
    xb = x.to(torch.bfloat16)
    rc = lib().csaq_qgemv_ext(_lib.tier_array(d), len(d), 256, xb.data_ptr(), dtype_code(xb.dtype), 2, 256,
                              ctypes.byref(ext), stream_of(xb))
    assert rc == -1  # CSAQ_ERR_ARG

