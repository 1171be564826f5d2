"""The allocation-free GEMV entry point, csaq_qgemv_static.

It runs the tensor-core GEMV with scratch that lives inside the library (a
fixed 1 MiB device array per device) instead of a caller workspace, for callers
that cannot allocate device memory. The GPU test compares it, through the C
ABI, with csaq_qgemv on a mixed-precision layer, two calls in a row; the CPU
test checks that a launch needing more scratch than the buffer holds is
refused on the host before anything is enqueued. This file is named to be
collected last, so the GPU test also runs after every other test.
"""

import ctypes

import pytest
import torch

from _tol import assert_linear_close

DEV = "cuda"


def _layer(n, k, seed):
    from csaq import _synthetic as syn
    from csaq.kernels import CSAQLinear
    case = syn.mixed_linear(n=n, k=k, m=1, seed=seed, dtype=torch.bfloat16, bits=(16, 8, 4),
                            fracs=(0.1, 0.2))
    lin = torch.nn.Linear(k, n, bias=True, dtype=torch.bfloat16).to(DEV)
    lin.weight.data = case.W.to(DEV)
    lin.bias.data = (torch.randn(n, generator=torch.Generator().manual_seed(seed)) * 0.1).to(
        torch.bfloat16).to(DEV)
    return CSAQLinear.from_tiers(lin, case.tier_rows, group_size=128)


def test_static_scratch_refuses_oversized_launch():
    """Needing more than CSAQ_QGEMV_STATIC_SCRATCH_BYTES gives CSAQ_ERR_SCRATCH (-6)."""
    from csaq import _lib
    L = _lib.lib()
    dummy = ctypes.c_void_p(256)
    rows = ctypes.c_int32(0)
    # 2**21 fp16 rows: about 500 KB of unit tickets on top of the per-CTA sums
    t = _lib.CsaqTier(bits=16, n_rows=1 << 21, group_size=128, n_groups=1, row_bytes=256,
                      codes=dummy, out_rows=ctypes.addressof(rows), blocks=dummy, y=dummy, ldy=1 << 21)
    arr = _lib.tier_array([t])
    assert L.csaq_qgemv_workspace_bytes(arr, 1, 128) > (1 << 20)
    assert L.csaq_qgemv_static(arr, 1, 128, dummy, 2, 1, 128, None) == -6
    assert b"scratch" in L.csaq_status_string(-6)
    assert L.csaq_qgemv_static(arr, 0, 128, dummy, 2, 1, 128, None) == -1


@pytest.mark.gpu
@pytest.mark.parametrize("shape", [(4096, 4096), (1024, 14336)])
def test_static_scratch_gemv_matches_workspace_gemv(shape):
    from csaq import _lib
    from csaq._lib import check, dtype_code, lib, stream_of
    n, k = shape
    layer = _layer(n, k, seed=11)
    for m in (1, 5):
        x = torch.randn(m, k, generator=torch.Generator().manual_seed(m)).to(torch.bfloat16).to(DEV)
        y_ref = torch.empty(m, n, dtype=torch.bfloat16, device=DEV)
        _lib.qgemv(layer.gemv_descriptors(y_ref), k, x, m, _lib.Workspace())
        for _ in range(2):  # two calls in a row: the first leaves the scratch ready for the second
            y = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=DEV)
            d = layer.gemv_descriptors(y)
            check(lib().csaq_qgemv_static(_lib.tier_array(d), len(d), k, x.data_ptr(), dtype_code(x.dtype),
                                          m, x.stride(0), stream_of(x)), "qgemv_static")
            torch.cuda.synchronize()
            assert_linear_close(y.float().cpu().numpy(), y_ref.float().cpu().numpy(),
                                what=f"static scratch {shape} m={m}")
