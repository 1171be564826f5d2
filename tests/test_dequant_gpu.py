"""csaq_dequant (the reference's _dequantize, csaq/kernels.py:603-619): the
vectorised path (eight columns per thread) gives the bits of the
one-element-per-thread path and of torch's fp32 (q - zp) * s on the
unpacked codes. The scalar path is taken by handing the same call an output
that is not 16-byte aligned; ragged column counts take it by themselves."""

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _dequant(q, s, z, bits, rows, cols, gs, nan, out_dtype, offset):
    from csaq._lib import check, dtype_code, lib
    buf = torch.zeros(rows * cols + 16, dtype=out_dtype, device=DEV)
    out = buf[offset: offset + rows * cols]
    st = torch.cuda.current_stream().cuda_stream
    check(lib().csaq_dequant(q.data_ptr(), s.data_ptr() if s is not None else None,
                             z.data_ptr() if z is not None else None, bits, rows, cols, gs, nan,
                             dtype_code(out_dtype), out.data_ptr(), st), "dequant")
    torch.cuda.synchronize()
    return out.view(rows, cols).clone()


def _bits_equal(a, b):
    it = torch.int32 if a.dtype == torch.float32 else torch.int16
    return torch.equal(a.view(it), b.view(it))


def _torch_ref(qw, rows, cols):
    """fp32 (q - zp) * s from the unpacked codes, with torch's elementwise ops."""
    from csaq.kernels import _unpack
    if qw.bits == 16:
        return qw.qdata.view(torch.float16).reshape(rows, cols).float()
    q = _unpack(qw.qdata, qw.bits, rows, cols).to(DEV).float()
    gs = qw.group_size if 0 < qw.group_size < cols else cols
    g = torch.arange(cols, device=DEV) // gs
    s = qw.scales.to(DEV).reshape(rows, -1)[:, g]
    z = qw.zero_points.to(DEV).reshape(rows, -1)[:, g].float()
    return (q - z) * s


@pytest.mark.parametrize("bits", [2, 4, 8, 16])
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("gs", [128, -1, 8])
def test_vector_path_matches_scalar_path(bits, out_dtype, gs):
    from csaq.kernels import quantize_per_channel
    rows, cols = 37, 1024
    W = (torch.randn(rows, cols, generator=torch.Generator().manual_seed(bits)) * 0.05).to(DEV)
    W[3, 5] = 40.0  # an outlier
    qw = quantize_per_channel(W, bits, gs)
    q = qw.qdata.contiguous().to(DEV)
    s = None if bits == 16 else qw.scales.contiguous().to(DEV)
    z = None if bits == 16 else qw.zero_points.to(torch.int32).contiguous().to(DEV)
    gsz = qw.group_size if bits != 16 else -1
    ref = _torch_ref(qw, rows, cols).to(out_dtype)
    for nan in (0, 1):
        a = _dequant(q, s, z, bits, rows, cols, gsz, nan, out_dtype, 0)
        b = _dequant(q, s, z, bits, rows, cols, gsz, nan, out_dtype, 1)  # misaligned output: the scalar path
        assert _bits_equal(a, b), (bits, out_dtype, gs, nan)
        assert _bits_equal(a, ref), (bits, out_dtype, gs, nan)


def test_ragged_columns_use_the_scalar_path():
    from csaq.kernels import quantize_per_channel
    W = torch.randn(9, 1003, generator=torch.Generator().manual_seed(1)).to(DEV)
    for bits in (2, 4, 8):
        qw = quantize_per_channel(W, bits, 128)
        a = _dequant(qw.qdata.contiguous().to(DEV), qw.scales.contiguous().to(DEV),
                     qw.zero_points.to(torch.int32).contiguous().to(DEV), bits, 9, 1003, qw.group_size, 1,
                     torch.float32, 0)
        assert _bits_equal(a, _torch_ref(qw, 9, 1003)), bits
