"""The allocation-free decode-attention entry point, csaq_decode_attention_static.

It runs the split-K decode attention with its scratch (per-chunk partial
softmax results and the per-head tickets) inside the library, a fixed 4 MiB
device array per device, instead of caller-provided `part` and `tickets`, for
callers that cannot allocate device memory. The GPU test compares it, through
the C ABI, with csaq_decode_attention on the same inputs, two calls in a row;
the CPU test checks that a call needing more scratch than the buffer holds is
refused on the host before anything is enqueued. This file is named to be
collected last, so the GPU test also runs after every other test.
"""

import ctypes
import math

import pytest
import torch

DEV = "cuda"


def test_static_attention_refuses_oversized_call():
    """Needing more than CSAQ_ATTENTION_STATIC_SCRATCH_BYTES gives CSAQ_ERR_SCRATCH (-6)."""
    from csaq import _lib
    L = _lib.lib()
    dummy = ctypes.c_void_p(256)
    B, S, Hq, Hkv, D, Lmax = 1, 1, 32, 8, 128, 100_000
    assert L.csaq_attention_workspace_floats(B, S, Hq, Hkv, D, Lmax) * 4 > (4 << 20)
    assert L.csaq_decode_attention_static(dummy, dummy, dummy, dummy, B, S, Hq, Hkv, D, Lmax, 0.1, dummy, 2,
                                          None) == -6
    assert b"scratch" in L.csaq_status_string(-6)
    assert L.csaq_decode_attention_static(None, dummy, dummy, dummy, B, S, Hq, Hkv, D, 64, 0.1, dummy, 2,
                                          None) == -1


@pytest.mark.gpu
@pytest.mark.parametrize("B,S,pos", [(1, 1, (517,)), (2, 5, (300, 777))])
def test_static_attention_matches_attention(B, S, pos):
    from csaq._lib import check, lib, stream_of
    Hq, Hkv, D, Lmax = 32, 8, 128, 800
    g = torch.Generator().manual_seed(7)
    q = torch.randn(B * S, Hq * D, generator=g).to(torch.bfloat16).to(DEV)
    kc = torch.randn(B, Hkv, Lmax, D, generator=g).to(torch.bfloat16).to(DEV)
    vc = torch.randn(B, Hkv, Lmax, D, generator=g).to(torch.bfloat16).to(DEV)
    pos0 = torch.tensor(pos, dtype=torch.int32, device=DEV)
    scale = 1.0 / math.sqrt(D)
    st = stream_of(q)
    floats = lib().csaq_attention_workspace_floats(B, S, Hq, Hkv, D, Lmax)
    part = torch.zeros(floats, dtype=torch.float32, device=DEV)
    tickets = torch.zeros(B * Hkv, dtype=torch.int32, device=DEV)
    ref = torch.empty(B * S, Hq * D, dtype=torch.bfloat16, device=DEV)
    check(lib().csaq_decode_attention(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), pos0.data_ptr(), B, S, Hq, Hkv,
                                      D, Lmax, scale, part.data_ptr(), tickets.data_ptr(), ref.data_ptr(), 2, st),
          "attention")
    for _ in range(2):  # two calls in a row: the first leaves the tickets ready for the second
        out = torch.full((B * S, Hq * D), float("nan"), dtype=torch.bfloat16, device=DEV)
        check(lib().csaq_decode_attention_static(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), pos0.data_ptr(), B, S,
                                                 Hq, Hkv, D, Lmax, scale, out.data_ptr(), 2, st), "attention_static")
        torch.cuda.synchronize()
        r, o = ref.float(), out.float()
        assert torch.isfinite(o).all()
        rel = float((o - r).norm() / r.norm())
        assert rel <= 1e-2 and float((o - r).abs().max() / r.abs().max()) <= 1e-2, rel
