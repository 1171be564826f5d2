"""The allocation-free decode-attention entry point, csaq_decode_attention_static.

It runs the split-K decode attention with its scratch (per-chunk partial
softmax results and the per-head tickets) inside the library, a fixed 4 MiB
device array per device, instead of caller-provided `part` and `tickets`, for
callers that cannot allocate device memory. The GPU tests call it through the
C ABI with shapes that change from call to call (large, small, large again:
a speculative decoder alternates one-token draft steps with K+1-token verify
steps) and compare every output with an fp32 PyTorch attention and with
csaq_decode_attention. The CPU test checks that a call needing more scratch
than the buffer holds is refused on the host before anything is enqueued.
This file is named to be collected last, so the GPU tests also run after
every other test.
"""

import ctypes
import math

import pytest
import torch

DEV = "cuda"
MAX_HEADS = 1024  # CSAQ_ATTENTION_STATIC_MAX_HEADS


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
    # more (sequence, KV head) pairs than the fixed ticket region holds
    assert L.csaq_decode_attention_static(dummy, dummy, dummy, dummy, MAX_HEADS // 8 + 1, 1, 8, 8, 64, 64, 0.1,
                                          dummy, 2, None) == -6
    assert L.csaq_decode_attention_static(None, dummy, dummy, dummy, B, S, Hq, Hkv, D, 64, 0.1, dummy, 2,
                                          None) == -1


def _attention_fp32(q, kc, vc, pos, B, S, Hq, Hkv, D, scale):
    """softmax(q k^T * scale) v in fp32 with GQA; token (b, s) sees keys 0..pos[b]+s."""
    G = Hq // Hkv
    qf = q.float().view(B, S, Hq, D)
    out = torch.empty(B, S, Hq, D, dtype=torch.float32, device=q.device)
    for b in range(B):
        for s in range(S):
            n = pos[b] + s + 1
            k = kc[b, :, :n].float().repeat_interleave(G, dim=0)  # (Hq, n, D)
            v = vc[b, :, :n].float().repeat_interleave(G, dim=0)
            w = torch.softmax(torch.einsum("hd,hnd->hn", qf[b, s], k) * scale, dim=-1)
            out[b, s] = torch.einsum("hn,hnd->hd", w, v)
    return out.view(B * S, Hq * D)


def _case(B, S, pos, Lmax, seed, Hq=32, Hkv=8, D=128):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B * S, Hq * D, generator=g).to(torch.bfloat16).to(DEV)
    kc = torch.randn(B, Hkv, Lmax, D, generator=g).to(torch.bfloat16).to(DEV)
    vc = torch.randn(B, Hkv, Lmax, D, generator=g).to(torch.bfloat16).to(DEV)
    return dict(B=B, S=S, pos=pos, Lmax=Lmax, Hq=Hq, Hkv=Hkv, D=D, q=q, kc=kc, vc=vc,
                pos0=torch.tensor(pos, dtype=torch.int32, device=DEV))


def _run_static(c, scale, st):
    from csaq._lib import check, lib
    out = torch.full((c["B"] * c["S"], c["Hq"] * c["D"]), float("nan"), dtype=torch.bfloat16, device=DEV)
    check(lib().csaq_decode_attention_static(c["q"].data_ptr(), c["kc"].data_ptr(), c["vc"].data_ptr(),
                                             c["pos0"].data_ptr(), c["B"], c["S"], c["Hq"], c["Hkv"], c["D"],
                                             c["Lmax"], scale, out.data_ptr(), 2, st), "attention_static")
    return out


def _run_allocating(c, scale, st):
    from csaq._lib import check, lib
    B, S, Hq, Hkv, D, Lmax = c["B"], c["S"], c["Hq"], c["Hkv"], c["D"], c["Lmax"]
    floats = lib().csaq_attention_workspace_floats(B, S, Hq, Hkv, D, Lmax)
    part = torch.zeros(floats, dtype=torch.float32, device=DEV)
    tickets = torch.zeros(B * Hkv, dtype=torch.int32, device=DEV)
    out = torch.empty(B * S, Hq * D, dtype=torch.bfloat16, device=DEV)
    check(lib().csaq_decode_attention(c["q"].data_ptr(), c["kc"].data_ptr(), c["vc"].data_ptr(),
                                      c["pos0"].data_ptr(), B, S, Hq, Hkv, D, Lmax, scale, part.data_ptr(),
                                      tickets.data_ptr(), out.data_ptr(), 2, st), "attention")
    return out


@pytest.mark.gpu
def test_static_attention_changing_shapes():
    """Large, small, large again: each output matches fp32 attention and csaq_decode_attention (1e-2)."""
    from csaq._lib import stream_of
    large = _case(2, 5, (300, 777), 800, seed=7)
    small = _case(1, 1, (517,), 600, seed=8)
    wide = _case(4, 2, (10, 1000, 64, 333), 1100, seed=9, Hq=16, Hkv=4, D=64)
    for c in (large, small, large, wide, small):
        scale = 1.0 / math.sqrt(c["D"])
        st = stream_of(c["q"])
        out = _run_static(c, scale, st)
        ref_kernel = _run_allocating(c, scale, st)
        torch.cuda.synchronize()
        ref = _attention_fp32(c["q"], c["kc"], c["vc"], c["pos"], c["B"], c["S"], c["Hq"], c["Hkv"], c["D"], scale)
        o = out.float()
        assert torch.isfinite(o).all(), "static attention left output rows unwritten"
        for r in (ref, ref_kernel.float()):
            rel = float((o - r).norm() / r.norm())
            mx = float((o - r).abs().max() / r.abs().max())
            assert rel <= 1e-2 and mx <= 1e-2, (c["B"], c["S"], rel, mx)


@pytest.mark.gpu
@pytest.mark.parametrize("B,S,pos", [(1, 1, (517,)), (2, 5, (300, 777))])
def test_static_attention_matches_attention(B, S, pos):
    """Two calls in a row of one shape agree with csaq_decode_attention within 1e-2."""
    from csaq._lib import stream_of
    c = _case(B, S, pos, 800, seed=7)
    scale = 1.0 / math.sqrt(c["D"])
    st = stream_of(c["q"])
    ref = _run_allocating(c, scale, st).float()
    for _ in range(2):
        o = _run_static(c, scale, st).float()
        torch.cuda.synchronize()
        assert torch.isfinite(o).all()
        rel = float((o - ref).norm() / ref.norm())
        assert rel <= 1e-2 and float((o - ref).abs().max() / ref.abs().max()) <= 1e-2, rel
