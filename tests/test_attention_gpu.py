"""Decode attention with the rotary embedding fused in (csaq_decode_attention_rope).

One launch rotates the step's queries and new keys, writes the new keys and
values to the cache and attends; it must equal csaq_rope_kv followed by
csaq_decode_attention bit for bit (output and both caches), including new
positions that straddle a 64-key chunk boundary and 64-wide heads, and match
an fp32 PyTorch rotary attention within 1e-2.
"""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _tables(Lmax, D, dtype):
    inv = 1.0 / (10000.0 ** (torch.arange(0, D, 2).float() / D))
    f = torch.arange(Lmax).float()[:, None] * inv[None, :]
    emb = torch.cat([f, f], dim=-1)
    return (emb.cos().to(dtype).float().contiguous().to(DEV), emb.sin().to(dtype).float().contiguous().to(DEV))


def _rope_ref(x, cos, sin):
    half = x.shape[-1] // 2
    rot = torch.cat([-x[..., half:], x[..., :half]], dim=-1)
    return x * cos + rot * sin


@pytest.mark.parametrize("B,S,Hq,Hkv,D,pos", [
    (1, 1, 32, 8, 128, (517,)),
    (2, 5, 32, 8, 128, (62, 300)),
    (3, 2, 16, 16, 64, (0, 63, 127)),
])
def test_fused_rope_attention_bitwise(B, S, Hq, Hkv, D, pos):
    from csaq._lib import check, lib, stream_of
    dt = torch.bfloat16
    Lmax = 640
    nq, nkv = Hq * D, Hkv * D
    g = torch.Generator().manual_seed(B * 100 + S)
    qkv = torch.randn(B * S, nq + 2 * nkv, generator=g).to(dt).to(DEV)
    kc0 = torch.randn(B, Hkv, Lmax, D, generator=g).to(dt).to(DEV)
    vc0 = torch.randn(B, Hkv, Lmax, D, generator=g).to(dt).to(DEV)
    cos, sin = _tables(Lmax, D, dt)
    pos0 = torch.tensor(pos, dtype=torch.int32, device=DEV)
    scale = 1.0 / math.sqrt(D)
    st = stream_of(qkv)
    floats = lib().csaq_attention_workspace_floats(B, S, Hq, Hkv, D, Lmax)
    # A: RoPE kernel, then attention
    kA, vA = kc0.clone(), vc0.clone()
    q_rot = torch.empty(B * S, nq, dtype=dt, device=DEV)
    check(lib().csaq_rope_kv(qkv.data_ptr(), qkv.stride(0), qkv[:, nq:].data_ptr(), qkv.stride(0),
                             qkv[:, nq + nkv:].data_ptr(), qkv.stride(0), pos0.data_ptr(), B, S, Hq, Hkv, D,
                             cos.data_ptr(), sin.data_ptr(), q_rot.data_ptr(), kA.data_ptr(), vA.data_ptr(), Lmax,
                             2, st), "rope_kv")
    outA = torch.empty(B * S, nq, dtype=dt, device=DEV)
    part = torch.zeros(floats, dtype=torch.float32, device=DEV)
    tick = torch.zeros(B * Hkv, dtype=torch.int32, device=DEV)
    check(lib().csaq_decode_attention(q_rot.data_ptr(), kA.data_ptr(), vA.data_ptr(), pos0.data_ptr(), B, S, Hq,
                                      Hkv, D, Lmax, scale, part.data_ptr(), tick.data_ptr(), outA.data_ptr(), 2, st),
          "attention")
    # B: one launch
    kB, vB = kc0.clone(), vc0.clone()
    outB = torch.full((B * S, nq), float("nan"), dtype=dt, device=DEV)
    part2 = torch.zeros(floats, dtype=torch.float32, device=DEV)
    tick2 = torch.zeros(B * Hkv, dtype=torch.int32, device=DEV)
    for _ in range(2):  # twice: the tickets are left at zero for the next call
        check(lib().csaq_decode_attention_rope(qkv.data_ptr(), qkv[:, nq:].data_ptr(), qkv[:, nq + nkv:].data_ptr(),
                                               qkv.stride(0), pos0.data_ptr(), B, S, Hq, Hkv, D, cos.data_ptr(),
                                               sin.data_ptr(), kB.data_ptr(), vB.data_ptr(), Lmax, scale,
                                               part2.data_ptr(), tick2.data_ptr(), outB.data_ptr(), 2, st),
              "attention_rope")
        torch.cuda.synchronize()
        assert torch.equal(outA, outB)
        assert torch.equal(kA, kB) and torch.equal(vA, vB)
    assert int(tick2.abs().sum()) == 0
    # against fp32 rotary attention
    G = Hq // Hkv
    q = qkv[:, :nq].float().view(B, S, Hq, D)
    kn = qkv[:, nq:nq + nkv].float().view(B, S, Hkv, D)
    ref = torch.empty(B, S, Hq, D, device=DEV)
    for b in range(B):
        for s in range(S):
            p = pos[b] + s
            qr = _rope_ref(q[b, s], cos[p], sin[p]).to(dt).float()
            keys = kB[b, :, :p + 1].float()  # the cache, new keys included (checked bitwise above)
            kr = _rope_ref(kn[b, s], cos[p], sin[p]).to(dt).float()
            assert torch.allclose(keys[:, p], kr, atol=0, rtol=0) or torch.allclose(keys[:, p], kr, rtol=1e-2)
            w = torch.softmax(torch.einsum("hd,hnd->hn", qr, keys.repeat_interleave(G, 0)) * scale, -1)
            ref[b, s] = torch.einsum("hn,hnd->hd", w, vB[b, :, :p + 1].float().repeat_interleave(G, 0))
    o = outB.float().view(B, S, Hq, D)
    rel = float((o - ref).norm() / ref.norm())
    assert rel <= 1e-2 and float((o - ref).abs().max() / ref.abs().max()) <= 1e-2, rel
