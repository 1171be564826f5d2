"""GPU parity of the quantisation kernels and the quantised linear.

Integer outputs (codes, scales, zero points, unpacked codes, dequantised fp32
weights) are compared bit for bit with the fixtures recorded from csaq-quant
and with the oracle; linear outputs use the 1e-2 relative bound of _tol.py.
"""

import hashlib
import warnings

import numpy as np
import pytest
import torch

from _tol import assert_linear_close
from oracle import csaq_oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _t(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    return t if dtype is None else t.to(dtype)


def _w_from_golden(kgold, key):
    bits, gs, r, c, dt = kgold[f"{key}_meta"]
    W = kgold[f"{key}_W"]
    tdt = {0: torch.float32, 1: torch.float16, 2: torch.bfloat16}[int(dt)]
    return _t(W).to(tdt), int(bits), int(gs)


def _qpc_keys(g):
    return sorted({k.split("_")[0] for k in g.files if k.startswith("qpc")}, key=lambda s: int(s[3:]))


def _sha(t):
    return hashlib.sha256(np.ascontiguousarray(t.cpu().numpy()).tobytes()).hexdigest()


def test_quantize_per_channel_matches_reference(kgold):
    from csaq.kernels import quantize_per_channel
    for key in _qpc_keys(kgold):
        W, bits, gs = _w_from_golden(kgold, key)
        qw = quantize_per_channel(W.to(DEV), bits, gs)
        assert qw.qdata.is_cuda
        np.testing.assert_array_equal(qw.qdata.cpu().numpy(), kgold[f"{key}_qdata"], err_msg=key)
        np.testing.assert_array_equal(qw.scales.cpu().numpy().view(np.uint32),
                                      kgold[f"{key}_scales"].view(np.uint32), err_msg=key)
        np.testing.assert_array_equal(qw.zero_points.cpu().numpy(), kgold[f"{key}_zps"], err_msg=key)
        if f"{key}_deq" in kgold.files:
            np.testing.assert_array_equal(qw.dequantize().cpu().numpy().view(np.uint32),
                                          kgold[f"{key}_deq"].view(np.uint32), err_msg=key)


def test_quantize_cpu_input_returns_cpu(kgold):
    from csaq.kernels import quantize_per_channel
    W, bits, gs = _w_from_golden(kgold, "qpc0")
    qw = quantize_per_channel(W, bits, gs)
    assert not qw.qdata.is_cuda
    np.testing.assert_array_equal(qw.qdata.numpy(), kgold["qpc0_qdata"])


def test_16bit_passthrough(kgold):
    from csaq.kernels import quantize_per_channel
    qw = quantize_per_channel(_t(kgold["q16_W"]).to(DEV), 16)
    np.testing.assert_array_equal(qw.qdata.cpu().numpy(), kgold["q16_qdata"])
    np.testing.assert_array_equal(qw.dequantize().cpu().numpy(), kgold["q16_deq"])


def test_shared_scale_matches_reference(kgold):
    from csaq.kernels import quantize_shared_scale
    keys = sorted({k.rsplit("_", 1)[0] for k in kgold.files if k.startswith("qss")})
    for key in keys:
        bits, gs, n_warn = kgold[f"{key}_meta"]
        with warnings.catch_warnings(record=True) as wl:
            warnings.simplefilter("always")
            qw = quantize_shared_scale(_t(kgold[f"{key}_W"]).to(DEV), _t(kgold[f"{key}_L"]).to(DEV),
                                       int(bits), int(gs))
        assert len([w for w in wl if "Follower row outlier" in str(w.message)]) == n_warn, key
        assert qw.shared_scale
        np.testing.assert_array_equal(qw.qdata.cpu().numpy(), kgold[f"{key}_qdata"], err_msg=key)
        np.testing.assert_array_equal(qw.scales.cpu().numpy(), kgold[f"{key}_scales"], err_msg=key)
        np.testing.assert_array_equal(qw.zero_points.cpu().numpy(), kgold[f"{key}_zps"], err_msg=key)


@pytest.mark.parametrize("bits", [2, 4, 8])
def test_pack_unpack(kgold, bits):
    from csaq.kernels import _pack, _unpack
    for (r, c) in [(16, 64), (8, 37), (3, 5)]:
        k = f"pk{bits}_{r}x{c}"
        p = _pack(_t(kgold[f"{k}_q"]).to(DEV), bits)
        np.testing.assert_array_equal(p.cpu().numpy(), kgold[f"{k}_packed"])
        np.testing.assert_array_equal(_unpack(p, bits, r, c).cpu().numpy(), kgold[f"{k}_unpacked"])
    with pytest.raises(ValueError, match="Unsupported bits for packing"):
        _pack(torch.zeros(2, 2, dtype=torch.int32, device=DEV), 3)
    with pytest.raises(ValueError, match="Unsupported bits for unpacking"):
        _unpack(torch.zeros(2, 2, dtype=torch.uint8, device=DEV), 16, 2, 1)


def test_float_to_int_matches_oracle():
    from csaq.kernels import _float_to_int
    g = torch.Generator().manual_seed(3)
    W = torch.randn(33, 77, generator=g)
    s = torch.rand(33, generator=g) * 0.1 + 1e-3
    z = torch.randint(0, 16, (33,), generator=g, dtype=torch.int32)
    q = _float_to_int(W.to(DEV), s.to(DEV), z.to(DEV), 4).cpu().numpy()
    np.testing.assert_array_equal(q, O.float_to_int(W.numpy(), s.numpy(), z.numpy(), 4))


def _cliques_from_golden(kgold, k):
    rows, lens = kgold[f"{k}_rows"], kgold[f"{k}_clen"]
    cl, s = [], 0
    for n, b, l in zip(lens, kgold[f"{k}_cbits"], kgold[f"{k}_clead"]):
        cl.append({"rows": rows[s:s + n].tolist(), "bits": int(b), "leader": int(l)})
        s += n
    return cl


def test_from_cliques_matches_reference(kgold):
    from csaq.kernels import CSAQLinear
    for fi in range(3):
        k = f"fc{fi}"
        lin = torch.nn.Linear(128, 48, bias=True).to(DEV)
        lin.weight.data = _t(kgold[f"{k}_W"]).to(DEV)
        lin.bias.data = _t(kgold[f"{k}_bias"]).to(DEV)
        layer = CSAQLinear.from_cliques(lin, _cliques_from_golden(kgold, k), verbose=False)
        assert layer.bits == int(kgold[f"{k}_bits"][0])
        np.testing.assert_array_equal(layer.weight_packed.cpu().numpy(), kgold[f"{k}_packed"])
        np.testing.assert_array_equal(layer.weight_scales.cpu().numpy(), kgold[f"{k}_scales"])
        np.testing.assert_array_equal(layer.weight_zp.cpu().numpy(), kgold[f"{k}_zp"])
        # fp32 activations go through the CUDA-core kernel
        y = layer(_t(kgold[f"{k}_x"]).to(DEV))
        assert_linear_close(y.cpu().numpy(), kgold[f"{k}_y"], what=k)
        # bf16 activations through the tensor-core kernel (K = 128)
        xb = _t(kgold[f"{k}_x"]).to(DEV).to(torch.bfloat16)
        Wd = layer._get_weight_fp32().cpu().numpy()
        yb = layer(xb).float().cpu().numpy()
        assert_linear_close(yb, O.linear_ref(xb.float().cpu().numpy(), Wd, kgold[f"{k}_bias"]), what=k)


def test_mixed_tiers_reduced_golden(kgold):
    from csaq.kernels import quantize_per_channel
    W = _t(kgold["mix_W"]).to(DEV)
    for b in (16, 8, 4):
        rows = _t(kgold[f"mix_rows{b}"]).to(DEV)
        qw = quantize_per_channel(W[rows], b, 128)
        np.testing.assert_array_equal(qw.qdata.cpu().numpy(), kgold[f"mix_q{b}"])
        if b != 16:
            np.testing.assert_array_equal(qw.scales.cpu().numpy(), kgold[f"mix_s{b}"])
            np.testing.assert_array_equal(qw.zero_points.cpu().numpy(), kgold[f"mix_z{b}"])


def test_full_size_mixed_tiers_digest(digests):
    """The 4096x4096 mixed linear: GPU codes/scales/zps/dequant hash to the reference's digests."""
    from csaq import _synthetic as syn
    from csaq.kernels import quantize_per_channel
    case = syn.mixed_linear(n=4096, k=4096, m=1, seed=0)
    W = case.W.to(DEV)
    for b, rows in case.tier_rows.items():
        d = digests[f"mixed4096_tier{b}"]
        qw = quantize_per_channel(W[rows.to(DEV)], b, 128)
        assert _sha(qw.qdata) == d["qdata"], b
        assert _sha(qw.scales) == d["scales"], b
        assert _sha(qw.zero_points) == d["zps"], b
        assert _sha(qw.dequantize()) == d["deq"], b


# ── quantised linear ────────────────────────────────────────────────────────

def _mixed_layer(n, k, seed, dtype, bits=(16, 8, 4), protect=0.0, bias=False, group_size=128,
                 fracs=None):
    from csaq import _synthetic as syn
    from csaq.kernels import CSAQLinear
    fracs = fracs if fracs is not None else (0.1, 0.2, 0.3)[:len(bits) - 1]
    case = syn.mixed_linear(n=n, k=k, m=1, seed=seed, dtype=dtype, bits=bits, fracs=fracs)
    lin = torch.nn.Linear(k, n, bias=bias, dtype=dtype).to(DEV)
    lin.weight.data = case.W.to(DEV)
    if bias:
        lin.bias.data = (torch.randn(n, generator=torch.Generator().manual_seed(seed + 1)) * 0.1).to(dtype).to(DEV)
    prot = None
    if protect:
        prot = torch.sort(case.order[:max(1, int(protect * n))]).values
    layer = CSAQLinear.from_tiers(lin, case.tier_rows, group_size=group_size, protected_rows=prot)
    return layer, case, prot


def _oracle_mixed(case, group_size=128):
    W = case.W.float().numpy() if case.W.dtype == torch.bfloat16 else case.W.numpy()
    tiers = {b: r.numpy() for b, r in case.tier_rows.items()}
    return O.mixed_weight(W, tiers, group_size)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("m", [1, 3, 8, 9, 16, 40])
def test_qgemv_mixed_matches_oracle(dtype, m):
    layer, case, _ = _mixed_layer(256, 512, seed=m, dtype=dtype, bias=True)
    Wref = _oracle_mixed(case)
    g = torch.Generator().manual_seed(100 + m)
    x = torch.randn(m, 512, generator=g).to(dtype)
    y = layer(x.to(DEV)).float().cpu().numpy()
    y_ref = O.linear_ref(x.float().numpy(), Wref, layer.bias.float().cpu().numpy())
    assert_linear_close(y, y_ref, what=f"{dtype} m={m}")


@pytest.mark.parametrize("m", [5, 8])
def test_qgemv_long_k_split_records_matches_oracle(m):
    """K = 14336 with several tokens: the activation records no longer fit one
    CTA, so the two CTAs of a cluster each hold half of the chunks (read by
    the other through distributed shared memory). Against the oracle, and
    bitwise equal to one token at a time."""
    layer, case, _ = _mixed_layer(300, 14336, seed=m, dtype=torch.bfloat16, bias=True)
    Wref = _oracle_mixed(case)
    x = torch.randn(m, 14336, generator=torch.Generator().manual_seed(m)).to(torch.bfloat16)
    y = layer(x.to(DEV))
    y_ref = O.linear_ref(x.float().numpy(), Wref, layer.bias.float().cpu().numpy())
    assert_linear_close(y.float().cpu().numpy(), y_ref, what=f"K=14336 m={m}")
    y1 = torch.cat([layer(x[i:i + 1].to(DEV)) for i in range(m)])
    assert torch.equal(y1, y)


@pytest.mark.parametrize("bits", [(2,), (4,), (8,), (16,), (8, 2), (16, 4, 2)])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_qgemv_every_bit_width(bits, dtype):
    from csaq import _synthetic as syn
    from csaq.kernels import CSAQLinear
    n, k = 200, 384
    case = syn.mixed_linear(n=n, k=k, m=1, seed=7, dtype=dtype, bits=(4,), fracs=())
    order = case.order
    tier_rows, start = {}, 0
    for i, b in enumerate(bits):
        cnt = n - start if i == len(bits) - 1 else n // len(bits)
        tier_rows[b] = torch.sort(order[start:start + cnt]).values
        start += cnt
    case.tier_rows = tier_rows
    lin = torch.nn.Linear(k, n, bias=False, dtype=dtype).to(DEV)
    lin.weight.data = case.W.to(DEV)
    layer = CSAQLinear.from_tiers(lin, tier_rows, group_size=128)
    Wref = _oracle_mixed(case)
    x = torch.randn(5, k, generator=torch.Generator().manual_seed(1)).to(dtype)
    y = layer(x.to(DEV)).float().cpu().numpy()
    assert_linear_close(y, O.linear_ref(x.float().numpy(), Wref), what=str(bits))


@pytest.mark.parametrize("group_size", [256, -1])
def test_qgemv_group_sizes(group_size):
    """Scale groups wider than one 128-column chunk, and per-channel tiers."""
    layer, case, _ = _mixed_layer(96, 1024, seed=11, dtype=torch.bfloat16, bits=(8, 4, 2),
                                  group_size=group_size)
    W = case.W.float().numpy()
    Wref = O.mixed_weight(W, {b: r.numpy() for b, r in case.tier_rows.items()}, group_size)
    x = torch.randn(4, 1024, generator=torch.Generator().manual_seed(2)).to(torch.bfloat16)
    y = layer(x.to(DEV)).float().cpu().numpy()
    assert_linear_close(y, O.linear_ref(x.float().numpy(), Wref), what=f"gs={group_size}")


def test_qgemv_tensor_core_vs_cuda_core():
    """The two GPU kernels agree on the same descriptors."""
    from csaq import _lib
    from csaq._lib import check, dtype_code, lib, stream_of
    layer, case, _ = _mixed_layer(300, 1024, seed=5, dtype=torch.bfloat16, bits=(16, 8, 4, 2))
    x = torch.randn(7, 1024, generator=torch.Generator().manual_seed(9)).to(torch.bfloat16).to(DEV)
    ys = []
    for simt in (False, True):
        y = torch.zeros(7, 300, dtype=torch.bfloat16, device=DEV)
        d = layer.gemv_descriptors(y)
        if simt:
            check(lib().csaq_qgemv_simt(_lib.tier_array(d), len(d), 1024, x.data_ptr(), dtype_code(x.dtype), 7,
                                        1024, stream_of(x)), "qgemv")
        else:
            _lib.qgemv(d, 1024, x, 7)
        ys.append(y.float().cpu().numpy())
    assert_linear_close(ys[0], ys[1], what="mma vs simt")


def test_qgemv_verify_patch():
    """Verify mode: protected rows come from their fp16 originals, all others
    from the codes, in one launch."""
    # 8/4-bit tiers: the protected (most salient) rows are quantised in the draft pass
    layer, case, prot = _mixed_layer(256, 512, seed=3, dtype=torch.bfloat16, protect=0.1,
                                     bits=(8, 4), fracs=(0.1,))
    Wq = _oracle_mixed(case)
    Wv = Wq.copy()
    p = prot.numpy()
    Wv[p] = case.W.float().numpy()[p].astype(np.float16).astype(np.float32)
    x = torch.randn(5, 512, generator=torch.Generator().manual_seed(4)).to(torch.bfloat16)
    xd = x.to(DEV)
    layer.verify_mode = False
    y_draft = layer(xd).float().cpu().numpy()
    layer.verify_mode = True
    y_ver = layer(xd).float().cpu().numpy()
    layer.verify_mode = False
    assert_linear_close(y_draft, O.linear_ref(x.float().numpy(), Wq), what="draft")
    assert_linear_close(y_ver, O.linear_ref(x.float().numpy(), Wv), what="verify")
    assert np.abs(y_ver - y_draft)[:, p].max() > 0


def test_qgemv_residual_fusion():
    from csaq import _lib
    from csaq._lib import check, dtype_code, lib, stream_of
    layer, case, _ = _mixed_layer(128, 256, seed=8, dtype=torch.bfloat16)
    x = torch.randn(3, 256, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16).to(DEV)
    r = torch.randn(3, 128, generator=torch.Generator().manual_seed(2)).to(torch.bfloat16).to(DEV)
    y = r.clone()
    d = layer.gemv_descriptors(y, residual=y)
    _lib.qgemv(d, 256, x, 3)
    ref = r.float() + layer(x).float()
    assert_linear_close(y.float().cpu().numpy(), ref.cpu().numpy(), what="residual")


def test_qgemv_full_size_mixed_linear():
    """4096x4096 mixed linear (16/8/4 tiers), X fp16 at M = 1 and 16."""
    layer, case, _ = _mixed_layer(4096, 4096, seed=0, dtype=torch.float16)
    Wref = _oracle_mixed(case)
    for m in (1, 16):
        x = torch.randn(m, 4096, generator=torch.Generator().manual_seed(m)).half()
        y = layer(x.to(DEV)).float().cpu().numpy()
        assert_linear_close(y, O.linear_ref(x.float().numpy(), Wref), what=f"4096 m={m}")


@pytest.mark.parametrize("shape", [(4096, 4096), (1024, 14336), (300, 512)])
def test_qgemv_token_result_independent_of_m(shape):
    """A token's output is bitwise the same whether it is launched alone or
    with other tokens (the work partition does not depend on M)."""
    n, k = shape
    layer, _, _ = _mixed_layer(n, k, seed=3, dtype=torch.bfloat16)
    x = torch.randn(13, k, generator=torch.Generator().manual_seed(5)).to(torch.bfloat16).to(DEV)
    y_all = layer(x)
    for m in (1, 5, 13):
        y_m = layer(x[:m])
        assert torch.equal(y_m, y_all[:m]), m


def test_qgemv_no_abandoned_waits():
    """After the GEMV tests above, no warp gave up waiting for a weight copy."""
    import ctypes
    from csaq._lib import check, lib
    n = ctypes.c_int64(-1)
    check(lib().csaq_qgemv_wait_timeouts(ctypes.byref(n)), "wait_timeouts")
    assert n.value == 0


@pytest.mark.parametrize("m,n,k", [(32, 300, 512), (130, 256, 4096), (512, 1100, 1024)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_qgemm_matches_oracle(m, n, k, dtype):
    """The tcgen05 GEMM (M >= 32) against the oracle: within 1e-2 of the fp32
    dequant-then-matmul, and within the output dtype's rounding of the
    reference's own numerics (weights rounded to x.dtype before the matmul)."""
    from csaq import _lib
    layer, case, _ = _mixed_layer(n, k, seed=m + k, dtype=dtype, bias=True)
    Wref = _oracle_mixed(case)
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(m)).to(dtype)
    r = torch.randn(m, n, generator=torch.Generator().manual_seed(m + 1)).to(dtype)
    y = r.clone().to(DEV)
    d = layer.gemv_descriptors(y, residual=y)
    _lib.qgemm(d, k, x.to(DEV), m)
    got = y.float().cpu().numpy()
    bias = layer.bias.float().cpu().numpy()
    ref = O.linear_ref(x.float().numpy(), Wref, bias) + r.float().numpy()
    assert_linear_close(got, ref, what=f"qgemm {m}x{n}x{k} {dtype}")
    Wx = torch.from_numpy(Wref).to(dtype).float().numpy()   # the reference rounds W to x.dtype
    ref_x = O.linear_ref(x.float().numpy(), Wx, bias) + r.float().numpy()
    tight = 4e-3 if dtype == torch.bfloat16 else 2e-3        # the output's own rounding: 2^-8 / 2^-11
    assert_linear_close(got, ref_x, rtol=tight, what=f"qgemm (x-dtype weights) {m}x{n}x{k}")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_qgemm_low_bit_tiers(dtype):
    """8/4/2-bit tiers (the 70B prefill mix), group 256, ragged M and rows."""
    from csaq import _lib
    layer, case, _ = _mixed_layer(600, 1024, seed=7, dtype=dtype, bits=(8, 4, 2), fracs=(0.1, 0.6),
                                  group_size=256)
    Wref = _oracle_mixed(case, group_size=256)
    for m in (40, 300):
        x = torch.randn(m, 1024, generator=torch.Generator().manual_seed(m)).to(dtype)
        y = torch.zeros(m, 600, dtype=dtype, device=DEV)
        _lib.qgemm(layer.gemv_descriptors(y), 1024, x.to(DEV), m)
        got = y.float().cpu().numpy()
        assert_linear_close(got, O.linear_ref(x.float().numpy(), Wref), what=f"qgemm 8/4/2 m={m}")
        Wx = torch.from_numpy(Wref).to(dtype).float().numpy()
        tight = 4e-3 if dtype == torch.bfloat16 else 2e-3
        assert_linear_close(got, O.linear_ref(x.float().numpy(), Wx), rtol=tight, what=f"qgemm 8/4/2 x-dtype m={m}")
        # without the GEMV blocks the scales come from the reference layout: same bits
        y2 = torch.zeros_like(y)
        descs = layer.gemv_descriptors(y2)
        for d in descs:
            d.blocks = None
        _lib.qgemm(descs, 1024, x.to(DEV), m)
        assert torch.equal(y2, y)


def test_qgemm_token_result_independent_of_m():
    """A token's GEMM output is bitwise the same for any M (tiles split tokens,
    never the K accumulation)."""
    from csaq import _lib
    layer, _, _ = _mixed_layer(520, 1024, seed=11, dtype=torch.bfloat16)
    x = torch.randn(300, 1024, generator=torch.Generator().manual_seed(2)).to(torch.bfloat16).to(DEV)
    outs = {}
    for m in (33, 140, 300):
        y = torch.zeros(m, 520, dtype=torch.bfloat16, device=DEV)
        _lib.qgemm(layer.gemv_descriptors(y), 1024, x[:m], m)
        outs[m] = y
    assert torch.equal(outs[33], outs[300][:33])
    assert torch.equal(outs[140], outs[300][:140])


def test_qgemm_forward_dispatch_and_no_timeouts():
    """CSAQLinear.forward takes the GEMM from 32 tokens on; it agrees with the GEMV."""
    import ctypes
    from csaq import _lib
    from csaq._lib import check, lib
    layer, _, _ = _mixed_layer(512, 1024, seed=5, dtype=torch.bfloat16)
    x = torch.randn(48, 1024, generator=torch.Generator().manual_seed(2)).to(torch.bfloat16).to(DEV)
    y_gemm = layer(x)
    y_gemv = torch.empty_like(y_gemm)
    _lib.qgemv(layer.gemv_descriptors(y_gemv), 1024, x, 48)
    assert_linear_close(y_gemm.float().cpu().numpy(), y_gemv.float().cpu().numpy(), what="gemm vs gemv")
    n = ctypes.c_int64(-1)
    check(lib().csaq_qgemm_wait_timeouts(ctypes.byref(n)), "timeouts")
    assert n.value == 0


def test_uniform_layer_ragged_shapes():
    """K = 37 (no 128-column chunks): the CUDA-core kernel serves it."""
    from csaq.kernels import CSAQLinear
    lin = torch.nn.Linear(37, 11, bias=True).to(DEV)
    W = lin.weight.data.clone().cpu().numpy()
    cl = [{"rows": list(range(11)), "bits": 4, "leader": 2}]
    layer = CSAQLinear.from_cliques(lin, cl)
    packed, scales, zp, bits = O.from_cliques(W, cl)
    np.testing.assert_array_equal(layer.weight_packed.cpu().numpy(), packed)
    x = torch.randn(2, 5, 37)
    for dt in (torch.float32, torch.float16, torch.bfloat16):
        y = layer(x.to(DEV).to(dt)).float().cpu().numpy().reshape(10, 11)
        Wd = O.get_weight_fp32(packed, scales, zp, bits, 11, 37)
        ref = O.linear_ref(x.to(dt).float().numpy().reshape(10, 37), Wd, layer.bias.float().cpu().numpy())
        assert_linear_close(y, ref, what=str(dt))
