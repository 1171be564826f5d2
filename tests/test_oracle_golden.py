"""The CPU oracle against fixtures recorded from csaq-quant itself.

Every check is bit-exact except the fp32 reference forward of from_cliques
layers (a matmul, compared with a tolerance).
"""

import warnings

import numpy as np
import pytest

from oracle import csaq_oracle as O


def _widen(W, dt):
    return W.astype(np.float16) if dt == 1 else W.astype(np.float32)


def _qpc_keys(g):
    return sorted({k.split("_")[0] for k in g.files if k.startswith("qpc")},
                  key=lambda s: int(s[3:]))


def test_quantize_per_channel_bit_exact(kgold):
    keys = _qpc_keys(kgold)
    assert len(keys) >= 90
    for key in keys:
        bits, gs, r, c, dt = kgold[f"{key}_meta"]
        W = _widen(kgold[f"{key}_W"], dt)
        qw = O.quantize_per_channel(W, int(bits), int(gs))
        np.testing.assert_array_equal(qw.qdata, kgold[f"{key}_qdata"], err_msg=key)
        np.testing.assert_array_equal(qw.scales.view(np.uint32),
                                      kgold[f"{key}_scales"].view(np.uint32), err_msg=key)
        np.testing.assert_array_equal(qw.zero_points, kgold[f"{key}_zps"], err_msg=key)
        if f"{key}_deq" in kgold.files:
            np.testing.assert_array_equal(qw.dequantize().view(np.uint32),
                                          kgold[f"{key}_deq"].view(np.uint32), err_msg=key)


def test_degenerate_groups_pinned(kgold):
    """Constant 0.5 / -0.75 rows: w_min + 1e-8 rounds back to w_min in fp32, so
    the reference stores scale 0 and saturates zero point and codes through +-inf."""
    seen = False
    for key in _qpc_keys(kgold):
        if (kgold[f"{key}_scales"] == 0).any():
            seen = True
    assert seen


def test_16bit_passthrough(kgold):
    qw = O.quantize_per_channel(kgold["q16_W"], 16)
    np.testing.assert_array_equal(qw.qdata, kgold["q16_qdata"])
    np.testing.assert_array_equal(qw.dequantize(), kgold["q16_deq"])


def test_shared_scale_bit_exact(kgold):
    keys = sorted({k.rsplit("_", 1)[0] for k in kgold.files if k.startswith("qss")})
    assert "qss_outlier" in keys
    for key in keys:
        bits, gs, n_warn = kgold[f"{key}_meta"]
        with warnings.catch_warnings(record=True) as wl:
            warnings.simplefilter("always")
            qw = O.quantize_shared_scale(kgold[f"{key}_W"], kgold[f"{key}_L"], int(bits), int(gs))
        assert len(wl) == n_warn, key
        np.testing.assert_array_equal(qw.qdata, kgold[f"{key}_qdata"], err_msg=key)
        np.testing.assert_array_equal(qw.scales, kgold[f"{key}_scales"], err_msg=key)
        np.testing.assert_array_equal(qw.zero_points, kgold[f"{key}_zps"], err_msg=key)


@pytest.mark.parametrize("bits", [2, 4, 8])
def test_pack_unpack_golden(kgold, bits):
    for (r, c) in [(16, 64), (8, 37), (3, 5)]:
        k = f"pk{bits}_{r}x{c}"
        p = O.pack(kgold[f"{k}_q"], bits)
        np.testing.assert_array_equal(p, kgold[f"{k}_packed"])
        np.testing.assert_array_equal(O.unpack(p, bits, r, c), kgold[f"{k}_unpacked"])
        np.testing.assert_array_equal(O.unpack(p, bits, r, c), kgold[f"{k}_q"])


def test_from_cliques_bit_exact(kgold):
    for fi in range(3):
        k = f"fc{fi}"
        rows = kgold[f"{k}_rows"]
        lens = kgold[f"{k}_clen"]
        cl, s = [], 0
        for n, b, l in zip(lens, kgold[f"{k}_cbits"], kgold[f"{k}_clead"]):
            cl.append({"rows": rows[s:s + n].tolist(), "bits": int(b), "leader": int(l)})
            s += n
        packed, scales, zp, bits = O.from_cliques(kgold[f"{k}_W"], cl)
        assert bits == int(kgold[f"{k}_bits"][0])
        np.testing.assert_array_equal(packed, kgold[f"{k}_packed"])
        np.testing.assert_array_equal(scales, kgold[f"{k}_scales"])
        np.testing.assert_array_equal(zp, kgold[f"{k}_zp"])
        W = O.get_weight_fp32(packed, scales, zp, bits, 48, 128)
        y = O.linear_ref(kgold[f"{k}_x"], W, kgold[f"{k}_bias"])
        np.testing.assert_allclose(y, kgold[f"{k}_y"], rtol=1e-5, atol=1e-6)


def test_mixed_tiers_bit_exact(kgold):
    W = kgold["mix_W"]
    for b in (16, 8, 4):
        rows = kgold[f"mix_rows{b}"]
        qw = O.quantize_per_channel(W[rows], b, 128)
        np.testing.assert_array_equal(qw.qdata, kgold[f"mix_q{b}"])
        np.testing.assert_array_equal(qw.scales, kgold[f"mix_s{b}"])
        np.testing.assert_array_equal(qw.zero_points, kgold[f"mix_z{b}"])


def test_coactivation_and_cliques(cgold):
    mask = cgold["cl_mask"]
    inter, f = O.coact_counts(mask)
    np.testing.assert_array_equal(inter, cgold["cl_inter"])
    np.testing.assert_array_equal(f, cgold["cl_f"])
    J = O.jaccard(inter, f)
    for thr in (0.85, 0.6, 0.3, 0.0, 1.5):
        cl = O.greedy_cliques(J, thr)
        np.testing.assert_array_equal(np.concatenate(cl), cgold[f"cl_flat_{thr}"])
        np.testing.assert_array_equal([len(c) for c in cl], cgold[f"cl_len_{thr}"])


def test_topk_masks(cgold):
    for hi in range(5):
        alpha, dt = cgold[f"tk{hi}_meta"]
        o = cgold[f"tk{hi}_out"]
        o = o.astype(np.float16) if int(dt) == 1 else o.astype(np.float32)
        m = O.topk_mask(o, float(alpha))
        np.testing.assert_array_equal(m, cgold[f"tk{hi}_mask"], err_msg=str(hi))


def test_salience(cgold):
    sal = O.salience_accumulate(cgold["sal_W"], list(cgold["sal_G"]))
    np.testing.assert_allclose(sal, cgold["sal_ref"], rtol=1e-6, atol=0)


def test_solver(cgold):
    sal = {"a.q": cgold["sv_sal_a"], "b.k": cgold["sv_sal_b"]}
    cliques = {"a.q": [[i] for i in range(40)],
               "b.k": [[0, 3, 5], [1, 2], [4]] + [[i] for i in range(6, 24)]}
    for si in range(4):
        meta = cgold[f"sv{si}_meta"]
        tb, floor, actual = meta[:3]
        opts = [int(b) for b in meta[3:]]
        budget, stats, act = O.solve_clique_budget(sal, cliques, tb, opts, floor)
        recs = [(0 if l == "a.q" else 1, c["rows"][0], c["bits"], c["leader"])
                for l, cl in budget.items() for c in cl]
        np.testing.assert_array_equal(np.asarray(recs), cgold[f"sv{si}_recs"])
        assert act == pytest.approx(actual, rel=0, abs=1e-12)
        np.testing.assert_array_equal([stats.get(f"int{b}", 0) for b in (2, 4, 8, 16)],
                                      cgold[f"sv{si}_stats"])


def test_protected_rows(cgold):
    rows = O.protected_rows(cgold["sv_sal_b"].sum(axis=1), 0.1)
    np.testing.assert_array_equal(rows, cgold["prot_rows"])


def test_greedy_accept():
    assert O.greedy_accept([5, 6, 7], [5, 6, 7, 8]) == (4, [5, 6, 7, 8])
    assert O.greedy_accept([5, 6, 7], [5, 9, 7, 8]) == (2, [5, 9])
    assert O.greedy_accept([5], [1, 2]) == (1, [1])


def test_full_size_mixed_tiers_digest(digests):
    """Oracle on the full 4096x4096 mixed linear matches the reference's sha256 digests."""
    import hashlib
    from csaq import _synthetic as syn
    case = syn.mixed_linear(n=4096, k=4096, m=1, seed=0)
    W = case.W.numpy()
    for b, rows in case.tier_rows.items():
        d = digests[f"mixed4096_tier{b}"]
        r = rows.numpy()
        assert hashlib.sha256(r.tobytes()).hexdigest() == d["rows"]
        qw = O.quantize_per_channel(W[r], b, 128)
        for name, arr in (("qdata", qw.qdata), ("scales", qw.scales), ("zps", qw.zero_points)):
            assert hashlib.sha256(np.ascontiguousarray(arr).tobytes()).hexdigest() == d[name], (b, name)
