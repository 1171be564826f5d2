"""Generate golden fixtures by running csaq-quant v0.5.9 itself.

Run in the build container (where the reference source tree is present):

    python tests/golden/make_goldens.py --ref <reference source tree> [--full]

Outputs (committed):
  tests/golden/kernels_golden.npz  quant/pack/dequant/shared-scale/from_cliques cases
  tests/golden/calib_golden.npz    masks, co-activation counts, cliques, salience, solver
  tests/golden/digests.json        sha256 digests of full-size workloads (--full):
                                   4096x4096 mixed linear tiers, 11008-channel co-activation

Inputs are regenerated from csaq/_synthetic.py or stored with the case, so the
fixtures are self-contained. The reference is imported from a temporary copy
so nothing is written into its tree.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import shutil
import sys
import tempfile
import warnings

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def _load_synthetic():
    """Load csaq-quant_b200/csaq/_synthetic.py by path: the reference package is
    also named ``csaq``, so the two cannot share ``sys.modules['csaq']``."""
    import importlib.util
    path = os.path.join(REPO, "csaq-quant_b200", "csaq", "_synthetic.py")
    spec = importlib.util.spec_from_file_location("csaq_b200_synthetic", path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod
    spec.loader.exec_module(mod)
    return mod


syn = _load_synthetic()


def _import_reference(ref_root: str):
    tmp = tempfile.mkdtemp(prefix="csaq_ref_")
    shutil.copytree(os.path.join(ref_root, "csaq"), os.path.join(tmp, "csaq"))
    sys.dont_write_bytecode = True
    sys.path.insert(0, tmp)
    import csaq.kernels as rk  # noqa: E402
    import csaq.core as rc  # noqa: E402
    import csaq.config as rcfg  # noqa: E402
    sys.path.remove(tmp)
    return rk, rc, rcfg


def sha(t) -> str:
    a = t.numpy() if isinstance(t, torch.Tensor) else np.asarray(t)
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def labels_from_cliques(cliques, n):
    lab = np.full(n, -1, np.int64)
    for ci, c in enumerate(cliques):
        lab[np.asarray(c, np.int64)] = ci
    return lab


def kernel_cases(rk, out: dict):

    def rand(rows, cols, seed, dtype=torch.float32, scale=1.0):
        g = torch.Generator().manual_seed(seed)
        return (torch.randn(rows, cols, generator=g) * scale).to(dtype)

    cases = []
    for (r, c) in [(16, 64), (8, 37), (9, 300), (5, 128), (3, 256)]:
        for bits in (2, 4, 8):
            for gs in (-1, 32, 64, 128, 100, 4096):
                cases.append((r, c, bits, gs, torch.float32, 1.0))
    for bits in (2, 4, 8):
        cases.append((24, 512, bits, 128, torch.float16, 0.02))
        cases.append((24, 512, bits, 128, torch.bfloat16, 0.02))
    names = []
    for idx, (r, c, bits, gs, dt, sc) in enumerate(cases):
        W = rand(r, c, 1000 + idx, dt, sc)
        if idx % 7 == 3:  # degenerate groups: constant and zero rows
            W[0, :] = 0.0
            if r > 1:
                W[1, :] = 0.5
            if r > 2:
                W[2, :] = -0.75
        qw = rk.quantize_per_channel(W, bits, gs)
        key = f"qpc{idx}"
        names.append(key)
        out[f"{key}_W"] = W.float().numpy() if dt == torch.bfloat16 else W.numpy()
        out[f"{key}_meta"] = np.array([bits, gs, r, c, {torch.float32: 0, torch.float16: 1,
                                                          torch.bfloat16: 2}[dt]], np.int64)
        out[f"{key}_qdata"] = qw.qdata.numpy()
        out[f"{key}_scales"] = qw.scales.numpy()
        out[f"{key}_zps"] = qw.zero_points.numpy()
        try:
            out[f"{key}_deq"] = qw.dequantize().numpy()
        except Exception:
            pass  # the reference cannot dequantise ragged groups
    # 16-bit passthrough
    W = rand(8, 32, 77)
    qw = rk.quantize_per_channel(W, 16)
    out["q16_W"], out["q16_qdata"], out["q16_deq"] = W.numpy(), qw.qdata.numpy(), qw.dequantize().numpy()

    # shared scale
    sidx = 0
    for bits in (2, 4, 8):
        for gs in (-1, 32, 100):
            W = rand(16, 64 if gs != 100 else 250, 500 + sidx)
            leader = W[sidx % 16].clone()
            with warnings.catch_warnings(record=True) as wlist:
                warnings.simplefilter("always")
                qw = rk.quantize_shared_scale(W, leader, bits, gs)
            key = f"qss{sidx}"
            out[f"{key}_W"], out[f"{key}_L"] = W.numpy(), leader.numpy()
            out[f"{key}_meta"] = np.array([bits, gs, len(wlist)], np.int64)
            out[f"{key}_qdata"] = qw.qdata.numpy()
            out[f"{key}_scales"] = qw.scales.numpy()
            out[f"{key}_zps"] = qw.zero_points.numpy()
            sidx += 1
    torch.manual_seed(99)
    leader = torch.randn(64) * 0.01
    W = torch.randn(8, 64) * 10.0
    with warnings.catch_warnings(record=True) as wlist:
        warnings.simplefilter("always")
        qw = rk.quantize_shared_scale(W, leader, 4)
    out["qss_outlier_W"], out["qss_outlier_L"] = W.numpy(), leader.numpy()
    out["qss_outlier_meta"] = np.array([4, -1, len(wlist)], np.int64)
    out["qss_outlier_qdata"] = qw.qdata.numpy()
    out["qss_outlier_scales"] = qw.scales.numpy()
    out["qss_outlier_zps"] = qw.zero_points.numpy()

    # pack / unpack
    for bits in (2, 4, 8):
        for (r, c) in [(16, 64), (8, 37), (3, 5)]:
            g = torch.Generator().manual_seed(bits * 100 + c)
            q = torch.randint(0, 2 ** bits, (r, c), generator=g, dtype=torch.int32)
            p = rk._pack(q, bits)
            out[f"pk{bits}_{r}x{c}_q"] = q.numpy()
            out[f"pk{bits}_{r}x{c}_packed"] = p.numpy()
            out[f"pk{bits}_{r}x{c}_unpacked"] = rk._unpack(p, bits, r, c).numpy()

    # from_cliques + CSAQLinear.forward (fp32)
    for fi, (bits_list, seed) in enumerate([([4, 4, 8], 3), ([8, 8, 4], 4), ([2, 2, 4], 5)]):
        torch.manual_seed(seed)
        lin = torch.nn.Linear(128, 48, bias=True)
        lin.weight.data = torch.randn(48, 128) * 0.02
        W = lin.weight.data.clone()
        cl = [
            {"rows": [0, 5, 9, 17], "bits": bits_list[0], "leader": 5},
            {"rows": list(range(20, 40)), "bits": bits_list[1], "leader": 31},
            {"rows": [1, 2, 3], "bits": bits_list[2], "leader": 1},
        ]  # rows 4, 6-8, 10-16, 18, 19, 40-47 uncovered
        layer = rk.CSAQLinear.from_cliques(lin, cl, verbose=False)
        x = torch.randn(3, 128)
        with torch.no_grad():
            y = layer(x)
        key = f"fc{fi}"
        out[f"{key}_W"], out[f"{key}_bias"], out[f"{key}_x"] = W.numpy(), lin.bias.data.numpy(), x.numpy()
        out[f"{key}_rows"] = np.concatenate([np.asarray(c["rows"]) for c in cl])
        out[f"{key}_clen"] = np.asarray([len(c["rows"]) for c in cl])
        out[f"{key}_cbits"] = np.asarray([c["bits"] for c in cl])
        out[f"{key}_clead"] = np.asarray([c["leader"] for c in cl])
        out[f"{key}_packed"] = layer.weight_packed.numpy()
        out[f"{key}_scales"] = layer.weight_scales.numpy()
        out[f"{key}_zp"] = layer.weight_zp.numpy()
        out[f"{key}_bits"] = np.asarray([layer.bits])
        out[f"{key}_y"] = y.numpy()

    # reduced mixed linear (the 4096x4096 workload's recipe at 256x512)
    case = syn.mixed_linear(n=256, k=512, m=16, seed=0)
    out["mix_W"] = case.W.numpy()
    out["mix_X"] = case.X.numpy()
    for b, rows in case.tier_rows.items():
        out[f"mix_rows{b}"] = rows.numpy()
        qw = rk.quantize_per_channel(case.W[rows], b, 128)
        out[f"mix_q{b}"] = qw.qdata.numpy()
        out[f"mix_s{b}"] = qw.scales.numpy()
        out[f"mix_z{b}"] = qw.zero_points.numpy()

    return names


def calib_cases(rk, rc, rcfg, out: dict):
    import torch.nn as nn

    class _One(nn.Module):
        def __init__(self, cin, cout):
            super().__init__()
            self.fc = nn.Linear(cin, cout)

    # Jaccard cliques through the reference's own _build_cliques
    act = syn.activations(384, 96, seed=1)
    mask = act > 0.5
    out["cl_act"] = act.numpy()
    out["cl_mask"] = mask.numpy()
    m = mask.float()
    out["cl_inter"] = torch.matmul(m.t(), m).to(torch.int64).numpy()
    out["cl_f"] = m.sum(0).to(torch.int64).numpy()
    for thr in (0.85, 0.6, 0.3, 0.0, 1.5):
        cfg = rcfg.CSAQConfig(clique_threshold=thr)
        prof = rc.CausalProfiler(_One(8, 96), cfg)
        prof._act_history["fc"] = [mask[:200], mask[200:]]
        cl = prof._build_cliques()["fc"]
        out[f"cl_labels_{thr}"] = labels_from_cliques(cl, 96)
        out[f"cl_flat_{thr}"] = np.concatenate([np.asarray(c) for c in cl])
        out[f"cl_len_{thr}"] = np.asarray([len(c) for c in cl])
    # per_channel mode
    prof = rc.CausalProfiler(_One(8, 96), rcfg.CSAQConfig(clique_mode="per_channel"))
    out["cl_perchannel_len"] = np.asarray([len(c) for c in prof._build_cliques()["fc"]])

    # forward-hook top-k masks
    for hi, (alpha, dt, shape) in enumerate([(1.0, torch.float16, (2, 50, 200)),
                                            (0.5, torch.float32, (7, 333)),
                                            (3.0, torch.bfloat16, (4, 64)),
                                            (20.0, torch.float16, (3, 40)),
                                            (1.0, torch.float16, (5, 9))]):
        g = torch.Generator().manual_seed(700 + hi)
        o = (torch.randn(*shape, generator=g) * 2).round(decimals=1).to(dt)  # ties
        cfg = rcfg.CSAQConfig(salience_alpha=alpha)
        cin = 4
        prof = rc.CausalProfiler(_One(cin, shape[-1]), cfg)
        hook = list(prof._modules["fc"]._forward_hooks.values())[0]
        hook(prof._modules["fc"], (torch.zeros(1, cin),), o)
        msk = prof._act_history["fc"][0]
        out[f"tk{hi}_out"] = o.float().numpy() if dt == torch.bfloat16 else o.numpy()
        out[f"tk{hi}_meta"] = np.asarray([alpha, {torch.float32: 0, torch.float16: 1,
                                                  torch.bfloat16: 2}[dt]], np.float64)
        out[f"tk{hi}_mask"] = msk.numpy()

    # salience: the reference accumulation arithmetic in fp32
    W, grads = syn.salience_inputs(24, 40, 3, seed=2)
    acc = torch.zeros(24, 40)
    for G in grads:
        acc += (G.float() * W.float()).abs()
    out["sal_W"] = W.numpy()
    out["sal_G"] = np.stack([G.numpy() for G in grads])
    out["sal_ref"] = (acc / 3).numpy()

    # solver + protected rows
    g = torch.Generator().manual_seed(5)
    sal = {"a.q": torch.rand(40, 16, generator=g), "b.k": torch.rand(24, 32, generator=g) * 2}
    cliques = {"a.q": [[i] for i in range(40)],
               "b.k": [[0, 3, 5], [1, 2], [4]] + [[i] for i in range(6, 24)]}
    for si, (tb, opts, floor) in enumerate([(4.0, [4, 8, 16], 0.1), (5.0, [4, 8, 16], 0.1),
                                            (3.0, [2, 4, 8], 0.2), (8.0, [8, 16], 0.0)]):
        cfg = rcfg.CSAQConfig(target_bits=tb, bit_options=opts, protection_floor=floor)
        budget, stats, actual = rc.solve_clique_budget(sal, cliques, cfg)
        recs = []
        for layer, cl in budget.items():
            for c in cl:
                recs.append((0 if layer == "a.q" else 1, c["rows"][0], c["bits"], c["leader"]))
        out[f"sv{si}_recs"] = np.asarray(recs, np.int64)
        out[f"sv{si}_meta"] = np.asarray([tb, floor, actual] + list(opts), np.float64)
        out[f"sv{si}_stats"] = np.asarray([stats.get(f"int{b}", 0) for b in (2, 4, 8, 16)])
    out["sv_sal_a"] = sal["a.q"].numpy()
    out["sv_sal_b"] = sal["b.k"].numpy()
    row_sal = sal["b.k"].sum(dim=1)
    out["prot_rows"] = row_sal.topk(max(1, int(0.1 * 24))).indices.sort().values.numpy()


def full_digests(rk, rc, rcfg) -> dict:
    import torch.nn as nn
    d = {}
    case = syn.mixed_linear(n=4096, k=4096, m=16, seed=0)
    for b, rows in case.tier_rows.items():
        qw = rk.quantize_per_channel(case.W[rows], b, 128)
        d[f"mixed4096_tier{b}"] = {
            "rows": sha(rows), "n_rows": int(rows.numel()), "qdata": sha(qw.qdata),
            "scales": sha(qw.scales), "zps": sha(qw.zero_points), "deq": sha(qw.dequantize()),
        }

    class _One(nn.Module):
        def __init__(self, cin, cout):
            super().__init__()
            self.fc = nn.Linear(cin, cout)

    act = syn.activations(64 * 128, 11008, seed=0)
    mask = act > 0.5
    m = mask.float()
    inter = torch.matmul(m.t(), m).to(torch.int32)
    d["coact11008"] = {"inter_i32": sha(inter), "f_i32": sha(m.sum(0).to(torch.int32)),
                       "density": float(m.mean())}
    del inter, m
    for thr in (0.85, 0.6):
        prof = rc.CausalProfiler(_One(8, 11008), rcfg.CSAQConfig(clique_threshold=thr))
        prof._act_history["fc"] = [mask]
        cl = prof._build_cliques()["fc"]
        lab = labels_from_cliques(cl, 11008)
        d["coact11008"][f"labels_{thr}"] = sha(lab)
        d["coact11008"][f"n_cliques_{thr}"] = len(cl)
    d["torch"] = torch.__version__
    return d


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="the csaq-quant v0.5.9 source tree (read only)")
    ap.add_argument("--full", action="store_true", help="also compute full-size digests")
    args = ap.parse_args()
    rk, rc, rcfg = _import_reference(args.ref)
    out: dict = {}
    kernel_cases(rk, out)
    np.savez_compressed(os.path.join(HERE, "kernels_golden.npz"), **out)
    out = {}
    calib_cases(rk, rc, rcfg, out)
    np.savez_compressed(os.path.join(HERE, "calib_golden.npz"), **out)
    if args.full:
        d = full_digests(rk, rc, rcfg)
        with open(os.path.join(HERE, "digests.json"), "w") as f:
            json.dump(d, f, indent=1, sort_keys=True)
    print("goldens written; torch", torch.__version__)


if __name__ == "__main__":
    main()
