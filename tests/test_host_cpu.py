"""The product's host-side pieces of the path against fixtures recorded from
csaq-quant itself, on the CPU (no kernels involved):

* csaq.core.solve_clique_budget (csaq/core.py:294-361): the bit assignment,
  leaders, achieved bits and tier statistics of four budgets;
* the protected-row choice of apply_csaq (csaq/core.py:382-403).
"""

import numpy as np
import pytest
import torch


def _budget_case(cgold):
    sal = {"a.q": torch.from_numpy(cgold["sv_sal_a"]), "b.k": torch.from_numpy(cgold["sv_sal_b"])}
    cliques = {"a.q": [[i] for i in range(40)],
               "b.k": [[0, 3, 5], [1, 2], [4]] + [[i] for i in range(6, 24)]}
    return sal, cliques


@pytest.mark.parametrize("si", range(4))
def test_solver_matches_reference(cgold, si):
    from csaq.config import CSAQConfig
    from csaq.core import solve_clique_budget
    sal, cliques = _budget_case(cgold)
    meta = cgold[f"sv{si}_meta"]
    tb, floor, actual = meta[:3]
    opts = [int(b) for b in meta[3:]]
    cfg = CSAQConfig(target_bits=float(tb), bit_options=opts, protection_floor=float(floor))
    budget, stats, act = solve_clique_budget(sal, cliques, cfg)
    recs = [(0 if l == "a.q" else 1, c["rows"][0], c["bits"], c["leader"])
            for l, cl in budget.items() for c in cl]
    # same cliques, bits and leaders, in the reference's order (layer by layer, by salience density)
    assert recs == list(map(tuple, cgold[f"sv{si}_recs"].tolist()))
    assert act == pytest.approx(float(actual), rel=0, abs=1e-12)
    assert [stats.get(f"int{b}", 0) for b in (2, 4, 8, 16)] == cgold[f"sv{si}_stats"].tolist()


def test_protected_rows_match_reference(cgold):
    from csaq.core import _protect_rows
    rows = _protect_rows(torch.from_numpy(cgold["sv_sal_b"]).sum(dim=1), 0.1)
    np.testing.assert_array_equal(rows.numpy(), cgold["prot_rows"])


def _sequential_budget(recs, config):
    """The reference's greedy (csaq/core.py:294-361) as a plain loop over
    (layer, rows, salience, elems, leader) records."""
    options = sorted(config.bit_options)
    total = sum(r[3] for r in recs)
    bits = [options[0]] * len(recs)
    current = sum(r[3] * options[0] for r in recs)
    target_total = config.target_bits * total
    order = sorted(range(len(recs)), key=lambda i: recs[i][2] / max(recs[i][3], 1), reverse=True)
    n_protect = max(1, int(config.protection_floor * len(recs)))
    floor_target = min(8, max(options))
    for i in order[:n_protect]:
        fb = max(bits[i], floor_target)
        if fb > bits[i] and fb in options:
            current += (fb - bits[i]) * recs[i][3]
            bits[i] = fb
    for i in order:
        for b in options:
            if b <= bits[i]:
                continue
            cost = (b - bits[i]) * recs[i][3]
            if current + cost <= target_total:
                current += cost
                bits[i] = b
            else:
                break
    return [(recs[i][0], recs[i][1], bits[i]) for i in order], current / max(total, 1)


@pytest.mark.parametrize("window", [65536, 7])
@pytest.mark.parametrize("seed", range(40))
def test_solver_scan_equals_sequential_greedy(seed, window, monkeypatch):
    """Random layers, clique sizes, ties, options, targets and floors: the
    scan gives the sequential greedy's bits, order and achieved bits (also
    with a 7-clique scan window, so runs cross window boundaries)."""
    from csaq import core
    from csaq.config import CSAQConfig
    from csaq.core import solve_clique_budget
    monkeypatch.setattr(core, "_SCAN_WINDOW", window)
    rng = np.random.default_rng(seed)
    all_opts = [[4, 8, 16], [2, 4, 8], [2, 4, 8, 16], [4, 8], [8, 16], [2, 16]]
    opts = all_opts[seed % len(all_opts)]
    lo, hi = min(opts), max(opts)
    target = float(rng.uniform(lo, hi)) if seed % 5 else float(lo)
    floor = [0.0, 0.05, 0.1, 0.3][seed % 4]
    sal, cliques = {}, {}
    for li in range(int(rng.integers(1, 5))):
        C, K = int(rng.integers(3, 300)), int(rng.choice([8, 64, 128, 512]))
        s = rng.random((C, 1)).astype(np.float32)
        if seed % 3 == 0:
            s = np.round(s * 4) / 4  # many ties
        sal[f"l{li}"] = torch.from_numpy(np.repeat(s, K, axis=1))
        perm = rng.permutation(C).tolist()
        cl, pos = [], 0
        while pos < C:
            n = int(rng.integers(1, 6)) if seed % 2 else 1
            cl.append(sorted(perm[pos:pos + n]))
            pos += n
        cliques[f"l{li}"] = cl
    cfg = CSAQConfig(target_bits=target, bit_options=opts, protection_floor=floor)
    budget, stats, act = solve_clique_budget(sal, cliques, cfg)
    # records in the reference's enumeration order: layers as given, cliques as listed
    by_key = {(c["layer"], tuple(c["rows"])): c for cl in budget.values() for c in cl}
    recs = [(name, c["rows"], c["salience"], c["elems"], c["leader"])
            for name, cl in cliques.items() for c in (by_key[(name, tuple(r))] for r in cl)]
    seq, act_seq = _sequential_budget(recs, cfg)
    got = {(c["layer"], tuple(c["rows"])): c["bits"] for cl in budget.values() for c in cl}
    assert {(l, tuple(r)): b for l, r, b in seq} == got
    # the per-layer lists follow the global density order
    order = [(l, tuple(r)) for l, r, _ in seq]
    for name, cl in budget.items():
        assert [(name, tuple(c["rows"])) for c in cl] == [k for k in order if k[0] == name]
    assert act == act_seq
    for bits in set(got.values()):
        assert stats[f"int{bits}"] == sum(c["elems"] for cl in budget.values() for c in cl if c["bits"] == bits)
