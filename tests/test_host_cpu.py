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
