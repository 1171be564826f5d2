"""CausalProfiler.profile (csaq/core.py:109-287) against the reference run on
the same tiny net and calibration batches (tests/golden/profile_golden.npz,
written by tests/golden/make_ref_cases.py from csaq-quant itself): the
Spearman early stop fires at the same batch (csaq/core.py:212-230), the
salience agrees within 1e-3 relative and the cliques are identical."""

import contextlib
import io
import os
import re
import sys

import numpy as np
import pytest
import torch

from _tol import SALIENCE_RTOL

pytestmark = pytest.mark.gpu

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def test_profile_matches_reference_early_stop_salience_cliques():
    if HERE not in sys.path:
        sys.path.insert(0, HERE)
    import tiny_nets
    from csaq.config import CSAQConfig
    from csaq.core import CausalProfiler
    g = np.load(os.path.join(HERE, "profile_golden.npz"))
    model = tiny_nets.tiny_net()
    model.load_state_dict({k[2:]: torch.from_numpy(g[k]) for k in g.files if k.startswith("w_")})
    model = model.cuda()
    calib = [{"input_ids": torch.from_numpy(ids)} for ids in g["calib_ids"]]
    prof = CausalProfiler(model, CSAQConfig(clique_threshold=0.5))
    buf = io.StringIO()
    torch.manual_seed(tiny_nets.PROFILE_SEED)
    with contextlib.redirect_stdout(buf):
        sal, cliques = prof.profile(calib, verbose=True)
    m = re.search(r"Early stop at batch (\d+)/", buf.getvalue())
    stop = int(m.group(1)) if m else len(calib)
    assert stop == int(g["stop_batch"][0]), buf.getvalue()
    for name in ("fc1", "fc2"):
        s, ref = sal[name].float().cpu().numpy(), g[f"sal_{name}"]
        rel = np.abs(s - ref).max() / np.abs(ref).max()
        assert rel <= SALIENCE_RTOL, (name, rel)
        lab = np.full(ref.shape[0], -1, np.int64)
        for ci, c in enumerate(cliques[name]):
            lab[np.asarray(c, np.int64)] = ci
        np.testing.assert_array_equal(lab, g[f"labels_{name}"])
        np.testing.assert_array_equal(np.array([c[0] for c in cliques[name]]), g[f"seeds_{name}"])
