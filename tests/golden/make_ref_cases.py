"""Fixtures from csaq-quant v0.5.9 itself for the profiler's early stop and
the export format (run in the build container, where the reference source
tree is present; nothing here runs at test time):

    python tests/golden/make_ref_cases.py --ref <reference source tree>

Outputs (committed):
  tests/golden/profile_golden.npz  CausalProfiler.profile on TinyNet and 40
      calibration batches after torch.manual_seed(PROFILE_SEED): the early-stop
      batch (csaq/core.py:212-230), the salience and the cliques of fc1/fc2.
  tests/golden/export_golden.npz   a tiny Llama whose decoder linears are
      quantised at 4 bits by inject_csaq_linear (csaq/kernels.py:271-300),
      its weights and the quantised buffers, and the SHA-256 of the three
      files export_csaq_model (csaq/utils.py:225-318) writes.
"""

from __future__ import annotations

import argparse
import contextlib
import hashlib
import io
import os
import re
import shutil
import sys
import tempfile

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import tiny_nets as T  # noqa: E402


def _import_reference(ref_root: str):
    tmp = tempfile.mkdtemp(prefix="csaq_ref_")
    shutil.copytree(os.path.join(ref_root, "csaq"), os.path.join(tmp, "csaq"))
    sys.dont_write_bytecode = True
    sys.path.insert(0, tmp)
    import csaq  # noqa: F401,E402
    import csaq.config as rcfg  # noqa: E402
    import csaq.core as rc  # noqa: E402
    import csaq.kernels as rk  # noqa: E402
    import csaq.utils as ru  # noqa: E402
    return rcfg, rc, rk, ru


def profile_case(rcfg, rc) -> dict:
    model = T.tiny_net()
    out = {f"w_{k}": v.detach().numpy() for k, v in model.state_dict().items()}
    calib = T.calib_batches()
    out["calib_ids"] = np.stack([b["input_ids"].numpy() for b in calib])
    cfg = rcfg.CSAQConfig(clique_threshold=0.5)
    prof = rc.CausalProfiler(model, cfg)
    buf = io.StringIO()
    torch.manual_seed(T.PROFILE_SEED)
    with contextlib.redirect_stdout(buf):
        sal, cliques = prof.profile(calib, verbose=True)
    m = re.search(r"Early stop at batch (\d+)/", buf.getvalue())
    out["stop_batch"] = np.array([int(m.group(1)) if m else len(calib)], np.int64)
    for name in ("fc1", "fc2"):
        out[f"sal_{name}"] = sal[name].numpy()
        lab = np.full(sal[name].shape[0], -1, np.int64)
        for ci, c in enumerate(cliques[name]):
            lab[np.asarray(c, np.int64)] = ci
        out[f"labels_{name}"] = lab
        out[f"seeds_{name}"] = np.array([c[0] for c in cliques[name]], np.int64)
    return out


def export_case(rcfg, rk, ru) -> dict:
    model = T.tiny_llama()
    out = {f"w_{k}": v.detach().numpy() for k, v in model.state_dict().items()}
    budget = T.uniform_budget(model, 4)
    with contextlib.redirect_stdout(io.StringIO()):
        rk.inject_csaq_linear(model, budget, verbose=False)
    for k, v in model.state_dict().items():
        out[f"q_{k}"] = v.numpy()
    cfg = rcfg.CSAQConfig(target_bits=4.0, bit_options=[4, 8], group_size=-1)
    info = {"causal_map": {"model.layers.0.mlp.down_proj": [1, 5, 9]}, "tier_stats": {"int4": 1234},
            "actual_bits": 4.0, "cliques_count": 7}
    d = tempfile.mkdtemp(prefix="csaq_export_")
    with contextlib.redirect_stdout(io.StringIO()):
        ru.export_csaq_model(model, cfg, budget, d, info)
    for f in ("config.json", "csaq_manifest.json", "model.safetensors", "tokenizer_config.json"):
        with open(os.path.join(d, f), "rb") as fh:
            out[f"sha_{f}"] = np.frombuffer(hashlib.sha256(fh.read()).digest(), np.uint8)
    out["torch"] = np.frombuffer(torch.__version__.encode(), np.uint8)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="the csaq-quant v0.5.9 source tree (read only)")
    args = ap.parse_args()
    rcfg, rc, rk, ru = _import_reference(args.ref)
    np.savez_compressed(os.path.join(HERE, "profile_golden.npz"), **profile_case(rcfg, rc))
    np.savez_compressed(os.path.join(HERE, "export_golden.npz"), **export_case(rcfg, rk, ru))
    print("fixtures written; torch", torch.__version__)


if __name__ == "__main__":
    main()
