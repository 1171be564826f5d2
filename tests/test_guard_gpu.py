"""The checked build (libcsaq_b200_checked.so, CSAQ_LIB=checked).

A child process loads the checked library and:
* runs ordinary work (mixed linear through the GEMV at M = 1, 4 and the
  tcgen05 GEMM at M = 64; self-speculative decode of a tiny decoder) and finds
  no failed index test;
* hands each guarded kernel one out-of-range index (an output row equal to
  ldy, a cache position equal to Lmax) and finds it recorded with its site,
  value and bound.
Every buffer those calls could reach past the given bounds is allocated with
slack, so the calls stay inside their allocations even without the guards.
"""

import json
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r"""
import ctypes, json, sys
import torch
sys.path.insert(0, REPO); sys.path.insert(0, REPO + "/csaq-quant_b200"); sys.path.insert(0, REPO + "/tests")
from csaq import _lib
from csaq._lib import lib, check, tier_array, dtype_code
from csaq import _synthetic as syn
from csaq.kernels import CSAQLinear
L = lib()
dev = torch.device("cuda", 0)
torch.cuda.set_device(dev)
st = torch.cuda.current_stream().cuda_stream
res = {"checked": L.csaq_checked_build()}

def report():
    v = [ctypes.c_int64() for _ in range(4)]
    check(L.csaq_guard_report(*[ctypes.byref(x) for x in v]), "guard_report")
    check(L.csaq_guard_clear(), "guard_clear")
    return [x.value for x in v]

check(L.csaq_guard_clear(), "guard_clear")
# ordinary work
case = syn.mixed_linear(n=256, k=512, m=64, seed=0, dtype=torch.bfloat16)
lin = torch.nn.Linear(512, 256, bias=True, dtype=torch.bfloat16).to(dev)
lin.weight.data = case.W.to(dev)
layer = CSAQLinear.from_tiers(lin, case.tier_rows, group_size=128)
for m in (1, 4, 64):
    layer(case.X[:m].to(dev))
from test_runtime_gpu import _prompt, _quantized
from csaq.inference import CSAQInferenceEngine
model, cmap, _ = _quantized("tiny-llama", seed=3)
eng = CSAQInferenceEngine(model, cmap, verbose=False)
out, rep = eng.generate(_prompt(1, 20, model.config.vocab_size, seed=1), speculative=True, lookahead=4,
                        temperature=0.0, max_new_tokens=16)
torch.cuda.synchronize()
res["clean"] = report()

# an output row equal to ldy in one tier, through the GEMV (M = 1) and the GEMM (M = 64)
N, K = 256, 512
for tag, M in (("gemv", 1), ("gemm", 64)):
    y = torch.zeros(M + 1, N, dtype=torch.bfloat16, device=dev)  # one spare row
    descs = layer.gemv_descriptors(y[:M])
    bad = [d for d in descs if d.bits == 4][0]
    rows_bad = torch.full((bad.n_rows,), N, dtype=torch.int32, device=dev)
    bad.out_rows = rows_bad.data_ptr()
    for d in descs:
        d.bias = None
    arr = tier_array(descs)
    x = case.X[:M].to(dev)
    fn = L.csaq_qgemv if M < 32 else L.csaq_qgemm
    check(fn(arr, len(descs), K, x.data_ptr(), dtype_code(x.dtype), M, x.stride(0), st), tag)
    torch.cuda.synchronize()
    res[tag] = report()
    res[tag + "_spare_row_untouched"] = bool((y[M] == 0).all())

# a cache position equal to Lmax (rope) and one that runs past it (attention)
B, S, Hq, Hkv, D, Lmax = 1, 1, 2, 1, 128, 8
dt = torch.bfloat16
q = torch.randn(B * S, Hq * D, dtype=dt, device=dev)
k = torch.randn(B * S, Hkv * D, dtype=dt, device=dev)
v = torch.randn(B * S, Hkv * D, dtype=dt, device=dev)
cos = torch.ones(Lmax + 1, D, dtype=torch.float32, device=dev)
sin = torch.zeros(Lmax + 1, D, dtype=torch.float32, device=dev)
kc = torch.zeros(B, Hkv, Lmax + 64, D, dtype=dt, device=dev)
vc = torch.zeros(B, Hkv, Lmax + 64, D, dtype=dt, device=dev)
q_out = torch.empty(B * S, Hq * D, dtype=dt, device=dev)
pos0 = torch.tensor([Lmax], dtype=torch.int32, device=dev)
check(L.csaq_rope_kv(q.data_ptr(), q.stride(0), k.data_ptr(), k.stride(0), v.data_ptr(), v.stride(0),
                     pos0.data_ptr(), B, S, Hq, Hkv, D, cos.data_ptr(), sin.data_ptr(), q_out.data_ptr(),
                     kc.data_ptr(), vc.data_ptr(), Lmax, dtype_code(dt), st), "rope")
torch.cuda.synchronize()
res["rope"] = report()
res["rope_cache_untouched"] = bool((kc == 0).all() and (vc == 0).all())
pos0.fill_(Lmax - S + 1)
nf = L.csaq_attention_workspace_floats(B, S, Hq, Hkv, D, Lmax)
part = torch.zeros(nf + 4096, dtype=torch.float32, device=dev)
tickets = torch.zeros(B * Hkv, dtype=torch.int32, device=dev)
o = torch.zeros(B * S, Hq * D, dtype=dt, device=dev)
check(L.csaq_decode_attention(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), pos0.data_ptr(), B, S, Hq, Hkv, D,
                              Lmax, 0.088, part.data_ptr(), tickets.data_ptr(), o.data_ptr(), dtype_code(dt),
                              st), "attention")
torch.cuda.synchronize()
res["attn"] = report()
res["attn_tickets"] = tickets.tolist()
print("RESULT " + json.dumps(res))
"""


def test_checked_build_records_out_of_range_indices():
    lib_path = os.path.join(REPO, "csaq-quant_b200", "csaq", "lib", "libcsaq_b200_checked.so")
    if not os.path.exists(lib_path):
        pytest.fail("libcsaq_b200_checked.so is missing: run __graft_entry__.build()")
    env = dict(os.environ, CSAQ_LIB="checked")
    r = subprocess.run([sys.executable, "-c", f"REPO = {REPO!r}\n" + CHILD], capture_output=True, text=True,
                       timeout=600, env=env, cwd=REPO)
    assert r.returncode == 0, r.stderr[-3000:]
    line = [l for l in r.stdout.splitlines() if l.startswith("RESULT ")][-1]
    res = json.loads(line[len("RESULT "):])
    assert res["checked"] == 1
    assert res["clean"][0] == 0, res["clean"]
    for tag, site in (("gemv", 1), ("gemm", 2)):
        count, s, value, bound = res[tag]
        assert count >= 1 and s == site and value == 256 and bound == 256, (tag, res[tag])
        assert res[tag + "_spare_row_untouched"]
    count, s, value, bound = res["rope"]
    assert count >= 1 and s == 3 and value == 8 and bound == 8, res["rope"]
    assert res["rope_cache_untouched"]
    count, s, value, bound = res["attn"]
    assert count >= 1 and s == 4 and value == 8 and bound == 7, res["attn"]
    assert res["attn_tickets"] == [0]
