"""On-device sampling at temperature > 0 (csaq/inference.py:269-304 `_sample`,
:482-518 the rejection-sampling accept), checked by distribution.

* csaq_sample_rows: many identical rows draw independent tokens whose counts
  match softmax(clamp(logits) / T) (chi-square), and with top_p < 1 only the
  tokens the reference's sort-and-cumsum rule keeps are drawn.
* csaq_spec_sample_verify: speculative sampling emits tokens distributed as the
  verify distribution whatever the draft distribution (the rejection-sampling
  identity), for many sequences in one launch.
* The runtime: speculative sampling at T = 0.9, top_p = 0.9 runs on the device,
  and a seed reproduces its sequence.
"""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _chi2(counts, probs):
    exp = probs * counts.sum()
    keep = exp > 5
    return float((((counts - exp) ** 2) / np.maximum(exp, 1e-12))[keep].sum()), int(keep.sum()) - 1


def _ref_probs(logits, T, top_p):
    """The reference's _sample distribution (csaq/inference.py:269-304), in torch on the CPU."""
    z = torch.nan_to_num(torch.clamp(logits, -50.0, 50.0), nan=0.0, posinf=50.0, neginf=-50.0) / max(T, 1e-8)
    if top_p < 1.0:
        sl, si = torch.sort(z, descending=True)
        sp = torch.softmax(sl, dim=-1)
        remove = torch.cumsum(sp, dim=-1) - sp > top_p
        sl[remove] = float("-inf")
        z = torch.zeros_like(z).scatter(0, si, sl)
    return torch.softmax(z, dim=-1).double().numpy()


@pytest.mark.parametrize("T,top_p", [(1.0, 1.0), (0.7, 1.0), (1.0, 0.5)])
def test_sample_rows_distribution(T, top_p):
    from csaq._lib import check, lib
    V, rows = 64, 60000
    g = torch.Generator().manual_seed(3)
    logits = torch.randn(V, generator=g) * 2.0
    x = logits.repeat(rows, 1).to(DEV)
    out = torch.empty(rows, dtype=torch.int64, device=DEV)
    ctr = torch.zeros(2, dtype=torch.int64, device=DEV)
    st = torch.cuda.current_stream().cuda_stream
    check(lib().csaq_sample_rows(x.data_ptr(), 1, 0, V, V, rows, T, top_p, 1234, ctr.data_ptr(), out.data_ptr(), 0, st),
          "sample")
    torch.cuda.synchronize()
    assert int(ctr[0]) == 1 and int(ctr[1]) == 0  # the call counter advanced once
    toks = out.cpu().numpy()
    p = _ref_probs(logits, T, top_p)
    assert set(np.unique(toks)) <= set(np.nonzero(p > 0)[0])
    chi2, dof = _chi2(np.bincount(toks, minlength=V).astype(np.float64), p)
    assert chi2 < dof + 6 * np.sqrt(2 * dof), (chi2, dof)


def test_sample_rows_across_vocabulary_slices():
    """Tensor-parallel layout: each row is two vocabulary slices, rows*V/2 apart."""
    from csaq._lib import check, lib
    V, rows, W = 40, 40000, 2
    g = torch.Generator().manual_seed(5)
    logits = torch.randn(V, generator=g)
    parts = logits.view(W, 1, V // W).repeat(1, rows, 1).contiguous().to(DEV)  # (W, rows, V/W)
    out = torch.empty(rows, dtype=torch.int64, device=DEV)
    ctr = torch.zeros(2, dtype=torch.int64, device=DEV)
    st = torch.cuda.current_stream().cuda_stream
    check(lib().csaq_sample_rows(parts.data_ptr(), W, rows * (V // W), V // W, V // W, rows, 1.0, 1.0, 7,
                                 ctr.data_ptr(), out.data_ptr(), 0, st), "sample")
    torch.cuda.synchronize()
    chi2, dof = _chi2(np.bincount(out.cpu().numpy(), minlength=V).astype(np.float64), _ref_probs(logits, 1.0, 1.0))
    assert chi2 < dof + 6 * np.sqrt(2 * dof), (chi2, dof)


def test_spec_sample_emits_the_verify_distribution():
    from csaq._lib import check, lib
    V, B, K, T = 48, 40000, 1, 0.8
    g = torch.Generator().manual_seed(11)
    d = torch.randn(V, generator=g) * 1.5
    v = torch.randn(V, generator=g) * 1.5
    pd = torch.softmax(d / T, dim=-1).double().numpy()
    pv = torch.softmax(v / T, dim=-1).double().numpy()
    rng = np.random.default_rng(0)
    draft = torch.from_numpy(rng.choice(V, size=(B, K), p=pd / pd.sum())).to(DEV)
    dlog = d.view(1, 1, V).repeat(K, B, 1).contiguous().to(DEV)
    vlog = v.view(1, 1, V).repeat(B, K + 1, 1).contiguous().to(DEV)  # rows b*(K+1)+k
    vt = torch.full((B, K + 1), -1, dtype=torch.int64, device=DEV)
    ctr = torch.zeros(2, dtype=torch.int64, device=DEV)
    st = torch.cuda.current_stream().cuda_stream
    check(lib().csaq_spec_sample_verify(draft.data_ptr(), dlog.data_ptr(), vlog.data_ptr(), 1, 0, V, V, B, K, T,
                                        1.0, 99, ctr.data_ptr(), vt.data_ptr(), 0, st), "spec_sample")
    torch.cuda.synchronize()
    first = vt[:, 0].cpu().numpy()
    assert first.min() >= 0 and first.max() < V
    chi2, dof = _chi2(np.bincount(first, minlength=V).astype(np.float64), pv)
    assert chi2 < dof + 6 * np.sqrt(2 * dof), (chi2, dof)
    # a rejected draft token is never re-emitted
    acc = (vt[:, 0] == draft[:, 0]).cpu().numpy()
    ratio = np.minimum(1.0, pv[draft[:, 0].cpu().numpy()] / pd[draft[:, 0].cpu().numpy()])
    assert abs(acc.mean() - ratio.mean()) < 0.01


def test_runtime_speculative_sampling():
    """Sampled self-speculative decoding through the engine's fast path: valid
    tokens, consistent accept statistics, and the same seed drawing the same
    sequence (every random number comes from the device counter)."""
    from test_runtime_gpu import _prompt, _quantized
    from csaq.inference import CSAQInferenceEngine
    model, cmap, _ = _quantized("tiny-llama", seed=2)
    eng = CSAQInferenceEngine(model, cmap, verbose=False)
    prompt = _prompt(1, 24, model.config.vocab_size, seed=9)
    hot, rep = eng.generate(prompt, speculative=True, lookahead=4, temperature=0.9, top_p=0.9, max_new_tokens=20,
                            seed=6)
    assert rep.mode == "speculative"
    assert hot.shape == (1, 44)
    assert torch.equal(hot[:, :24].cpu(), prompt)
    assert int(hot.min()) >= 0 and int(hot.max()) < model.config.vocab_size
    assert rep.verify_calls >= 1 and rep.tokens_accepted + rep.tokens_rejected == rep.verify_calls * 4
    hot2, _ = eng.generate(prompt, speculative=True, lookahead=4, temperature=0.9, top_p=0.9, max_new_tokens=20,
                           seed=6)
    assert torch.equal(hot, hot2)  # the same seed draws the same numbers
    other, _ = eng.generate(prompt, speculative=True, lookahead=4, temperature=0.9, top_p=0.9, max_new_tokens=20,
                            seed=7)
    assert not torch.equal(hot, other)
