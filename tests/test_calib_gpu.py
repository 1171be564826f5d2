"""GPU calibration kernels against the reference's own results.

Goldens (tests/golden/calib_golden.npz, digests.json) come from the
reference's CausalProfiler: its forward-hook top-k masks
(csaq/core.py:143-155), its _build_cliques over injected mask histories
(csaq/core.py:240-287) and its fp32 salience arithmetic (csaq/core.py:204-210,
232-233). Masks, intersection counts, activation counts and cliques are
bit-exact; salience is within 1e-3 relative (and checked exact as well).
"""

import hashlib

import numpy as np
import pytest
import torch
import torch.nn as nn

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _sha(a):
    a = a.cpu().numpy() if isinstance(a, torch.Tensor) else np.asarray(a)
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def _unpack_mask(mh):
    """(n_tok, C) bool from a MaskHistory's channel-major bit words."""
    bits = mh.bits[:, : mh.words_used()].cpu().numpy().view(np.uint32)
    C, W = bits.shape
    b = (bits[:, :, None] >> np.arange(32, dtype=np.uint32)) & 1
    return b.reshape(C, W * 32)[:, : mh.n_tok].T.astype(bool)


def _labels(cliques, n):
    lab = np.full(n, -1, np.int64)
    for ci, c in enumerate(cliques):
        lab[np.asarray(c, np.int64)] = ci
    return lab


class _One(nn.Module):
    def __init__(self, cin, cout):
        super().__init__()
        self.fc = nn.Linear(cin, cout)


@pytest.mark.parametrize("case", range(5))
def test_topk_masks_match_reference_hook(cgold, case):
    """Per-token top-k masks (k = max(1, int(min(1, 0.1 alpha) C)), ties kept)."""
    from csaq.core import MaskHistory
    alpha, dt_code = cgold[f"tk{case}_meta"]
    dt = {0: torch.float32, 1: torch.float16, 2: torch.bfloat16}[int(dt_code)]
    out = torch.from_numpy(cgold[f"tk{case}_out"]).to(dt)
    C = out.shape[-1]
    k = max(1, int(min(1.0, 0.1 * float(alpha)) * C))
    mh = MaskHistory(C, torch.device(DEV))
    mh.append(out.to(DEV), mode=1, k=k)
    np.testing.assert_array_equal(_unpack_mask(mh), cgold[f"tk{case}_mask"])


def test_threshold_mask_and_counts_match_reference(cgold):
    """act > 0.5 masks appended in two batches; I = mask^T mask and f exact."""
    from csaq.core import MaskHistory, coactivation_counts
    act = torch.from_numpy(cgold["cl_act"]).to(DEV)
    mh = MaskHistory(96, torch.device(DEV))
    mh.append(act[:200], mode=0, thr=0.5)
    mh.append(act[200:], mode=0, thr=0.5)
    m = _unpack_mask(mh)  # the first batch is padded to 224 tokens with empty bits
    np.testing.assert_array_equal(np.concatenate([m[:200], m[224:]]), cgold["cl_mask"])
    assert not m[200:224].any()
    inter, f = coactivation_counts(mh.bits, mh.words_used())
    np.testing.assert_array_equal(inter.cpu().numpy(), cgold["cl_inter"])
    np.testing.assert_array_equal(f.cpu().numpy(), cgold["cl_f"])


@pytest.mark.parametrize("thr", [0.85, 0.6, 0.3, 0.0, 1.5])
def test_profiler_cliques_match_reference(cgold, thr):
    from csaq.config import CSAQConfig
    from csaq.core import CausalProfiler
    act = torch.from_numpy(cgold["cl_act"]).to(DEV)
    prof = CausalProfiler(_One(8, 96).to(DEV), CSAQConfig(clique_threshold=thr))
    prof.add_activation_masks("fc", act[:200], threshold=0.5)
    prof.add_activation_masks("fc", act[200:], threshold=0.5)
    cl = prof._build_cliques()["fc"]
    np.testing.assert_array_equal(_labels(cl, 96), cgold[f"cl_labels_{thr}"])
    np.testing.assert_array_equal(np.concatenate([np.asarray(c) for c in cl]), cgold[f"cl_flat_{thr}"])
    np.testing.assert_array_equal(np.asarray([len(c) for c in cl]), cgold[f"cl_len_{thr}"])


def test_per_channel_cliques(cgold):
    from csaq.config import CSAQConfig
    from csaq.core import CausalProfiler
    prof = CausalProfiler(_One(8, 96).to(DEV), CSAQConfig(clique_mode="per_channel"))
    cl = prof._build_cliques()["fc"]
    np.testing.assert_array_equal(np.asarray([len(c) for c in cl]), cgold["cl_perchannel_len"])


def test_salience_accumulation_matches_reference(cgold):
    from csaq._lib import check, lib, stream_of
    from csaq.core import salience_accumulate
    W = torch.from_numpy(cgold["sal_W"]).to(DEV)
    acc = torch.zeros(W.shape, dtype=torch.float32, device=DEV)
    for G in cgold["sal_G"]:
        salience_accumulate(acc, torch.from_numpy(G).to(DEV), W)
    check(lib().csaq_salience_finalize(acc.data_ptr(), acc.numel(), 3, stream_of(acc)), "finalize")
    ref = cgold["sal_ref"]
    got = acc.cpu().numpy()
    assert np.abs(got - ref).max() <= 1e-3 * np.abs(ref).max()
    np.testing.assert_array_equal(got, ref)  # same fp32 operations in the same order


def test_full_size_coactivation_digest(digests):
    """8192 tokens x 11008 channels (act > 0.5): counts and cliques hash to the reference's."""
    from csaq import _synthetic as syn
    from csaq.config import CSAQConfig
    from csaq.core import CausalProfiler, MaskHistory, coactivation_counts, jaccard_cliques
    d = digests["coact11008"]
    act = syn.activations(64 * 128, 11008, seed=0).to(DEV)
    mh = MaskHistory(11008, torch.device(DEV), capacity_tokens=8192)
    mh.append(act, mode=0, thr=0.5)
    inter, f = coactivation_counts(mh.bits, mh.words_used())
    assert _sha(f) == d["f_i32"]
    assert abs(float(f.double().sum()) / (8192 * 11008) - d["density"]) < 1e-6  # an fp32 mean there
    assert _sha(inter) == d["inter_i32"]
    for thr in (0.85, 0.6):
        cl = jaccard_cliques(inter, f, thr)
        assert len(cl) == d[f"n_cliques_{thr}"], thr
        assert _sha(_labels(cl, 11008)) == d[f"labels_{thr}"], thr


def _greedy_ref(rows, C):
    """Seed-order partition (csaq/core.py:268-285) over sparse adjacency rows:
    seed i takes itself and every unvisited j > i of its row."""
    visited = np.zeros(C, bool)
    lab = np.empty(C, np.int32)
    nid = 0
    for i in range(C):
        if visited[i]:
            continue
        mem = [j for j in rows[i] if j > i and not visited[j]] + [i]
        visited[mem] = True
        lab[mem] = nid
        nid += 1
    return lab, nid


@pytest.mark.parametrize("C,ld_pad,per_row", [(3000, 3, 6), (33, 0, 20), (40000, 0, 3)])
def test_greedy_cliques_on_arbitrary_adjacency(C, ld_pad, per_row):
    """csaq_greedy_cliques on random (asymmetric) adjacency bits, including a
    padded row stride and rows wider than one CTA (C > 32768)."""
    from csaq._lib import check, lib
    rng = np.random.default_rng(C)
    words = (C + 31) // 32
    ld = words + ld_pad
    rows = [np.unique(rng.integers(0, C, size=per_row)) for _ in range(C)]
    adj = np.zeros((C, ld), np.uint32)
    for i, r in enumerate(rows):
        np.bitwise_or.at(adj[i], r // 32, (np.uint32(1) << (r % 32).astype(np.uint32)))
    a = torch.from_numpy(adj.view(np.int32)).to(DEV)
    labels = torch.full((C,), -7, dtype=torch.int32, device=DEV)
    n = torch.zeros(1, dtype=torch.int32, device=DEV)
    check(lib().csaq_greedy_cliques(a.data_ptr(), ld, C, labels.data_ptr(), n.data_ptr(),
                                    torch.cuda.current_stream().cuda_stream), "greedy")
    ref, nid = _greedy_ref(rows, C)
    assert int(n.item()) == nid
    np.testing.assert_array_equal(labels.cpu().numpy(), ref)


def test_profile_end_to_end_tiny_decoder():
    """CausalProfiler.profile on a tiny Llama: salience is |G W| averaged over
    batches (checked against torch on the same grads) and cliques partition
    every layer's channels."""
    from csaq import _synthetic as syn
    from csaq.config import CSAQConfig
    from csaq.core import CausalProfiler
    model = syn.build_decoder("tiny-llama", device=DEV, seed=0, dtype=torch.float32)
    g = torch.Generator().manual_seed(3)
    calib = [{"input_ids": torch.randint(0, 2048, (1, 32), generator=g)} for _ in range(3)]
    ref = {}
    for b in calib:
        model.zero_grad()
        out = model(input_ids=b["input_ids"].to(DEV), labels=b["input_ids"].to(DEV))
        out.loss.backward()
        for n, m in model.named_modules():
            if isinstance(m, nn.Linear) and "lm_head" not in n:
                ref[n] = ref.get(n, 0) + (m.weight.grad.float() * m.weight.data.float()).abs()
    model.zero_grad()
    prof = CausalProfiler(model, CSAQConfig(clique_threshold=0.6, salience_alpha=1.0))
    sal, cliques = prof.profile(calib, verbose=False)
    for n, s in sal.items():
        if n in ref:
            r = (ref[n] / 3).cpu()
            assert torch.allclose(s.cpu(), r, rtol=1e-3, atol=1e-12), n
        C = s.shape[0]
        flat = sorted(i for c in cliques[n] for i in c)
        assert flat == list(range(C)), n


@pytest.mark.parametrize("group_size", [128, -1])
def test_quantize_end_to_end_tiny_decoder(group_size):
    """quantize(): profile -> solve -> apply on a tiny Llama; every quantisable
    linear becomes a CSAQLinear and the quantised logits track the
    full-precision ones."""
    from csaq import _synthetic as syn
    from csaq.config import CSAQConfig
    from csaq.core import quantize
    from csaq.kernels import CSAQLinear
    model = syn.build_decoder("tiny-llama", device=DEV, seed=1, dtype=torch.bfloat16)
    g = torch.Generator().manual_seed(4)
    ids = torch.randint(0, 2048, (2, 24), generator=g).to(DEV)
    with torch.no_grad():
        ref = model(input_ids=ids).logits.float()
    calib = [{"input_ids": torch.randint(0, 2048, (1, 32), generator=g)} for _ in range(4)]
    cfg = CSAQConfig(target_bits=4.0, bit_options=[4, 8, 16], group_size=group_size, clique_threshold=0.6)
    model, info = quantize(model, calib, cfg, verbose=False)
    n_lin = sum(isinstance(m, CSAQLinear) for m in model.modules())
    assert n_lin == 2 * 7
    # the protection floor (top 10 % of cliques at >= 8 bits) may lift the average above target
    assert 4.0 <= info["actual_bits"] <= 16.0
    with torch.no_grad():
        got = model(input_ids=ids).logits.float()
        # the same model with every CSAQLinear computed as F.linear on its dequantised weight
        saved = {}
        for m in model.modules():
            if isinstance(m, CSAQLinear):
                W = m._get_weight_fp32()
                saved[m] = m.forward
                m.forward = (lambda W_, b_: (lambda x: torch.nn.functional.linear(
                    x, W_.to(x.dtype), None if b_ is None else b_.to(x.dtype))))(W, m.bias)
        deq = model(input_ids=ids).logits.float()
        for m, f in saved.items():
            m.forward = f
    assert torch.isfinite(got).all()
    cos_deq = torch.nn.functional.cosine_similarity(got.flatten(), deq.flatten(), dim=0)
    assert cos_deq > 0.999, float(cos_deq)
    cos = torch.nn.functional.cosine_similarity(got.flatten(), ref.flatten(), dim=0)
    assert cos > 0.9, float(cos)  # 4-bit random weights: coarse, but the same function
