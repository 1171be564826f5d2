"""Decode runtime and self-speculative engine on tiny random-init decoders.

* The runtime's logits (fused sm_100a kernels, static KV cache) match the HF
  forward of the same quantised model (HF attention/norms, CSAQLinear GEMV)
  within a bf16-level tolerance.
* Greedy self-speculative decoding returns exactly the tokens of greedy
  decoding with the verify weights, for one and for several sequences.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _quantized(name, seed=0):
    from csaq import _synthetic as syn
    from csaq.config import CSAQConfig
    from csaq.core import apply_csaq, solve_clique_budget
    model = syn.build_decoder(name, device=DEV, seed=seed)
    sal = syn.synthetic_salience(model, seed=seed + 1)
    cfg = CSAQConfig(target_bits=4.0, bit_options=[4, 8, 16], group_size=128, protection_floor=0.1)
    cliques = {n: [[i] for i in range(s.shape[0])] for n, s in sal.items()}
    budget, stats, actual = solve_clique_budget(sal, cliques, cfg)
    cmap = apply_csaq(model, budget, sal, cfg, verbose=False)
    return model, cmap, actual


@pytest.fixture(scope="module")
def tiny_llama():
    return _quantized("tiny-llama")


@pytest.fixture(scope="module")
def tiny_qwen2():
    return _quantized("tiny-qwen2", seed=5)


@pytest.fixture(scope="module")
def tiny_qwen2_d64():
    """64-wide heads (hidden 256, 4 heads), the head width of Qwen1.5-0.5B."""
    return _quantized("tiny-qwen2-d64", seed=6)


def _prompt(B, P, V, seed=0):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, V, (B, P), generator=g)


@pytest.mark.parametrize("which", ["tiny_llama", "tiny_qwen2", "tiny_qwen2_d64"])
@pytest.mark.parametrize("verify", [False, True])
def test_runtime_logits_match_hf(which, verify, request):
    from csaq.inference import CSAQInferenceEngine
    model, cmap, _ = request.getfixturevalue(which)
    V = model.config.vocab_size
    prompt = _prompt(1, 70, V, seed=3)
    eng = CSAQInferenceEngine(model, cmap, verbose=False)
    rt = eng.runtime(1, 256, 4)
    rt.reset(prompt.to(DEV), max_new=4, verify=verify)  # one prefill chunk (fused attention)
    got = rt.prefill_logits.float()
    rt.prefill_chunk = 32
    rt.reset(prompt.to(DEV), max_new=4, verify=verify)  # 32 + 32 (fused attention, causal / offset mask) + 6
    got2 = rt.prefill_logits.float()
    rt.prefill_chunk = 16
    rt.reset(prompt.to(DEV), max_new=4, verify=verify)  # 16-token chunks: decode attention kernel
    got3 = rt.prefill_logits.float()
    rt.prefill_chunk = 512
    (eng._swap_to_verify if verify else eng._swap_to_draft)()
    with torch.no_grad():
        ref = model(prompt.to(DEV)).logits[:, -1].float()
    eng._swap_to_draft()
    for g in (got, got2, got3):
        err = (g - ref).abs().max().item() / ref.abs().max().item()
        assert err < 3e-2, err
        cos = torch.nn.functional.cosine_similarity(g, ref).item()
        assert cos > 0.999, cos


def test_verify_weights_differ_from_draft(tiny_llama):
    from csaq.inference import CSAQInferenceEngine
    model, cmap, _ = tiny_llama
    eng = CSAQInferenceEngine(model, cmap, verbose=False)
    assert eng._hooks, "quantised layers must register protected rows"
    rt = eng.runtime(1, 256, 4)
    prompt = _prompt(1, 20, model.config.vocab_size, seed=4).to(DEV)
    rt.reset(prompt, 4, verify=True)
    a = rt.prefill_logits.clone()
    rt.reset(prompt, 4, verify=False)
    b = rt.prefill_logits.clone()
    assert (a - b).abs().max() > 0


@pytest.mark.parametrize("which,B,K", [("tiny_llama", 1, 4), ("tiny_llama", 3, 4), ("tiny_llama", 2, 2),
                                       ("tiny_llama", 16, 4), ("tiny_qwen2_d64", 2, 4)])
def test_speculative_equals_greedy_verify(which, B, K, request):
    from csaq.inference import CSAQInferenceEngine
    model, cmap, _ = request.getfixturevalue(which)
    V = model.config.vocab_size
    prompt = _prompt(B, 33, V, seed=7 + B)
    eng = CSAQInferenceEngine(model, cmap, verbose=False)
    out, rep = eng.generate(prompt, speculative=True, lookahead=K, temperature=0.0, max_new_tokens=40)
    assert out.shape == (B, 33 + 40)
    assert rep.mode == "speculative" and rep.verify_calls > 0
    assert 0.0 <= rep.acceptance_rate <= 1.0
    rt = eng.runtime(B, 33 + 40 + 2 * K + 2, K)
    rt.reset(prompt.to(DEV), 40, verify=True)
    rt.generate_greedy(40, verify=True)
    greedy = rt.outputs()[:, :40].cpu()
    assert torch.equal(out[:, 33:].cpu(), greedy)


def test_standard_generate_shape(tiny_llama):
    from csaq.inference import CSAQInferenceEngine
    model, cmap, _ = tiny_llama
    eng = CSAQInferenceEngine(model, cmap, verbose=False)
    prompt = _prompt(1, 8, model.config.vocab_size, seed=1)
    out, rep = eng.generate(prompt, speculative=False, temperature=0.0, max_new_tokens=6)
    assert out.shape == (1, 14)
    assert rep.mode == "standard" and rep.tokens_generated == 6


def test_general_path_speculative_runs(tiny_qwen2):
    """Sampling uses the HF-forward loop with the same verify/draft weights."""
    from csaq.inference import CSAQInferenceEngine
    model, cmap, _ = tiny_qwen2
    eng = CSAQInferenceEngine(model, cmap, verbose=False)
    prompt = _prompt(1, 12, model.config.vocab_size, seed=2).to(DEV)
    torch.manual_seed(0)
    out, rep = eng.generate(prompt, speculative=True, lookahead=3, temperature=0.8, max_new_tokens=10)
    assert out.shape[1] == 22
    assert rep.tokens_generated == 10 and rep.verify_calls >= 1
