"""The reference-facing Python API on the CPU: module paths and names,
CSAQConfig validation (csaq/config.py:19-145), the unsupported-bits
ValueError raised before any device work (csaq/kernels.py:488-492, 569, 600),
the SpeculativeReport arithmetic (csaq/inference.py:37-111), and the
calibration-data, perplexity and report helpers (csaq/utils.py:25-218)."""

import math
import warnings

import pytest
import torch


def test_reference_names_importable():
    import csaq.core as core
    import csaq.inference as inference
    import csaq.kernels as kernels
    import csaq.modeling as modeling
    import csaq.utils as utils
    from csaq.config import CSAQConfig  # noqa: F401
    for name in ("QuantizedWeight", "quantize_per_channel", "quantize_shared_scale", "_pack", "_unpack",
                 "_dequantize", "_float_to_int", "inject_csaq_linear", "CSAQLinear"):
        assert hasattr(kernels, name), name
    for name in ("CausalProfiler", "solve_clique_budget", "apply_csaq", "quantize"):
        assert hasattr(core, name), name
    for name in ("CSAQInferenceEngine", "SpeculativeReport"):
        assert hasattr(inference, name), name
    assert hasattr(utils, "export_csaq_model")
    assert hasattr(modeling, "CSAQModelForCausalLM")
    lin = kernels.CSAQLinear(64, 32, bits=4)
    for buf in ("weight_packed", "weight_scales", "weight_zp"):
        assert buf in dict(lin.named_buffers()), buf
    assert lin.weight_packed.dtype == torch.uint8 and lin.weight_packed.shape == (32, 32)
    assert lin.weight_scales.dtype == torch.float32 and lin.weight_zp.dtype == torch.int32


def test_config_defaults_and_properties():
    from csaq.config import CSAQConfig
    c = CSAQConfig()
    assert (c.target_bits, c.bit_options, c.clique_threshold) == (4.0, [4, 8, 16], 0.85)
    assert (c.protection_floor, c.group_size, c.clique_mode) == (0.10, -1, "jaccard")
    assert (c.min_bits, c.max_bits) == (4, 16)
    assert CSAQConfig(target_bits=4.0, bit_options=[16, 8, 4, 8]).bit_options == [4, 8, 16]
    d = CSAQConfig(target_bits=3.0, bit_options=[2, 4], group_size=128).to_dict()
    assert d["model_type"] == "csaq" and d["bit_options"] == [2, 4] and d["group_size"] == 128


def test_config_registered_with_autoconfig():
    from transformers import AutoConfig
    from csaq.config import CSAQConfig
    assert isinstance(AutoConfig.for_model("csaq", target_bits=8.0, bit_options=[8, 16]), CSAQConfig)


def test_config_validation():
    from csaq.config import CSAQConfig
    with pytest.warns(UserWarning, match="unsupported widths"):
        c = CSAQConfig(target_bits=4.0, bit_options=[3, 4, 8])
    assert c.bit_options == [4, 8]
    with pytest.warns(UserWarning):
        with pytest.raises(ValueError, match="No valid bit_options"):
            CSAQConfig(target_bits=2.0, bit_options=[1, 3])
    with pytest.raises(ValueError, match="target_bits"):
        CSAQConfig(target_bits=17.0)
    with pytest.raises(ValueError, match="target_bits"):
        CSAQConfig(target_bits=2.0, bit_options=[4, 8])
    for bad in (-0.01, 2.01):
        with pytest.raises(ValueError, match="clique_threshold"):
            CSAQConfig(clique_threshold=bad)
    assert CSAQConfig(clique_threshold=2.0).clique_threshold == 2.0  # singleton ablation
    for bad in (-0.1, 1.0):
        with pytest.raises(ValueError, match="protection_floor"):
            CSAQConfig(protection_floor=bad)
    with pytest.raises(ValueError, match="clique_mode"):
        CSAQConfig(clique_mode="spectral")
    with warnings.catch_warnings():
        warnings.simplefilter("error")
        CSAQConfig(target_bits=16.0, bit_options=[16])


def test_unsupported_bits_raise_value_error_before_device_work():
    from csaq.kernels import _pack, _unpack, quantize_per_channel, quantize_shared_scale
    q = torch.zeros(2, 8, dtype=torch.int32)
    for bits in (1, 3, 16):
        with pytest.raises(ValueError):
            _pack(q, bits)
    with pytest.raises(ValueError):
        _unpack(torch.zeros(2, 4, dtype=torch.uint8), 5, 2, 8)
    W = torch.randn(4, 8)
    with pytest.raises(ValueError):
        quantize_per_channel(W, 3)
    with pytest.raises(ValueError):
        quantize_shared_scale(W, W[0], 6)


def test_speculative_report_arithmetic():
    from csaq.inference import SpeculativeReport
    r = SpeculativeReport(tokens_generated=40, tokens_accepted=24, tokens_rejected=8, draft_calls=32,
                          verify_calls=8, total_wallclock_s=0.5)
    assert r.acceptance_rate == pytest.approx(0.75)
    assert r.speedup_factor == pytest.approx(1.0)
    assert r.inter_token_latency_ms == pytest.approx(12.5)
    assert r.block_efficiency == pytest.approx(3.0)
    assert r.tokens_per_second == pytest.approx(80.0)
    assert math.isnan(r.p95_latency_ms)
    s = r.summary()
    assert s["mode"] == "speculative" and s["p95_latency_ms"] == "nan" and s["tokens_per_second"] == 80.0
    empty = SpeculativeReport()
    assert empty.acceptance_rate == 0.0 and empty.tokens_per_second == 0.0


class _Encoding(dict):
    """A dict whose keys also read as attributes, like HF's BatchEncoding."""

    def __getattr__(self, k):
        return self[k]


class _FakeTokenizer:
    """Characters -> ids, with the HF call signature the helpers use."""

    def __call__(self, text, return_tensors="pt", max_length=None, truncation=False, padding=None):
        ids = [ord(c) % 97 + 1 for c in text]
        if truncation and max_length is not None:
            ids = ids[:max_length]
        mask = [1] * len(ids)
        if padding == "max_length" and max_length is not None:
            mask += [0] * (max_length - len(ids))
            ids += [0] * (max_length - len(ids))

        return _Encoding(input_ids=torch.tensor([ids]), attention_mask=torch.tensor([mask]))


def test_calibration_data_and_report(tmp_path):
    import json
    from csaq.utils import build_calibration_data, generate_csaq_report
    with pytest.raises(ValueError, match="custom_texts is empty"):
        build_calibration_data(_FakeTokenizer(), [])
    with pytest.warns(UserWarning, match="Only 3 calibration samples"):
        batches = build_calibration_data(_FakeTokenizer(), ["abc", "a much longer sentence here", "x"], seq_len=8)
    assert len(batches) == 3 and all(b["input_ids"].shape == (1, 8) for b in batches)
    assert int(batches[0]["attention_mask"].sum()) == 3 and int(batches[1]["attention_mask"].sum()) == 8
    assert len(build_calibration_data(_FakeTokenizer(), ["t"] * 20, n=16)) == 16
    info = {"tier_stats": {"int4": 300, "int8": 100}, "actual_bits": 5.0, "cliques_count": 12, "elapsed_s": 1.234}
    rep = generate_csaq_report(info, str(tmp_path / "r" / "CSAQ_Report.json"))
    assert rep["bit_distribution_pct"] == {"int4": 75.0, "int8": 25.0}
    assert rep["total_quantized_params"] == 400 and rep["ppl"] == "not_computed"
    assert json.load(open(tmp_path / "r" / "CSAQ_Report.json")) == rep


def test_perplexity_on_a_cpu_model():
    from csaq.utils import compute_perplexity

    class _Uniform(torch.nn.Module):
        """Uniform logits over 100 tokens: the loss is ln(100) for any input."""

        def __init__(self):
            super().__init__()
            self.w = torch.nn.Parameter(torch.zeros(1))

        def forward(self, ids, labels=None):
            logits = torch.zeros(ids.shape[0], ids.shape[1], 100) + self.w
            loss = torch.nn.functional.cross_entropy(logits[:, :-1].reshape(-1, 100), labels[:, 1:].reshape(-1))

            class _Out:
                pass
            o = _Out()
            o.loss = loss
            return o

    ppl = compute_perplexity(_Uniform(), _FakeTokenizer(), ["some evaluation text"] * 3, seq_len=16, stride=8)
    assert ppl == pytest.approx(100.0, rel=1e-5)
    with pytest.raises(ValueError):
        compute_perplexity(_Uniform(), _FakeTokenizer(), [])
