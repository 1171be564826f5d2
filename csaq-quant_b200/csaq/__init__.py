"""csaq — Causal Salience-Aware Quantization, B200-native (sm_100a).

Drop-in for csaq-quant's public API; the quantised hot path runs in
``libcsaq_b200.so`` (hand-written sm_100a CUDA behind a C ABI)::

    from csaq import quantize, CSAQConfig, build_calibration_data, CSAQInferenceEngine

    config = CSAQConfig(target_bits=4.0, bit_options=[4, 8, 16], group_size=128)
    model, info = quantize(model.cuda(), build_calibration_data(tokenizer, texts), config=config)
    engine = CSAQInferenceEngine(model, info["causal_map"], tokenizer)
    output, report = engine.generate(input_ids, max_new_tokens=256, speculative=True, lookahead=4)
"""

from .config import CSAQConfig
from .core import CausalProfiler, apply_csaq, quantize, solve_clique_budget
from .inference import CSAQInferenceEngine, SpeculativeReport
from .kernels import CSAQLinear, QuantizedWeight
from .modeling import CSAQModelForCausalLM
from .utils import build_calibration_data, compute_perplexity, export_csaq_model, generate_csaq_report

__version__ = "0.5.9+b200.0.1"

__all__ = [
    "CSAQConfig", "CausalProfiler", "apply_csaq", "quantize", "solve_clique_budget",
    "CSAQInferenceEngine", "SpeculativeReport", "CSAQLinear", "QuantizedWeight",
    "CSAQModelForCausalLM", "build_calibration_data", "compute_perplexity", "export_csaq_model",
    "generate_csaq_report",
]
