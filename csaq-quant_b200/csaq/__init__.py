"""csaq — Causal Salience-Aware Quantization, B200-native (sm_100a).

Drop-in for csaq-quant's public API; the quantised hot path runs in
``libcsaq_b200.so`` (hand-written sm_100a CUDA behind a C ABI).
"""

from .config import CSAQConfig
from .kernels import CSAQLinear, QuantizedWeight

__version__ = "0.5.9+b200.0.1"

__all__ = ["CSAQConfig", "CSAQLinear", "QuantizedWeight"]
