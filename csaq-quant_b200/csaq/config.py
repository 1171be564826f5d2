"""csaq.config — CSAQConfig, an HF ``PretrainedConfig`` with validated fields.

Same fields, defaults, validation and messages as csaq-quant's
``csaq/config.py:19-145``; registered with ``AutoConfig`` as ``"csaq"``.
"""

from __future__ import annotations

import warnings
from typing import List, Optional

from transformers import AutoConfig, PretrainedConfig

# Bit-widths with a storage format (csaq/config.py:16).
_SUPPORTED_BITS = frozenset({2, 4, 8, 16})


class CSAQConfig(PretrainedConfig):
    """Configuration for Causal Salience-Aware Quantization.

    Args mirror csaq/config.py:26-52: ``target_bits`` (average bits per
    weight), ``bit_options`` (subset of {2, 4, 8, 16}), ``clique_threshold``
    in [0, 2] (values > 1 force singleton cliques), ``auto_scale_memory``,
    ``speculative_lookahead``, ``speculative_temperature``, ``salience_alpha``
    (top-10 % activation mask at 1.0), ``protection_floor`` in [0, 1),
    ``group_size`` (-1 = per-channel), ``clique_mode`` ("jaccard" or
    "per_channel").
    """

    model_type: str = "csaq"
    quant_type: str = "csaq"

    def __init__(self, target_bits: float = 4.0, bit_options: Optional[List[int]] = None,
                 clique_threshold: float = 0.85, auto_scale_memory: bool = True,
                 speculative_lookahead: int = 4, speculative_temperature: float = 1.0,
                 salience_alpha: float = 1.0, protection_floor: float = 0.10, group_size: int = -1,
                 clique_mode: str = "jaccard", base_model_type: str = "",
                 base_model_name_or_path: str = "", **kwargs: object) -> None:
        super().__init__(**kwargs)
        self.base_model_type = base_model_type
        self.base_model_name_or_path = base_model_name_or_path

        if bit_options is None:
            bit_options = [4, 8, 16]
        unsupported = sorted(set(bit_options) - _SUPPORTED_BITS)
        if unsupported:
            warnings.warn(
                f"[CSAQConfig] bit_options contains unsupported widths {unsupported} — they "
                f"will be silently ignored.  Supported: {sorted(_SUPPORTED_BITS)}.", stacklevel=2)
            bit_options = [b for b in bit_options if b in _SUPPORTED_BITS]
        if not bit_options:
            raise ValueError("[CSAQConfig] No valid bit_options remain after filtering.  "
                             f"Choose from {sorted(_SUPPORTED_BITS)}.")
        bit_options = sorted(set(bit_options))

        lo, hi = float(min(bit_options)), float(max(bit_options))
        if not (lo <= target_bits <= hi):
            raise ValueError(f"[CSAQConfig] target_bits={target_bits} is outside the range "
                             f"[{lo}, {hi}] implied by bit_options={bit_options}.")
        if not (0.0 <= clique_threshold <= 2.0):
            raise ValueError("[CSAQConfig] clique_threshold must be in [0, 2]. "
                             "Values > 1.0 force singleton cliques (ablation mode).")
        if not (0.0 <= protection_floor < 1.0):
            raise ValueError("[CSAQConfig] protection_floor must be in [0, 1).")
        if clique_mode not in ("jaccard", "per_channel"):
            raise ValueError("[CSAQConfig] clique_mode must be 'jaccard' or 'per_channel'.")

        self.target_bits = target_bits
        self.bit_options = bit_options
        self.clique_threshold = clique_threshold
        self.auto_scale_memory = auto_scale_memory
        self.speculative_lookahead = speculative_lookahead
        self.speculative_temperature = speculative_temperature
        self.salience_alpha = salience_alpha
        self.protection_floor = protection_floor
        self.group_size = group_size
        self.clique_mode = clique_mode

    @property
    def min_bits(self) -> int:
        return min(self.bit_options)

    @property
    def max_bits(self) -> int:
        return max(self.bit_options)


AutoConfig.register("csaq", CSAQConfig)
