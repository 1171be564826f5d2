"""Loading exported csaq models (the reference's csaq/modeling.py:15-87).

``CSAQModelForCausalLM`` rebuilds the base architecture, swaps every linear
listed in csaq_manifest.json for an empty ``CSAQLinear`` of the recorded
layout (``layer_bits`` for uniform layers; ``layer_tiers`` for mixed-row
layers), and loads model.safetensors into it. The base architecture comes
from the base model config embedded in the exported config.json (no download),
or, when that is unusable, from ``AutoConfig.from_pretrained`` of
``base_model_name_or_path`` as the reference does.
"""

from __future__ import annotations

import json
import os
from typing import Any, Dict, Optional

import torch
import torch.nn as nn
from transformers import AutoConfig, AutoModelForCausalLM, PreTrainedModel

from .config import CSAQConfig
from .kernels import CSAQLinear

_QUANT_KEYS = {"target_bits", "bit_options", "clique_threshold", "auto_scale_memory", "speculative_lookahead",
               "speculative_temperature", "salience_alpha", "protection_floor", "group_size", "clique_mode",
               "base_model_type", "base_model_name_or_path", "quant_type", "csaq_version", "model_type"}


def _read_manifest(path: str) -> Dict[str, Any]:
    mp = os.path.join(path, "csaq_manifest.json")
    if not os.path.exists(mp):
        raise FileNotFoundError(f"[CSAQ] csaq_manifest.json not found in {path}.")
    with open(mp, "r", encoding="utf-8") as f:
        return json.load(f)


def _base_config(config: CSAQConfig):
    base_type = getattr(config, "base_model_type", "") or ""
    fields = {k: v for k, v in config.to_dict().items() if k not in _QUANT_KEYS}
    if base_type and base_type not in ("unknown", "csaq"):
        try:
            return AutoConfig.for_model(base_type, **fields)
        except Exception:
            pass
    name = getattr(config, "base_model_name_or_path", "")
    if not name or name == "unknown":
        raise ValueError("[CSAQ] base_model_name_or_path is missing in config.")
    return AutoConfig.from_pretrained(name, trust_remote_code=True)


def _parent_of(root: nn.Module, name: str):
    parent_name, _, child = name.rpartition(".")
    parent = root.get_submodule(parent_name) if parent_name else root
    return parent, child


class CSAQModelForCausalLM(PreTrainedModel):
    config_class = CSAQConfig
    base_model_prefix = "model"

    def __init__(self, config: CSAQConfig, manifest: Optional[Dict[str, Any]] = None):
        super().__init__(config)
        self.csaq_config = config
        self.model = AutoModelForCausalLM.from_config(_base_config(config))
        if manifest is None:
            manifest = _read_manifest(config.name_or_path)
        layer_bits = manifest.get("layer_bits", {})
        if not layer_bits:
            raise ValueError("[CSAQ] No layer_bits mapping found in csaq_manifest.json.")
        tiers = manifest.get("layer_tiers", {})
        gs = int(manifest.get("group_size", getattr(config, "group_size", -1)))
        for name, bits in layer_bits.items():
            try:
                parent, child = _parent_of(self.model, name)
            except AttributeError:
                continue
            lin = getattr(parent, child, None)
            if not isinstance(lin, nn.Linear):
                continue
            if name in tiers:
                layer = CSAQLinear.empty_tiers(lin.in_features, lin.out_features,
                                               {int(b): int(n) for b, n in tiers[name].items()},
                                               group_size=gs if gs > 0 else 128, bias=lin.bias)
            else:
                layer = CSAQLinear(lin.in_features, lin.out_features, int(bits), bias=lin.bias, group_size=gs)
            setattr(parent, child, layer)
        self._verify_layers = list(manifest.get("verify_layers", []))

    @classmethod
    def from_pretrained(cls, path: str, device: Optional[str] = None, dtype: Optional[torch.dtype] = None,
                        **_: Any) -> "CSAQModelForCausalLM":
        """Load an export_csaq_model directory (strict: every key must match)."""
        import safetensors.torch
        with open(os.path.join(path, "config.json"), "r", encoding="utf-8") as f:
            cfg_dict = json.load(f)
        cfg_dict.pop("model_type", None)
        config = CSAQConfig(**cfg_dict)
        config.name_or_path = path
        manifest = _read_manifest(path)
        model = cls(config, manifest)
        state = safetensors.torch.load_file(os.path.join(path, "model.safetensors"))
        verify = {}
        for name in model._verify_layers:
            verify[name] = (state.pop(f"{name}.verify_rows"), state.pop(f"{name}.verify_fp16"))
        if dtype is None:  # the dtype the floating parameters were saved in
            names = {n for n, _ in model.model.named_parameters()}
            dtype = next((v.dtype for k, v in state.items() if k in names and v.is_floating_point()), None)
        missing, unexpected = model.model.load_state_dict(state, strict=False)
        missing = [k for k in missing if not k.endswith(("_csaq_fp16_backup", "_csaq_hi_rows", "_csaq_quant_stash"))]
        if missing or unexpected:
            raise RuntimeError(f"[CSAQ] state dict mismatch: missing {missing[:8]}, unexpected {unexpected[:8]}")
        if dtype is not None:
            for p in model.model.parameters():
                p.data = p.data.to(dtype)
            for m in model.model.modules():
                if isinstance(m, CSAQLinear) and m.bias is not None:
                    m.bias = m.bias.to(dtype)
        if device is not None:
            model.to(device)
        for name, (rows, fp16) in verify.items():
            layer = model.model.get_submodule(name)
            dev = next((b.device for b in layer.buffers()), torch.device("cpu"))
            layer.set_protected_rows(rows.to(dev), fp16.to(dev))
        model.eval()
        return model

    def forward(self, *args, **kwargs):
        return self.model(*args, **kwargs)

    @classmethod
    def can_generate(cls) -> bool:
        return True

    def generate(self, *args, **kwargs):
        return self.model.generate(*args, **kwargs)

    def prepare_inputs_for_generation(self, *args, **kwargs):
        return self.model.prepare_inputs_for_generation(*args, **kwargs)


try:  # make AutoModelForCausalLM resolve model_type "csaq" (csaq/__init__.py registers the config)
    AutoModelForCausalLM.register(CSAQConfig, CSAQModelForCausalLM)
except Exception:
    pass
