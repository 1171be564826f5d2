"""Calibration data, evaluation, reporting and the on-disk format.

Same functions and files as csaq/utils.py of the reference:
build_calibration_data (csaq/utils.py:25-103), compute_perplexity (:106-171),
generate_csaq_report (:174-218) and export_csaq_model (:225-318).

The export writes the reference's three files: config.json (the base model
config with the quantisation config merged in and model_type "csaq"),
csaq_manifest.json and model.safetensors. Uniform-bit layers export exactly
the reference's buffers (``weight_packed`` uint8, ``weight_scales`` fp32,
``weight_zp`` int32, ``bias``). Mixed-row layers add, per bit-width b,
``tier{b}_rows`` / ``tier{b}_packed`` / ``tier{b}_scales`` / ``tier{b}_zp``;
the manifest then lists their tiers under ``layer_tiers`` (bits -> row count)
next to the reference's ``layer_bits`` (the dominant bit-width). With
``include_verify_rows`` the protected rows of the verify pass are kept as
``verify_rows`` (int64) and ``verify_fp16`` (their original fp16 weights).
"""

from __future__ import annotations

import json
import math
import os
import warnings
from typing import Any, Dict, List, Optional

import torch
import torch.nn as nn

FORMAT_VERSION = "0.5.1"          # the reference's csaq_version field
B200_FORMAT = "csaq-b200-tiers-1"  # marks the mixed-row extension


# ── calibration data ────────────────────────────────────────────────────────

def build_calibration_data(tokenizer: Any, custom_texts: List[str], n: Optional[int] = None,
                           seq_len: int = 128, device: str = "cpu") -> List[Dict[str, torch.Tensor]]:
    """Tokenise the caller's own texts into calibration batches (one text per
    batch, truncated / padded to ``seq_len``). There is no default dataset."""
    if not custom_texts:
        raise ValueError("[CSAQ] custom_texts is empty.\nProvide sentences in your target language/domain.\n"
                         "Example:\n  calib = build_calibration_data(tokenizer,\n"
                         "              custom_texts=['Your sentence 1', 'Your sentence 2', ...])")
    texts = list(custom_texts)
    if n is not None:
        texts = texts[:n]
    if len(texts) < 16:
        warnings.warn(f"[CSAQ] Only {len(texts)} calibration samples supplied. Salience estimates will be "
                      "noisy. Recommended minimum: 64.", stacklevel=2)
    out = []
    for t in texts:
        enc = tokenizer(str(t), return_tensors="pt", max_length=seq_len, truncation=True, padding="max_length")
        out.append({k: v.to(device) for k, v in enc.items()})
    return out


# ── evaluation ──────────────────────────────────────────────────────────────

def compute_perplexity(model: nn.Module, tokenizer: Any, eval_texts: List[str], max_tokens: int = 4096,
                       stride: int = 512, seq_len: int = 128, device: str = "cpu") -> float:
    """Sliding-window perplexity over the caller's texts joined by blank
    lines: windows of ``seq_len`` tokens every ``stride`` tokens, mean of the
    per-window losses, exponentiated. Non-finite window losses are dropped."""
    if not eval_texts:
        raise ValueError("[CSAQ] eval_texts is empty.")
    first = next(model.parameters()).device
    if first.type != "cpu" and device == "cpu":
        device = str(first)
    ids = tokenizer("\n\n".join(eval_texts), return_tensors="pt").input_ids[:, :max_tokens].to(device)
    losses: List[float] = []
    model.eval()
    with torch.no_grad():
        for begin in range(0, ids.shape[1] - 1, stride):
            chunk = ids[:, begin:min(begin + seq_len, ids.shape[1])]
            if chunk.shape[1] < 2:
                continue
            try:
                loss = model(chunk, labels=chunk).loss
            except Exception as exc:  # the reference keeps going past a failing window
                warnings.warn(f"[CSAQ] PPL chunk {begin}-{begin + chunk.shape[1]} failed: {exc}")
                continue
            if torch.isfinite(loss):
                losses.append(float(loss))
    if not losses:
        return float("inf")
    return float(math.exp(sum(losses) / len(losses)))


# ── report ──────────────────────────────────────────────────────────────────

def generate_csaq_report(info: Dict[str, Any], save_path: str = "./CSAQ_Report.json") -> Dict[str, Any]:
    """JSON report of a quantize() run (same keys as the reference's)."""
    tiers = info.get("tier_stats", {}) or {}
    total = sum(tiers.values()) if tiers else 0
    pct = {t: round(100.0 * c / total, 2) for t, c in tiers.items()} if total > 0 else {}
    report = {
        "csaq_version": FORMAT_VERSION,
        "actual_avg_bits": round(info.get("actual_bits", 0.0), 4),
        "total_cliques": info.get("cliques_count", 0),
        "total_quantized_params": total,
        "elapsed_seconds": round(info.get("elapsed_s", 0.0), 2),
        "bit_distribution": tiers,
        "bit_distribution_pct": pct,
        "ppl": info.get("ppl", "not_computed"),
        "calibration_domain": info.get("calibration_domain", "user_provided"),
        "salience_overlap_pct": info.get("overlap_pct", "not_computed"),
        "memory_before_gb": info.get("memory_before_gb", "not_measured"),
        "memory_after_gb": info.get("memory_after_gb", "not_measured"),
        "memory_saved_gb": info.get("memory_saved_gb", "not_measured"),
        "memory_saved_pct": info.get("memory_saved_pct", "not_measured"),
    }
    os.makedirs(os.path.dirname(os.path.abspath(save_path)), exist_ok=True)
    with open(save_path, "w", encoding="utf-8") as f:
        json.dump(report, f, indent=2)
    return report


# ── export ──────────────────────────────────────────────────────────────────

_SPECULATIVE_BUFFERS = ("_csaq_fp16_backup", "_csaq_quant_stash", "_csaq_hi_rows")


def _json_ready(v):
    return v.tolist() if hasattr(v, "tolist") else v


def export_csaq_model(model: nn.Module, config: Any, budget: Any, save_path: str,
                      info: Optional[Dict[str, Any]] = None, include_verify_rows: bool = False) -> str:
    """Write config.json, csaq_manifest.json and model.safetensors under
    ``save_path``; return its absolute path."""
    import safetensors.torch
    from .kernels import CSAQLinear

    os.makedirs(save_path, exist_ok=True)
    try:
        cfg = model.config.to_dict()
    except AttributeError:
        cfg = {}
    config.base_model_type = cfg.get("model_type", "unknown")
    config.base_model_name_or_path = cfg.get("_name_or_path", cfg.get("name_or_path", "unknown"))
    quant = config.to_dict()
    quant["quant_type"] = "csaq"
    quant["csaq_version"] = FORMAT_VERSION
    cfg["model_type"] = "csaq"
    cfg.update(quant)
    cfg.pop("quantization_config", None)
    with open(os.path.join(save_path, "config.json"), "w", encoding="utf-8") as f:
        json.dump(cfg, f, indent=2)
    tok_cfg = os.path.join(save_path, "tokenizer_config.json")
    if not os.path.exists(tok_cfg):
        with open(tok_cfg, "w", encoding="utf-8") as f:
            json.dump({}, f)

    layer_bits: Dict[str, int] = {}
    layer_tiers: Dict[str, Dict[str, int]] = {}
    verify_layers: List[str] = []
    extra: Dict[str, torch.Tensor] = {}
    for name, m in model.named_modules():
        if not isinstance(m, CSAQLinear):
            continue
        layer_bits[name] = m.bits
        if m.tier_bits:
            layer_tiers[name] = {str(b): int(getattr(m, f"tier{b}_rows").numel()) for b in m.tier_bits}
        hi = getattr(m, "_csaq_hi_rows", None)
        if include_verify_rows and hi is not None and hi.numel():
            extra[f"{name}.verify_rows"] = hi.to(torch.int64).contiguous()
            extra[f"{name}.verify_fp16"] = m._csaq_fp16_backup.to(torch.float16).contiguous()
            verify_layers.append(name)

    manifest: Dict[str, Any] = {
        "csaq_version": FORMAT_VERSION,
        "bit_distribution": info.get("tier_stats", {}) if info else {},
        "actual_avg_bits": info.get("actual_bits", 0.0) if info else 0.0,
        "cliques_count": info.get("cliques_count", 0) if info else 0,
        "causal_map": {k: _json_ready(v) for k, v in (info or {}).get("causal_map", {}).items()},
        "target_bits": config.target_bits,
        "bit_options": config.bit_options,
        "group_size": config.group_size,
        "calibration_domain": info.get("calibration_domain", "user_provided") if info else "user_provided",
        "layer_bits": layer_bits,
    }
    if layer_tiers or verify_layers:
        manifest["b200_format"] = B200_FORMAT
        manifest["layer_tiers"] = layer_tiers
        manifest["verify_layers"] = verify_layers
    with open(os.path.join(save_path, "csaq_manifest.json"), "w", encoding="utf-8") as f:
        json.dump(manifest, f, indent=2)

    state = {k: v.detach().contiguous().cpu() for k, v in model.state_dict().items()
             if not any(k.endswith(s) for s in _SPECULATIVE_BUFFERS)}
    state.update({k: v.cpu() for k, v in extra.items()})
    safetensors.torch.save_file(state, os.path.join(save_path, "model.safetensors"))
    path = os.path.abspath(save_path)
    print(f"[CSAQ] Model exported → {path}")
    return path
