"""On-disk format: export_csaq_model and CSAQModelForCausalLM (the reference's
csaq/utils.py:225-318 and csaq/modeling.py:15-87).

The CPU test builds a tiny Llama whose linears are CSAQLinear layers with
synthetic buffers (uniform and mixed-row), exports it and loads it back:
every buffer round-trips exactly, uniform layers use the reference's key
names, and the manifest records layer_bits (reference) plus layer_tiers (the
mixed-row extension). The GPU test does the same through quantize() and
compares logits before and after the round trip.
"""

import json
import os

import pytest
import torch
import torch.nn as nn


def _tiny_llama():
    from csaq import _synthetic as syn
    from transformers import AutoModelForCausalLM
    cfg = syn.decoder_config("tiny-llama", None)
    torch.manual_seed(0)
    return AutoModelForCausalLM.from_config(cfg, dtype=torch.float32)


def _fill_synthetic(model):
    """Replace every decoder linear by a CSAQLinear with random buffers:
    q/k/v/o uniform 4-bit per-channel, the MLP mixed {16, 8, 4} by row."""
    from csaq.kernels import CSAQLinear
    g = torch.Generator().manual_seed(1)
    for name, lin in list(model.named_modules()):
        if not isinstance(lin, nn.Linear) or "lm_head" in name:
            continue
        parent_name, _, child = name.rpartition(".")
        parent = model.get_submodule(parent_name)
        N, K = lin.out_features, lin.in_features
        if "mlp" in name:
            n16, n8 = N // 10, N // 5
            layer = CSAQLinear.empty_tiers(K, N, {16: n16, 8: n8, 4: N - n16 - n8}, group_size=128, bias=lin.bias)
            perm = torch.randperm(N, generator=g).to(torch.int32)
            start = 0
            for b in layer.tier_bits:
                n = getattr(layer, f"tier{b}_rows").numel()
                getattr(layer, f"tier{b}_rows").copy_(torch.sort(perm[start:start + n]).values)
                start += n
                pk = getattr(layer, f"tier{b}_packed")
                pk.copy_(torch.randint(0, 256, pk.shape, generator=g, dtype=torch.int32).to(torch.uint8))
                getattr(layer, f"tier{b}_scales").copy_(torch.rand(getattr(layer, f"tier{b}_scales").shape, generator=g))
                zp = getattr(layer, f"tier{b}_zp")
                zp.copy_(torch.randint(0, 15, zp.shape, generator=g, dtype=torch.int32))
        else:
            layer = CSAQLinear(K, N, 4, bias=lin.bias, group_size=-1)
            layer.weight_packed.copy_(torch.randint(0, 256, layer.weight_packed.shape, generator=g,
                                                    dtype=torch.int32).to(torch.uint8))
            layer.weight_scales.copy_(torch.rand(N, generator=g))
            layer.weight_zp.copy_(torch.randint(0, 15, (N,), generator=g, dtype=torch.int32))
        setattr(parent, child, layer)
    return model


def test_export_and_load_round_trip_cpu(tmp_path):
    import safetensors.torch
    from csaq import CSAQConfig, CSAQModelForCausalLM, export_csaq_model
    from csaq.kernels import CSAQLinear
    model = _fill_synthetic(_tiny_llama())
    cfg = CSAQConfig(target_bits=4.0, bit_options=[4, 8, 16], group_size=128)
    info = {"tier_stats": {"4": 10, "8": 2, "16": 1}, "actual_bits": 4.33, "cliques_count": 7,
            "causal_map": {"model.layers.0.mlp.up_proj": [1, 2]}}
    path = export_csaq_model(model, cfg, None, str(tmp_path / "out"), info)
    for f in ("config.json", "csaq_manifest.json", "model.safetensors", "tokenizer_config.json"):
        assert os.path.exists(os.path.join(path, f)), f
    conf = json.load(open(os.path.join(path, "config.json")))
    assert conf["model_type"] == "csaq" and conf["quant_type"] == "csaq" and conf["base_model_type"] == "llama"
    man = json.load(open(os.path.join(path, "csaq_manifest.json")))
    assert man["csaq_version"] == "0.5.1" and man["group_size"] == 128
    assert man["layer_bits"]["model.layers.0.self_attn.q_proj"] == 4
    assert man["layer_tiers"]["model.layers.1.mlp.down_proj"] == {"16": 51, "8": 102, "4": 359}
    keys = safetensors.torch.load_file(os.path.join(path, "model.safetensors")).keys()
    q = "model.layers.0.self_attn.q_proj."
    assert {q + "weight_packed", q + "weight_scales", q + "weight_zp"} <= set(keys)
    assert not any(k.endswith(("_csaq_fp16_backup", "_csaq_hi_rows", "_csaq_quant_stash")) for k in keys)

    loaded = CSAQModelForCausalLM.from_pretrained(path)
    src = dict(model.named_buffers())
    dst = dict(loaded.model.named_buffers())
    n = 0
    for k, v in src.items():
        if k.endswith(("_csaq_fp16_backup", "_csaq_hi_rows")):
            continue
        assert k in dst, k
        assert torch.equal(v.cpu(), dst[k].cpu()), k
        n += 1
    assert n > 0
    for k, p in model.named_parameters():
        assert torch.equal(p.detach(), dict(loaded.model.named_parameters())[k].detach().float()), k
    assert sum(isinstance(m, CSAQLinear) for m in loaded.modules()) == 14


@pytest.mark.gpu
def test_quantize_export_load_logits_gpu(tmp_path):
    """quantize() -> export (with the verify rows) -> load: the same logits, draft and verify."""
    from csaq import CSAQConfig, CSAQModelForCausalLM, export_csaq_model, quantize
    from csaq import _synthetic as syn
    from csaq.kernels import CSAQLinear
    model = syn.build_decoder("tiny-llama", device="cuda", seed=2, dtype=torch.bfloat16)
    g = torch.Generator().manual_seed(5)
    calib = [{"input_ids": torch.randint(0, 2048, (1, 32), generator=g)} for _ in range(3)]
    cfg = CSAQConfig(target_bits=4.0, bit_options=[4, 8, 16], group_size=128, clique_threshold=0.6)
    model, info = quantize(model, calib, cfg, verbose=False)
    ids = torch.randint(0, 2048, (2, 20), generator=g).cuda()
    with torch.no_grad():
        ref = model(input_ids=ids).logits
        for m in model.modules():
            if isinstance(m, CSAQLinear):
                m.verify_mode = True
        ref_v = model(input_ids=ids).logits
    path = export_csaq_model(model, cfg, None, str(tmp_path / "q"), info, include_verify_rows=True)
    loaded = CSAQModelForCausalLM.from_pretrained(path, device="cuda")
    with torch.no_grad():
        got = loaded(input_ids=ids).logits
        for m in loaded.modules():
            if isinstance(m, CSAQLinear):
                m.verify_mode = True
        got_v = loaded(input_ids=ids).logits
    assert got.dtype == ref.dtype
    assert torch.equal(got, ref)
    assert torch.equal(got_v, ref_v)


# ── byte identity with the reference's export_csaq_model (uniform-bit layers) ──

def _golden_export():
    import sys
    import numpy as np
    here = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
    if here not in sys.path:
        sys.path.insert(0, here)
    import tiny_nets
    return np.load(os.path.join(here, "export_golden.npz")), tiny_nets


def _export_and_digest(model, tmp_path, tiny_nets):
    import hashlib
    from csaq.config import CSAQConfig
    from csaq.utils import export_csaq_model
    cfg = CSAQConfig(target_bits=4.0, bit_options=[4, 8], group_size=-1)
    info = {"causal_map": {"model.layers.0.mlp.down_proj": [1, 5, 9]}, "tier_stats": {"int4": 1234},
            "actual_bits": 4.0, "cliques_count": 7}
    d = str(tmp_path / "export")
    export_csaq_model(model, cfg, tiny_nets.uniform_budget(model, 4), d, info)
    out = {}
    for f in ("config.json", "csaq_manifest.json", "model.safetensors", "tokenizer_config.json"):
        with open(os.path.join(d, f), "rb") as fh:
            out[f] = hashlib.sha256(fh.read()).digest()
    return out


def test_uniform_export_byte_identical_to_reference(tmp_path):
    """A uniform 4-bit model with the reference's own quantised buffers exports
    config.json, csaq_manifest.json, model.safetensors and tokenizer_config.json
    byte for byte as the reference's export_csaq_model (csaq/utils.py:225-318)."""
    from csaq.kernels import CSAQLinear
    g, tiny_nets = _golden_export()
    model = tiny_nets.tiny_llama()
    for name, lin in list(model.named_modules()):
        if isinstance(lin, nn.Linear) and "lm_head" not in name:
            parent_name, _, child = name.rpartition(".")
            setattr(model.get_submodule(parent_name), child,
                    CSAQLinear(lin.in_features, lin.out_features, 4, bias=lin.bias, group_size=-1))
    state = {k[2:]: torch.from_numpy(g[k]) for k in g.files if k.startswith("q_")}
    model.load_state_dict(state, strict=True)
    got = _export_and_digest(model, tmp_path, tiny_nets)
    for f, dig in got.items():
        assert dig == g[f"sha_{f}"].tobytes(), f


@pytest.mark.gpu
def test_uniform_export_from_our_quantiser_byte_identical(tmp_path):
    """The same tiny Llama quantised by this package's inject_csaq_linear (GPU
    kernels) exports the reference's bytes."""
    from csaq.kernels import inject_csaq_linear
    g, tiny_nets = _golden_export()
    model = tiny_nets.tiny_llama()
    for k, v in model.state_dict().items():
        assert torch.equal(v, torch.from_numpy(g[f"w_{k}"])), k
    model = model.cuda()
    inject_csaq_linear(model, tiny_nets.uniform_budget(model, 4), verbose=False)
    got = _export_and_digest(model, tmp_path, tiny_nets)
    for f, dig in got.items():
        assert dig == g[f"sha_{f}"].tobytes(), f
