"""Tiny models shared by the reference-run fixture generator
(make_ref_cases.py) and the tests that read its fixtures: plain torch and
transformers, no csaq import (the reference package and this one are both
named ``csaq``)."""

from __future__ import annotations

from types import SimpleNamespace

import torch
import torch.nn as nn
import torch.nn.functional as F

VOCAB = 96
CALIB_BATCHES = 40
PROFILE_SEED = 7  # torch.manual_seed right before profile(): the early-stop sample draws from it


class TinyNet(nn.Module):
    """embed -> fc1 -> ReLU -> fc2 -> head, next-token cross-entropy."""

    def __init__(self, vocab: int = VOCAB, dim: int = 48, hidden: int = 80):
        super().__init__()
        self.embed = nn.Embedding(vocab, dim)
        self.fc1 = nn.Linear(dim, hidden)
        self.fc2 = nn.Linear(hidden, dim)
        self.lm_head = nn.Linear(dim, vocab, bias=False)

    def forward(self, input_ids, labels=None, attention_mask=None, **_):
        h = self.embed(input_ids)
        logits = self.lm_head(self.fc2(F.relu(self.fc1(h))))
        loss = None
        if labels is not None:
            loss = F.cross_entropy(logits[:, :-1].reshape(-1, logits.shape[-1]), labels[:, 1:].reshape(-1))
        return SimpleNamespace(loss=loss, logits=logits)


def tiny_net() -> TinyNet:
    torch.manual_seed(11)
    return TinyNet()


def calib_batches():
    g = torch.Generator().manual_seed(12)
    return [{"input_ids": torch.randint(0, VOCAB, (2, 24), generator=g)} for _ in range(CALIB_BATCHES)]


def tiny_llama_config():
    from transformers import LlamaConfig
    return LlamaConfig(hidden_size=64, intermediate_size=128, num_hidden_layers=2, num_attention_heads=4,
                       num_key_value_heads=2, vocab_size=128, max_position_embeddings=256,
                       tie_word_embeddings=False)


def tiny_llama():
    from transformers import AutoModelForCausalLM
    torch.manual_seed(13)
    return AutoModelForCausalLM.from_config(tiny_llama_config(), dtype=torch.float32)


def uniform_budget(model, bits: int = 4):
    """Per-channel cliques of every decoder linear at one bit-width, leaders =
    each row itself: the budget solve_clique_budget hands inject_csaq_linear
    for a uniform-bit model (csaq/core.py:294-361)."""
    budget = {}
    for name, m in model.named_modules():
        if isinstance(m, nn.Linear) and "lm_head" not in name:
            budget[name] = [{"rows": [i], "bits": bits, "leader": i} for i in range(m.out_features)]
    return budget
