"""TinyGPT of the reference's DDP trainer (python/nangila_ddp/train_nano.py:44-56):
token embedding + learned positions + ``nn.TransformerEncoder`` + linear head.
``causal=True`` adds the causal mask the reference omits (its encoder sees
future tokens); the default keeps the reference's behaviour.
"""
from __future__ import annotations

import torch
import torch.nn as nn


class TinyGPT(nn.Module):
    """The reference trainer's TinyGPT (python/nangila_ddp/train_nano.py:44-56)."""
    def __init__(self, d_model=256, nhead=4, nlayers=4, vocab=5000, block_size=128, causal=False):
        super().__init__()
        self.causal = causal
        self.emb = nn.Embedding(vocab, d_model)
        self.pos = nn.Parameter(torch.zeros(1, block_size, d_model))
        layer = nn.TransformerEncoderLayer(d_model=d_model, nhead=nhead, batch_first=True)
        self.enc = nn.TransformerEncoder(layer, nlayers, enable_nested_tensor=False)
        self.lm = nn.Linear(d_model, vocab)

    def forward(self, x, targets=None):
        """Logits for ``x``; with ``targets``, the mean cross-entropy instead
        (the form ``DDPTrainer`` steps)."""
        h = self.emb(x) + self.pos[:, : x.size(1), :]
        mask = nn.Transformer.generate_square_subsequent_mask(x.size(1), device=x.device) if self.causal else None
        h = self.enc(h, mask=mask, is_causal=self.causal)
        logits = self.lm(h)
        if targets is None:
            return logits
        return nn.functional.cross_entropy(logits.reshape(-1, logits.size(-1)), targets.reshape(-1))
