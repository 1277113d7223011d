"""GPT-2 small in stock PyTorch (the model's own forward/backward is not
part of the compressed path).  12 layers, d_model 768, 12 heads, FFN 3072,
vocab 50257, context 1024, tied input/output embeddings, weights N(0, 0.02).
Attention is ``F.scaled_dot_product_attention`` with a causal mask.

The embedding matrix is stored with its row count rounded up to a multiple
of ``pad_vocab_to`` (50257 -> 50304) so the output-projection GEMM gets
16-byte-aligned operands.  A fixed (non-trainable) bias of 0 on the real
columns and -inf on the padding columns is fused into that GEMM, so the
padding columns get probability 0 and zero gradient: the loss is the
cross-entropy over the 50257 real classes and the function computed is
exactly GPT-2 small's.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F


@dataclass
class GPT2Config:
    """GPT-2 dimensions; ``small()`` is the 124M model (12 layers, d 768, 12 heads, vocab 50257)."""
    vocab_size: int = 50257
    n_positions: int = 1024
    n_layer: int = 12
    n_head: int = 12
    n_embd: int = 768
    n_inner: int = 3072
    init_std: float = 0.02
    tie_embeddings: bool = True
    pad_vocab_to: int = 64

    @property
    def padded_vocab(self) -> int:
        p = max(1, self.pad_vocab_to)
        return (self.vocab_size + p - 1) // p * p

    @staticmethod
    def small() -> "GPT2Config":
        return GPT2Config()

    @staticmethod
    def tiny() -> "GPT2Config":
        return GPT2Config(vocab_size=512, n_positions=64, n_layer=2, n_head=4, n_embd=64, n_inner=256)


class CausalSelfAttention(nn.Module):
    def __init__(self, cfg: GPT2Config):
        super().__init__()
        self.n_head = cfg.n_head
        self.c_attn = nn.Linear(cfg.n_embd, 3 * cfg.n_embd)
        self.c_proj = nn.Linear(cfg.n_embd, cfg.n_embd)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        B, T, C = x.shape
        q, k, v = self.c_attn(x).split(C, dim=2)
        hd = C // self.n_head
        q = q.view(B, T, self.n_head, hd).transpose(1, 2)
        k = k.view(B, T, self.n_head, hd).transpose(1, 2)
        v = v.view(B, T, self.n_head, hd).transpose(1, 2)
        y = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        return self.c_proj(y.transpose(1, 2).reshape(B, T, C))


class MLP(nn.Module):
    def __init__(self, cfg: GPT2Config):
        super().__init__()
        self.c_fc = nn.Linear(cfg.n_embd, cfg.n_inner)
        self.c_proj = nn.Linear(cfg.n_inner, cfg.n_embd)

    def forward(self, x):
        return self.c_proj(F.gelu(self.c_fc(x), approximate="tanh"))


class Block(nn.Module):
    def __init__(self, cfg: GPT2Config):
        super().__init__()
        self.ln_1 = nn.LayerNorm(cfg.n_embd)
        self.attn = CausalSelfAttention(cfg)
        self.ln_2 = nn.LayerNorm(cfg.n_embd)
        self.mlp = MLP(cfg)

    def forward(self, x):
        x = x + self.attn(self.ln_1(x))
        return x + self.mlp(self.ln_2(x))


class GPT2(nn.Module):
    """Causal GPT-2 with tied embeddings; ``forward(x, y)`` returns the mean cross-entropy."""
    def __init__(self, cfg: GPT2Config):
        super().__init__()
        self.cfg = cfg
        self.wte = nn.Embedding(cfg.padded_vocab, cfg.n_embd)
        self.wpe = nn.Embedding(cfg.n_positions, cfg.n_embd)
        self.h = nn.ModuleList([Block(cfg) for _ in range(cfg.n_layer)])
        self.ln_f = nn.LayerNorm(cfg.n_embd)
        self.lm_head = nn.Linear(cfg.n_embd, cfg.padded_vocab, bias=False)
        if cfg.tie_embeddings:
            self.lm_head.weight = self.wte.weight
        pad_mask = torch.zeros(cfg.padded_vocab)
        pad_mask[cfg.vocab_size:] = float("-inf")
        self.register_buffer("vocab_mask", pad_mask, persistent=False)
        self.apply(self._init)

    def _init(self, m):
        if isinstance(m, (nn.Linear, nn.Embedding)):
            nn.init.normal_(m.weight, mean=0.0, std=self.cfg.init_std)
        if isinstance(m, nn.Linear) and m.bias is not None:
            nn.init.zeros_(m.bias)

    def forward(self, idx: torch.Tensor, targets: torch.Tensor | None = None):
        B, T = idx.shape
        pos = torch.arange(T, device=idx.device)
        x = self.wte(idx) + self.wpe(pos)
        for blk in self.h:
            x = blk(x)
        h = self.ln_f(x)
        if self.cfg.padded_vocab == self.cfg.vocab_size:
            logits = self.lm_head(h)
        else:
            logits = F.linear(h, self.lm_head.weight, self.vocab_mask.to(h.dtype if not torch.is_autocast_enabled()
                                                                          else torch.get_autocast_dtype("cuda")))
        if targets is None:
            return logits[..., : self.cfg.vocab_size]
        return F.cross_entropy(logits.reshape(-1, logits.size(-1)).float(), targets.reshape(-1))

    def num_params(self, exclude_padding: bool = True) -> int:
        n = sum(p.numel() for p in self.parameters())
        if exclude_padding:
            n -= (self.cfg.padded_vocab - self.cfg.vocab_size) * self.cfg.n_embd
        return n
