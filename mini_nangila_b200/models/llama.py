"""Llama-style decoder in stock PyTorch: RMSNorm, rotary position embedding,
grouped-query attention, SwiGLU FFN.  ``LlamaConfig.b1_1()`` is the 1.1B
configuration (22 layers, d_model 2048, 32 heads, 4 KV heads, FFN 5632,
vocab 32000, context 2048).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F


@dataclass
class LlamaConfig:
    """Llama-style dimensions; ``b1_1()`` is the 1.1B model (22 layers, d 2048, 32 heads, 4 KV heads)."""
    vocab_size: int = 32000
    max_seq: int = 2048
    n_layer: int = 22
    n_head: int = 32
    n_kv_head: int = 4
    d_model: int = 2048
    d_ff: int = 5632
    rope_theta: float = 10000.0
    eps: float = 1e-5
    init_std: float = 0.02

    @staticmethod
    def b1_1() -> "LlamaConfig":
        return LlamaConfig()

    @staticmethod
    def tiny() -> "LlamaConfig":
        return LlamaConfig(vocab_size=512, max_seq=64, n_layer=2, n_head=4, n_kv_head=2, d_model=64, d_ff=172)


class RMSNorm(nn.Module):
    def __init__(self, d: int, eps: float):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(d))

    def forward(self, x):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps)).to(x.dtype) * self.weight


def rope_tables(seq: int, hd: int, theta: float, device) -> tuple[torch.Tensor, torch.Tensor]:
    inv = 1.0 / (theta ** (torch.arange(0, hd, 2, device=device, dtype=torch.float32) / hd))
    t = torch.arange(seq, device=device, dtype=torch.float32)
    f = torch.outer(t, inv)
    return f.cos(), f.sin()


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    # x: (B, H, T, D); rotate pairs (even, odd) halves
    d = x.shape[-1] // 2
    x1, x2 = x[..., :d], x[..., d:]
    c = cos[None, None, : x.shape[2]].to(x.dtype)
    s = sin[None, None, : x.shape[2]].to(x.dtype)
    return torch.cat([x1 * c - x2 * s, x1 * s + x2 * c], dim=-1)


class Attention(nn.Module):
    def __init__(self, cfg: LlamaConfig):
        super().__init__()
        self.h, self.kvh = cfg.n_head, cfg.n_kv_head
        self.hd = cfg.d_model // cfg.n_head
        self.q = nn.Linear(cfg.d_model, cfg.n_head * self.hd, bias=False)
        self.k = nn.Linear(cfg.d_model, cfg.n_kv_head * self.hd, bias=False)
        self.v = nn.Linear(cfg.d_model, cfg.n_kv_head * self.hd, bias=False)
        self.o = nn.Linear(cfg.n_head * self.hd, cfg.d_model, bias=False)

    def forward(self, x, cos, sin):
        B, T, _ = x.shape
        q = self.q(x).view(B, T, self.h, self.hd).transpose(1, 2)
        k = self.k(x).view(B, T, self.kvh, self.hd).transpose(1, 2)
        v = self.v(x).view(B, T, self.kvh, self.hd).transpose(1, 2)
        q, k = apply_rope(q, cos, sin), apply_rope(k, cos, sin)
        y = F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=True)
        return self.o(y.transpose(1, 2).reshape(B, T, self.h * self.hd))


class SwiGLU(nn.Module):
    def __init__(self, cfg: LlamaConfig):
        super().__init__()
        self.gate = nn.Linear(cfg.d_model, cfg.d_ff, bias=False)
        self.up = nn.Linear(cfg.d_model, cfg.d_ff, bias=False)
        self.down = nn.Linear(cfg.d_ff, cfg.d_model, bias=False)

    def forward(self, x):
        return self.down(F.silu(self.gate(x)) * self.up(x))


class Layer(nn.Module):
    def __init__(self, cfg: LlamaConfig):
        super().__init__()
        self.n1 = RMSNorm(cfg.d_model, cfg.eps)
        self.attn = Attention(cfg)
        self.n2 = RMSNorm(cfg.d_model, cfg.eps)
        self.ffn = SwiGLU(cfg)

    def forward(self, x, cos, sin):
        x = x + self.attn(self.n1(x), cos, sin)
        return x + self.ffn(self.n2(x))


class Llama(nn.Module):
    """Llama-style decoder (RMSNorm, RoPE, grouped-query attention, SwiGLU); ``forward(x, y)`` returns the loss."""
    def __init__(self, cfg: LlamaConfig):
        super().__init__()
        self.cfg = cfg
        self.emb = nn.Embedding(cfg.vocab_size, cfg.d_model)
        self.layers = nn.ModuleList([Layer(cfg) for _ in range(cfg.n_layer)])
        self.norm = RMSNorm(cfg.d_model, cfg.eps)
        self.head = nn.Linear(cfg.d_model, cfg.vocab_size, bias=False)
        for m in self.modules():
            if isinstance(m, (nn.Linear, nn.Embedding)):
                nn.init.normal_(m.weight, mean=0.0, std=cfg.init_std)
        self._rope = None

    def forward(self, idx, targets=None):
        B, T = idx.shape
        if self._rope is None or self._rope[0].device != idx.device or self._rope[0].shape[0] < T:
            self._rope = rope_tables(max(T, self.cfg.max_seq), self.cfg.d_model // self.cfg.n_head,
                                     self.cfg.rope_theta, idx.device)
        cos, sin = self._rope
        x = self.emb(idx)
        for layer in self.layers:
            x = layer(x, cos, sin)
        logits = self.head(self.norm(x))
        if targets is None:
            return logits
        return F.cross_entropy(logits.reshape(-1, logits.size(-1)).float(), targets.reshape(-1))

    def num_params(self) -> int:
        return sum(p.numel() for p in self.parameters())
