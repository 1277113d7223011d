"""Synthetic and text token sources for the trainers (no network access).

* ``CharCorpus``: a character-level corpus.  The vocabulary is the sorted
  set of characters, so every rank that reads the same text builds the same
  vocabulary without a collective.  ``batch`` draws random windows (a
  nanoGPT-style random crop) from a generator keyed by (seed, rank, step):
  each rank sees its own stream of windows, reproducible from the key alone,
  so a resumed run continues the same stream.
* ``uniform_tokens``: tokens uniform over a vocabulary from a seed, the data
  of the GPT-2 / Llama throughput workloads.

The reference trainer loads TinyShakespeare (or, offline, the fallback text
``"abc def ghi " * 100000``) on rank 0 and broadcasts it, then shards fixed
windows with a ``DistributedSampler`` (python/nangila_ddp/train_nano.py:26-42,
:100-124).  There is no network here, so the fallback text is the default.
"""
from __future__ import annotations

import torch

FALLBACK_TEXT = "abc def ghi " * 100000


def _key(seed: int, rank: int, step: int) -> int:
    # splitmix-style mix of the three integers into one 63-bit seed
    x = (seed * 0x9E3779B97F4A7C15 + rank * 0xBF58476D1CE4E5B9 + step * 0x94D049BB133111EB) & ((1 << 64) - 1)
    x ^= x >> 31
    x = (x * 0xD6E8FEB86659FD93) & ((1 << 64) - 1)
    x ^= x >> 32
    return x & 0x7FFFFFFFFFFFFFFF


class CharCorpus:
    """Character tokens of a text with a deterministic vocabulary."""

    def __init__(self, text: str):
        if not text:
            raise ValueError("empty corpus")
        self.itos = sorted(set(text))
        stoi = {c: i for i, c in enumerate(self.itos)}
        self.vocab = len(self.itos)
        self.tokens = torch.tensor([stoi[c] for c in text], dtype=torch.long)

    @classmethod
    def from_path(cls, path: str | None) -> "CharCorpus":
        if path:
            with open(path, encoding="utf-8") as fh:
                return cls(fh.read())
        return cls(FALLBACK_TEXT)

    def batch(self, batch_size: int, block: int, *, seed: int, rank: int, step: int,
              device: torch.device | str = "cpu") -> tuple[torch.Tensor, torch.Tensor]:
        """(x, y): ``batch_size`` windows of ``block`` tokens and the same
        windows shifted by one."""
        span = self.tokens.numel() - block - 1
        if span <= 0:
            raise ValueError(f"corpus of {self.tokens.numel()} tokens is shorter than a window of {block + 1}")
        g = torch.Generator().manual_seed(_key(seed, rank, step))
        starts = torch.randint(0, span + 1, (batch_size,), generator=g)
        win = starts[:, None] + torch.arange(block + 1)[None, :]
        w = self.tokens[win]
        return w[:, :-1].contiguous().to(device), w[:, 1:].contiguous().to(device)


def uniform_tokens(vocab: int, batch_size: int, seq: int, *, seed: int, device) -> tuple[torch.Tensor, torch.Tensor]:
    """Tokens uniform over ``vocab`` from ``seed``: (x, y) with y = x shifted by one."""
    g = torch.Generator(device=device).manual_seed(seed)
    t = torch.randint(0, vocab, (batch_size, seq + 1), generator=g, device=device)
    return t[:, :-1].contiguous(), t[:, 1:].contiguous()


class MarkovTokens:
    """A learnable synthetic token stream: a fixed random first-order Markov
    chain over ``vocab`` tokens in which every token has ``branching``
    successors with probabilities proportional to 1/(i+1) (entropy about 1.8
    bits per token for 4 successors).  A model that learns the table reaches
    a loss near that entropy, far below the ln(vocab) of uniform tokens, so
    training curves of different gradient exchanges can be told apart.
    ``batch`` is a pure function of (seed, rank, step)."""

    def __init__(self, vocab: int, branching: int = 4, seed: int = 0):
        import numpy as np

        rng = np.random.default_rng(seed)
        self.vocab = vocab
        self.succ = rng.integers(0, vocab, size=(vocab, branching), dtype=np.int64)
        w = 1.0 / np.arange(1, branching + 1)
        self.cdf = np.cumsum(w / w.sum())
        self.entropy_nats = float(-(w / w.sum() * np.log(w / w.sum())).sum())

    def batch(self, batch_size: int, seq: int, *, seed: int, rank: int, step: int,
              device: torch.device | str = "cpu") -> tuple[torch.Tensor, torch.Tensor]:
        import numpy as np

        rng = np.random.default_rng(_key(seed, rank, step))
        t = np.empty((batch_size, seq + 1), np.int64)
        t[:, 0] = rng.integers(0, self.vocab, batch_size)
        choice = np.searchsorted(self.cdf, rng.random((batch_size, seq)), side="right")
        choice = np.minimum(choice, self.succ.shape[1] - 1)
        for i in range(seq):
            t[:, i + 1] = self.succ[t[:, i], choice[:, i]]
        w = torch.from_numpy(t)
        return w[:, :-1].contiguous().to(device), w[:, 1:].contiguous().to(device)
