"""The benchmark workloads, one frozen dataclass each, named by what they
are.  ``bench.py`` and the apps take their defaults from here, and
``tests/test_workloads.py`` keeps the model configurations and app defaults
consistent with them."""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class GPT2SmallDDP:
    """GPT-2 small data-parallel training with the compressed hook."""

    n_layer: int = 12
    d_model: int = 768
    n_head: int = 12
    d_ff: int = 3072
    vocab: int = 50257
    seq: int = 1024
    micro_batch: int = 8  # per GPU
    bucket_mb: float = 25.0
    lr: float = 6e-4
    init_std: float = 0.02
    precision: str = "bf16 autocast, fp32 master weights"
    hook: str = "INT4, stochastic, EMA predictor (beta 0.9), error feedback"


@dataclass(frozen=True)
class Llama1BTopK:
    """Llama-style 1.1B data-parallel training with top-k + error feedback."""

    n_layer: int = 22
    d_model: int = 2048
    n_head: int = 32
    n_kv_head: int = 4
    d_ff: int = 5632
    vocab: int = 32000
    seq: int = 2048
    micro_batch: int = 4
    keep_fractions: tuple = (0.05, 0.10)
    precision: str = "bf16"


@dataclass(frozen=True)
class ModeSwitchingAR1:
    """10,000-element AR(1) gradients, momentum + block INT4 training steps,
    error-bounded checkpoints every 10 steps."""

    n: int = 10_000
    steps: int = 50
    checkpoint_interval: int = 10
    rho: float = 0.9
    sigma: float = 1e-3
    sigma0: float = 1e-2
    sparse_frac: float = 0.7
    sparse_scale: float = 0.01
    beta: float = 0.9
    block: int = 256
    epsilon: float = 1e-3
    seed: int = 0


@dataclass(frozen=True)
class AllReduceSweep:
    """Compressed all-reduce of fp32 buckets whose contents evolve as AR(1)."""

    # 1 MB to 1 GB, plus the GPT-2 small bucket sizes (25 MB, and the 154 MB
    # tied-embedding bucket)
    sizes_mb: tuple = (1, 4, 16, 25, 64, 154, 256, 1024)
    steps: int = 20
    rho: float = 0.9
    sigma: float = 1e-3
    modes: tuple = ("int4", "topk1", "topk5", "topk10")
    gpus: tuple = (2, 4, 8)


@dataclass(frozen=True)
class TrajectoryCodec:
    """LAMMPS-style trajectory: 1 M atoms x 100 steps, positions in a 100^3
    box with N(0, 0.01^2) steps, N(0, 1) velocities, eps 1e-3."""

    atoms: int = 1_000_000
    steps: int = 100
    box: float = 100.0
    sigma: float = 0.01
    epsilon: float = 1e-3
    codecs: tuple = ("eb", "bs", "bsrle")
    fields: tuple = ("pos", "vel")
