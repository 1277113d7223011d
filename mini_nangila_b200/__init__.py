"""mini-nangila-b200: predictive-residual compression for B200 (sm_100a).

Subpackages (imported on first use, so ``import mini_nangila_b200`` stays
light):

* ``core``: Q8.23 buffers, predictor / quantizer interfaces, UnifiedQuantizer,
  TopologyMask;
* ``ai`` and ``hpc``: momentum / linear predictors and their codecs;
* ``checkpoint``: ``.nz`` trajectories, LAMMPS dumps, chunked datasets,
  tensor checkpoints;
* ``ops``: the sm_100a codec and trajectory pipelines;
* ``parallel``: the DDP hook (``register_nangila_hook``), the fused
  communicator, the rank monitor;
* ``train``, ``models``, ``twin``, ``utils``, ``apps``, ``workloads``.
"""
import importlib

__version__ = "0.1.0"

_SUBMODULES = ("ai", "apps", "checkpoint", "core", "hpc", "models", "ops", "parallel", "train", "twin", "utils",
               "workloads")
__all__ = list(_SUBMODULES) + ["__version__"]


def __getattr__(name):
    if name in _SUBMODULES:
        return importlib.import_module(f".{name}", __name__)
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
