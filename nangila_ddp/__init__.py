"""Import path of the reference's DDP hook package (``nangila_ddp``), backed by
mini_nangila_b200: ``from nangila_ddp import register_nangila_hook`` keeps
working and gets the fused sm_100a hook on CUDA models.  The package's
modules keep their paths too: ``comm_hook``, ``train_nano``,
``plot_metrics``, ``plot_train_and_compression`` and
``examples.minigpt_train``."""
from .comm_hook import register_nangila_hook

__all__ = ["register_nangila_hook"]
