"""Import path of the reference's DDP hook package (``nangila_ddp``), backed by
mini_nangila_b200: ``from nangila_ddp import register_nangila_hook`` keeps
working and gets the fused sm_100a hook on CUDA models."""
from mini_nangila_b200.parallel.hook import register_nangila_hook

__all__ = ["register_nangila_hook"]
