"""Digital-twin domain: closed-loop edge/cloud sync (nangila-twin) and the
gRPC rotor service (examples/rotor_twin_net)."""
from .edge_sync import CloudNode, EdgeNode, SyncError

__all__ = ["CloudNode", "EdgeNode", "SyncError"]
