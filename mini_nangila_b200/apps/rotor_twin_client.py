"""gRPC rotor-twin client (examples/rotor_twin_net/src/bin/client.rs)."""
from __future__ import annotations

import argparse

from ..twin.rotor_net import RotorClient


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--server", default="127.0.0.1:50051")
    ap.add_argument("--rate-hz", type=int, default=50)
    ap.add_argument("--duration", type=int, default=5)
    ap.add_argument("--metrics", default="client_metrics.csv")
    ap.add_argument("--epsilon", type=float, default=0.05)
    ap.add_argument("--topk", type=float, default=0.0)
    a = ap.parse_args(argv)
    target = a.server.replace("http://", "").replace("https://", "")
    c = RotorClient(target, a.epsilon, a.topk, metrics_path=a.metrics)
    n = c.run(a.duration, a.rate_hz)
    c.close()
    print(f"sent {n} frames")


if __name__ == "__main__":
    main()
