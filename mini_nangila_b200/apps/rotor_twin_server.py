"""gRPC rotor-twin server (examples/rotor_twin_net/src/bin/server.rs)."""
from __future__ import annotations

import argparse
import time

from ..twin.rotor_net import RotorServer


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--listen", default="127.0.0.1:50051")
    ap.add_argument("--metrics", default="server_metrics.csv")
    ap.add_argument("--beta", type=float, default=0.9)
    a = ap.parse_args(argv)
    srv = RotorServer(beta=a.beta, metrics_path=a.metrics)
    server, port = srv.serve(a.listen)
    print(f"Rotor server listening on {a.listen}")
    try:
        while True:
            time.sleep(3600)
    except KeyboardInterrupt:
        server.stop(0)


if __name__ == "__main__":
    main()
