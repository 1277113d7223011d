"""Rotor digital-twin demo (examples/rotor_twin/src/main.rs): a 6-DOF IMU
stream through the closed-loop EdgeNode -> CloudNode pair (momentum 0.9,
error-bounded eps); reports compression and RMS error once per second."""
from __future__ import annotations

import argparse
import time

import numpy as np

from ..ai import MomentumPredictor
from ..core import FixedPointBuffer
from ..hpc import ErrorBoundedQuantizer
from ..twin import CloudNode, EdgeNode
from ..twin.rotor_net import imu_sample


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--duration", type=int, default=10)
    ap.add_argument("--rate-hz", type=int, default=100)
    ap.add_argument("--epsilon", type=float, default=0.05)
    ap.add_argument("--no-sleep", action="store_true")
    a = ap.parse_args(argv)
    edge = EdgeNode(MomentumPredictor(0.9), ErrorBoundedQuantizer(a.epsilon))
    cloud = CloudNode(MomentumPredictor(0.9), ErrorBoundedQuantizer(a.epsilon))
    raw = tx = 0
    se = 0.0
    cnt = 0
    for t in range(a.duration * a.rate_hz):
        x = imu_sample(t / a.rate_hz)
        s = FixedPointBuffer.from_f32(x)
        raw += x.size * 4
        b, sc = edge.send(s)
        tx += len(b) + 4
        r = cloud.receive(b, sc)
        d = s.to_f32().astype(np.float64) - r.to_f32().astype(np.float64)
        se += float((d * d).sum())
        cnt += d.size
        if t % a.rate_hz == 0:
            print(f"t={t // a.rate_hz:4d}s  compression={raw / tx:6.2f}×  rms_err={np.sqrt(se / cnt):.5f}")
        if not a.no_sleep:
            time.sleep(1.0 / a.rate_hz)
    rms = float(np.sqrt(se / max(cnt, 1)))
    print(f"Total raw: {raw / 1024:.2f} KB, tx: {tx / 1024:.2f} KB, ratio: {raw / tx:.2f}×, RMS err: {rms:.5f}")
    return raw / tx, rms


if __name__ == "__main__":
    main()
