"""Summarize (and optionally plot) run logs.

    python -m mini_nangila_b200.apps.analyze train train_log.csv [ddp_metrics.csv] [--plot]
    python -m mini_nangila_b200.apps.analyze metrics ddp_metrics.csv [--plot]
    python -m mini_nangila_b200.apps.analyze hpc hpc_bench.log [--plot]
    python -m mini_nangila_b200.apps.analyze twin client_metrics.csv [server_metrics.csv] [--plot]
    python -m mini_nangila_b200.apps.analyze entropy
    python -m mini_nangila_b200.apps.analyze checkpoint ckpt.h5 dataset
    python -m mini_nangila_b200.apps.analyze baselines baseline_comparison.csv [--plot]

The reference's plotting snippets (python/snippets/*.py,
python/nangila_ddp/plot_*.py, benchmarks/plot_baselines.py) as one CLI:
prints a JSON summary; ``--plot`` also writes the reference's PNGs (drawn by
``utils.plot``, no plotting library needed).
"""
from __future__ import annotations

import argparse
import json

import numpy as np

from ..utils import analysis as A


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("kind", choices=["train", "metrics", "hpc", "twin", "entropy", "checkpoint", "baselines"])
    ap.add_argument("files", nargs="*")
    ap.add_argument("--plot", action="store_true")
    a = ap.parse_args(argv)
    out: dict = {"kind": a.kind}
    if a.kind == "train":
        out.update(A.summarize_training(a.files[0], a.files[1] if len(a.files) > 1 else None))
        if a.plot and len(a.files) > 1:
            out["plot"] = A.plot_training(a.files[0], a.files[1])
    elif a.kind == "metrics":
        m = A.load_hook_metrics(a.files[0])
        r = m.get("ratio", np.array([]))
        out["ratio"] = A._stats(r)
        if a.plot:
            out["plot"] = A.plot_series(np.arange(r.size), r, "hook call index", "compression ratio",
                                        a.files[0].replace(".csv", "_ratio.png"), title="DDP hook compression ratio")
    elif a.kind == "hpc":
        out.update(A.summarize_hpc(a.files[0]))
        if a.plot:
            out["plot"] = A.plot_hpc(a.files[0])
    elif a.kind == "twin":
        out["client"] = A.summarize_ticks(a.files[0])
        if len(a.files) > 1:
            out["server"] = A.summarize_ticks(a.files[1])
        if a.plot:
            out["plot"] = A.plot_twin(a.files[0], a.files[1] if len(a.files) > 1 else None)
    elif a.kind == "entropy":
        out.update(A.entropy_reduction())
        if a.plot:
            out["plot"] = A.plot_entropy()
    elif a.kind == "baselines":
        out.update(A.summarize_baselines(a.files[0]))
        if a.plot:
            out["plot"] = A.plot_baselines(a.files[0], a.files[0].replace(".csv", ".png"))
    else:
        from ..checkpoint import hdf5

        x = hdf5.read_compressed_1d(a.files[0], a.files[1])
        out.update(n=int(x.size), min=float(x.min()) if x.size else None, max=float(x.max()) if x.size else None,
                   first=[float(v) for v in x[:8]])
    print(json.dumps(out))
    return out


if __name__ == "__main__":
    main()
