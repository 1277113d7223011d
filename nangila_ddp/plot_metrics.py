"""``nangila_ddp/plot_metrics.py``: compression ratio per hook call from a
metrics CSV (both the key,value layout and the older ``step,`` prefix).
Writes ``<csv>_ratio.png`` (drawn by ``utils.plot``) and prints the ratio
summary."""
import json
import sys

import numpy as np

from mini_nangila_b200.utils import analysis


def main(argv=None):
    argv = sys.argv[1:] if argv is None else argv
    path = argv[0] if argv else "ddp_metrics.csv"
    ratio = analysis.load_hook_metrics(path).get("ratio", np.array([]))
    if ratio.size == 0:
        print("No metrics found in", path)
        return None
    out = analysis.plot_series(np.arange(ratio.size), ratio, "hook call index", "compression ratio (raw/comp)",
                               path.replace(".csv", "_ratio.png"), title="DDP hook compression ratio")
    print("Saved plot:", out)
    print(json.dumps(analysis._stats(ratio)))
    return out


if __name__ == "__main__":
    main()
