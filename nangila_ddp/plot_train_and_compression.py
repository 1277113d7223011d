"""``nangila_ddp/plot_train_and_compression.py``: loss and compression ratio
over time from ``train_log.csv`` and the hook's metrics CSV.  Writes
``train_and_compression.png`` (drawn by ``utils.plot``) and prints the
numeric summary."""
import json
import sys

from mini_nangila_b200.utils import analysis


def main(argv=None):
    argv = sys.argv[1:] if argv is None else argv
    train_csv = argv[0] if argv else "train_log.csv"
    ddp_csv = argv[1] if len(argv) > 1 else "ddp_metrics.csv"
    out = analysis.plot_training(train_csv, ddp_csv, "train_and_compression.png")
    print("Saved:", out)
    print(json.dumps(analysis.summarize_training(train_csv, ddp_csv)))
    return out


if __name__ == "__main__":
    main()
