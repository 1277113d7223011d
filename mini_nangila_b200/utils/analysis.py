"""Log analysis for training, DDP-hook, HPC and twin runs.

Readers for the CSV/text layouts the apps write (the same layouts as the
reference's: ``train_log.csv`` rows ``ts,step,loss,...``
(python/nangila_ddp/train_nano.py:147-181), hook metrics rows of
``key,value`` pairs (comm_hook.py:307-319) or the older ``step,<n>,...``
prefix (python/nangila_ddp/plot_metrics.py:6-21), HPC bench lines
``step N ratio R ... max_err E`` (python/snippets/plot_hpc_logs.py:6-17),
twin metric CSVs with the tick first and the ratio last
(python/snippets/plot_rotor_net.py:6-19), the compression-baseline CSV of
``apps/baselines`` (benchmarks/plot_baselines.py:8-16)), numeric summaries
of each, and
PNG or SVG plots drawn by ``utils.plot`` (no plotting library needed).  ``entropy_reduction`` restates the reference's
entropy illustration (python/snippets/entropy_plot.py:5-33) as numbers: the
histogram entropy of a signal and of its EMA-prediction residual.
"""
from __future__ import annotations

import csv
import math
import re

import numpy as np


# ------------------------------------------------------------------ readers
def load_train_log(path: str):
    ts, step, loss = [], [], []
    with open(path) as fh:
        for row in csv.reader(fh):
            if not row or row[0] == "ts":
                continue
            try:
                ts.append(float(row[0]))
                step.append(int(row[1]))
                loss.append(float(row[2]))
            except (ValueError, IndexError):
                continue
    return np.array(ts), np.array(step, dtype=np.int64), np.array(loss)


def load_hook_metrics(path: str):
    """Rows of ``key,value`` pairs -> dict of arrays (ts, ratio, ...); rows
    with the older ``step,<n>,...,ratio,<r>`` prefix are read too."""
    cols: dict[str, list[float]] = {}
    with open(path) as fh:
        for line in fh:
            parts = line.strip().split(",")
            if len(parts) < 2 or parts[0] not in ("ts", "step"):
                continue
            kv = {parts[i]: parts[i + 1] for i in range(0, len(parts) - 1, 2)}
            if parts[0] == "step" and "ratio" not in kv:
                kv["ratio"] = parts[-1]
            for key, v in kv.items():
                try:
                    cols.setdefault(key, []).append(float(v))
                except ValueError:
                    continue
    return {k: np.array(v) for k, v in cols.items()}


_HPC_RE = re.compile(r"step\s+(\d+)\s+ratio\s+([0-9.eE+-]+).+max_err\s+([0-9.eE+-]+)", re.IGNORECASE)


def parse_hpc_log(path: str):
    steps, ratios, errs = [], [], []
    with open(path) as fh:
        for line in fh:
            m = _HPC_RE.search(line)
            if m:
                steps.append(int(m.group(1)))
                ratios.append(float(m.group(2)))
                errs.append(float(m.group(3)))
    return np.array(steps, dtype=np.int64), np.array(ratios), np.array(errs)


def load_tick_ratio_csv(path: str):
    ticks, ratios = [], []
    with open(path) as fh:
        rd = csv.reader(fh)
        next(rd, None)
        for row in rd:
            try:
                ticks.append(int(row[0]))
                ratios.append(float(row[-1]))
            except (ValueError, IndexError):
                continue
    return np.array(ticks, dtype=np.int64), np.array(ratios)


def load_baseline_rows(path: str) -> list[dict]:
    """OK rows with a nonzero size of a ``baseline_comparison.csv``."""
    with open(path, newline="") as fh:
        return [r for r in csv.DictReader(fh)
                if r.get("status") == "OK" and r.get("compressed_bytes") not in (None, "", "0")]


# ---------------------------------------------------------------- summaries
def _stats(x: np.ndarray) -> dict:
    if x.size == 0:
        return {"n": 0}
    return {"n": int(x.size), "first": float(x[0]), "last": float(x[-1]), "min": float(x.min()),
            "max": float(x.max()), "median": float(np.median(x)), "mean": float(x.mean())}


def summarize_training(train_csv: str, metrics_csv: str | None = None) -> dict:
    ts, step, loss = load_train_log(train_csv)
    out = {"loss": _stats(loss), "steps": int(step.size)}
    if ts.size > 1:
        out["seconds"] = float(ts[-1] - ts[0])
    if metrics_csv:
        m = load_hook_metrics(metrics_csv)
        out["ratio"] = _stats(m.get("ratio", np.array([])))
        if "res_mean_abs" in m:
            r = m["res_mean_abs"]
            out["res_mean_abs"] = _stats(r[np.isfinite(r)])
    return out


def summarize_hpc(path: str) -> dict:
    steps, ratios, errs = parse_hpc_log(path)
    return {"steps": int(steps.size), "ratio": _stats(ratios), "max_err": _stats(errs)}


def summarize_ticks(path: str) -> dict:
    t, r = load_tick_ratio_csv(path)
    return {"ticks": int(t.size), "ratio": _stats(r)}


def summarize_baselines(path: str) -> dict:
    """Per epsilon (empty for the general-purpose compressors): each tool's
    ratio and throughput, and the best ratio."""
    groups: dict = {}
    for r in load_baseline_rows(path):
        groups.setdefault(r.get("epsilon") or "", []).append(
            {"tool": r["tool"], "ratio": _float(r["ratio"]), "MBps": _float(r["throughput_MBps"])})
    return {eps or "general": {"tools": rs, "best_ratio": max(x["ratio"] for x in rs)} for eps, rs in groups.items()}


def _float(s, default: float = 0.0) -> float:
    try:
        return float(s)
    except (TypeError, ValueError):
        return default


def histogram_entropy(x: np.ndarray, bins: int = 100) -> float:
    """Shannon entropy (bits) of a ``bins``-bin histogram of x."""
    h, _ = np.histogram(np.asarray(x, np.float64), bins=bins)
    p = h[h > 0] / h.sum()
    return float(-(p * np.log2(p)).sum())


def ema_residual(x: np.ndarray, beta: float = 0.9) -> np.ndarray:
    """r_i = x_i - m_{i-1} with m = beta * m + (1 - beta) * x (m_{-1} = 0)."""
    x = np.asarray(x, np.float32)
    pred = np.empty_like(x)
    m = np.float32(0.0)
    b, omb = np.float32(beta), np.float32(1.0) - np.float32(beta)
    for i, v in enumerate(x):
        pred[i] = m
        m = b * m + omb * v
    return x - pred


def entropy_reduction(x: np.ndarray | None = None, beta: float = 0.9, bins: int = 100) -> dict:
    if x is None:
        t = np.arange(100000)
        x = (np.sin(t * 0.01) + 0.1 * np.sin(t * 0.05)
             + 0.01 * np.random.default_rng(0).standard_normal(t.size)).astype(np.float32)
    r = ema_residual(x, beta)
    return {"signal_entropy_bits": histogram_entropy(x, bins), "residual_entropy_bits": histogram_entropy(r, bins),
            "signal_std": float(np.std(x)), "residual_std": float(np.std(r)),
            "std_reduction": float(np.std(x) / max(np.std(r), 1e-30))}


# -------------------------------------------------------------------- plots
# Drawn by utils.plot (PNG or SVG by the output's extension); no plotting
# library is needed.
def plot_training(train_csv: str, metrics_csv: str, out: str = "train_and_compression.png") -> str:
    """Loss over time with the hook's compression ratio (and mean |residual|)
    on a second axis (python/nangila_ddp/plot_train_and_compression.py:8-95)."""
    from .plot import Figure

    ts, _, loss = load_train_log(train_csv)
    m = load_hook_metrics(metrics_csv)
    d_ts, ratio = m.get("ts", np.array([])), m.get("ratio", np.array([]))
    t0 = min(ts.min() if ts.size else math.inf, d_ts.min() if d_ts.size else math.inf)
    t0 = 0.0 if not math.isfinite(t0) else t0
    fig = Figure(900, 420)
    ax = fig.add_axes(title="training loss and compression", xlabel="time (s)", ylabel="loss")
    ax.line(ts - t0, loss, color="tab:blue", label="loss")
    ax2 = ax.twin(ylabel="compression ratio")
    ax2.points(d_ts - t0, ratio, color="tab:orange", alpha=0.3, label="ratio (raw/comp)")
    if ratio.size >= 10:
        k = max(1, ratio.size // 50)
        smooth = np.convolve(ratio, np.ones(k) / k, mode="same")
        ax2.line(d_ts - t0, smooth, color="tab:orange")
    return fig.save(out)


def plot_series(x, y, xlabel: str, ylabel: str, out: str, title: str = "", labels=None) -> str:
    """One or several y series against x (a list of arrays with ``labels``)."""
    from .plot import Figure

    fig = Figure(800, 400)
    ax = fig.add_axes(title=title, xlabel=xlabel, ylabel=ylabel)
    if labels is None:
        ax.line(x, y, marker=np.size(x) <= 200)
    else:
        for xi, yi, lab in zip(x, y, labels):
            ax.line(xi, yi, label=lab)
    return fig.save(out)


def plot_histogram(values, xlabel: str, out: str, bins: int = 20, title: str = "") -> str:
    from .plot import Figure

    v = np.asarray(values, float)
    v = v[np.isfinite(v)]
    counts, edges = np.histogram(v, bins=bins) if v.size else (np.zeros(1), np.array([0.0, 1.0]))
    fig = Figure(640, 400)
    ax = fig.add_axes(title=title, xlabel=xlabel, ylabel="count")
    centers = (edges[:-1] + edges[1:]) / 2
    ax.bars([f"{c:.3g}" if i % max(1, bins // 5) == 0 else "" for i, c in enumerate(centers)], counts)
    return fig.save(out)


def plot_hpc(log_path: str, out_prefix: str = "hpc") -> list[str]:
    """Ratio per step and the max-error histogram of an HPC bench log
    (python/snippets/plot_hpc_logs.py:22-46)."""
    steps, ratios, errs = parse_hpc_log(log_path)
    return [plot_series(steps, ratios, "step", "compression ratio (raw/comp)", f"{out_prefix}_ratio.png",
                        title="HPC compression ratio vs step"),
            plot_histogram(errs, "max error per step", f"{out_prefix}_eps_hist.png",
                           title="HPC max error distribution")]


def plot_twin(client_csv: str, server_csv: str | None = None, out: str = "rotor_net_ratio.png") -> str:
    """Client (and server) compression ratio per tick (python/snippets/plot_rotor_net.py:22-42)."""
    t, r = load_tick_ratio_csv(client_csv)
    xs, ys, labels = [t], [r], ["client ratio"]
    if server_csv:
        t2, r2 = load_tick_ratio_csv(server_csv)
        xs.append(t2)
        ys.append(r2)
        labels.append("server ratio")
    return plot_series(xs, ys, "tick", "compression ratio (raw/comp)", out, title="rotor twin network compression",
                       labels=labels)


def plot_entropy(out: str = "entropy_reduction.png", bins: int = 100) -> str:
    """Histograms of a signal and of its EMA-prediction residual, the
    reference's entropy illustration (python/snippets/entropy_plot.py:5-33)."""
    from .plot import Figure

    t = np.arange(100_000)
    x = (np.sin(t * 0.01) + 0.1 * np.sin(t * 0.05) + 0.01 * np.random.default_rng(0).standard_normal(t.size)
         ).astype(np.float32)
    r = ema_residual(x)
    fig = Figure(900, 640)
    for vals, name in ((x, "signal"), (r, "EMA residual")):
        counts, edges = np.histogram(vals, bins=bins)
        ax = fig.add_axes(title=f"{name}: entropy {histogram_entropy(vals, bins):.2f} bits", xlabel="value",
                          ylabel="count")
        ax.line((edges[:-1] + edges[1:]) / 2, counts)
    return fig.save(out)


def plot_baselines(csv_path: str, out: str = "baseline_comparison.png") -> str:
    """Ratio bars and throughput per tool, one panel per epsilon
    (benchmarks/plot_baselines.py)."""
    from .plot import Figure

    groups: dict = {}
    for r in load_baseline_rows(csv_path):
        groups.setdefault(r.get("epsilon") or "", []).append(r)
    if not groups:
        raise RuntimeError(f"no OK rows in {csv_path}")
    fig = Figure(900, 400 * len(groups))
    for eps, rs in groups.items():
        ax = fig.add_axes(title=f"baseline comparison (epsilon={eps})" if eps else "baseline comparison",
                          ylabel="ratio (raw/comp)")
        ax.bars([r["tool"] for r in rs], [_float(r["ratio"]) for r in rs], color="tab:blue", label="ratio")
        ax.twin(ylabel="throughput (MB/s)").line(range(len(rs)), [_float(r["throughput_MBps"]) for r in rs],
                                                 color="tab:orange", marker=True, label="throughput")
    return fig.save(out)
