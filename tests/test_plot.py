"""utils.plot (PNG / SVG charts without a plotting library) and the log plots
of utils.analysis that use it: the reference's plot scripts
(python/nangila_ddp/plot_train_and_compression.py, python/snippets/
plot_hpc_logs.py, plot_rotor_net.py, entropy_plot.py,
benchmarks/plot_baselines.py) produce these figures."""
import xml.etree.ElementTree as ET

import numpy as np

from mini_nangila_b200.utils import analysis
from mini_nangila_b200.utils.plot import COLORS, Figure, nice_ticks, png_bytes, read_png


def test_png_encoder_round_trip():
    img = (np.random.default_rng(0).integers(0, 256, (17, 23, 3))).astype(np.uint8)
    assert np.array_equal(read_png(png_bytes(img)), img)


def test_nice_ticks():
    assert nice_ticks(0.0, 10.0) == [0, 2, 4, 6, 8, 10]
    t = nice_ticks(0.013, 0.047)
    assert t[0] >= 0.013 - 1e-12 and t[-1] <= 0.047 + 1e-12 and len(t) >= 3
    assert len(nice_ticks(5.0, 5.0)) >= 1


def test_line_chart_pixels_and_svg(tmp_path):
    fig = Figure(400, 300)
    ax = fig.add_axes(title="loss", xlabel="step", ylabel="loss")
    x = np.arange(50)
    ax.line(x, np.exp(-x / 10.0), color="tab:blue", label="train")
    ax.twin(ylabel="ratio").points(x, 8 + np.sin(x), color="tab:orange")
    img = read_png(open(fig.save(str(tmp_path / "a.png")), "rb").read())
    assert img.shape == (300, 400, 3)
    blue = np.all(img == np.array(COLORS["tab:blue"], np.uint8), axis=-1)
    black = np.all(img == 0, axis=-1)
    assert blue.sum() > 200 and black.sum() > 500  # the curve, the frame and the text
    # the curve falls from left to right: its leftmost ink is above its rightmost
    ys, xs = np.nonzero(blue)
    assert ys[xs.argmin()] < ys[xs.argmax()]
    root = ET.fromstring(open(fig.save(str(tmp_path / "a.svg"))).read())
    tags = [el.tag.split("}")[-1] for el in root.iter()]
    assert tags.count("polyline") >= 2 and tags.count("circle") == 50 and "text" in tags


def test_analysis_plots(tmp_path, monkeypatch):
    monkeypatch.chdir(tmp_path)
    t = tmp_path / "train_log.csv"
    t.write_text("ts,step,loss,lr,tokens_per_sec,step_ms\n" +
                 "".join(f"{100 + i},{i},{4 - i * 0.01},0.0006,1000,10\n" for i in range(100)))
    m = tmp_path / "ddp_metrics.csv"
    m.write_text("".join(f"ts,{100.5 + i},hook_idx,{i},bucket_elems,10,raw_bytes,40,comp_bytes,5,ratio,{8 + i % 3},"
                         f"res_mean_abs,1e-3\n" for i in range(60)))
    h = tmp_path / "hpc.log"
    h.write_text("".join(f"step {i} ratio {2 + 0.01 * i:.3f} bytes 100 max_err {0.0009 + 1e-6 * i:.7f}\n"
                         for i in range(40)))
    c = tmp_path / "client.csv"
    c.write_text("tick,bytes,ratio\n" + "".join(f"{i},16,{1.5}\n" for i in range(30)))
    b = tmp_path / "base.csv"
    b.write_text("tool,epsilon,codec,compressed_bytes,ratio,comp_time_s,throughput_MBps,status\n"
                 "gzip-6,,gzip,100,1.1,0.5,200,OK\nnz-eb,0.001,EB,50,2.0,0.1,900,OK\n")
    outs = [analysis.plot_training(str(t), str(m)), *analysis.plot_hpc(str(h)),
            analysis.plot_twin(str(c), str(c)), analysis.plot_entropy(), analysis.plot_baselines(str(b), "b.png"),
            analysis.plot_series(np.arange(5), np.arange(5), "x", "y", "s.svg")]
    for o in outs:
        data = open(o, "rb").read()
        if o.endswith(".png"):
            img = read_png(data)
            assert img.ndim == 3 and (img != 255).any()
        else:
            ET.fromstring(data.decode())
