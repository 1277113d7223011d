"""The reference package's module paths (python/nangila_ddp/*) resolve to
this framework: the hook, the trainers and the two plot scripts."""
import importlib


def test_module_paths():
    import nangila_ddp
    from mini_nangila_b200.apps import minigpt_train, train_nano
    from mini_nangila_b200.parallel.hook import register_nangila_hook

    assert nangila_ddp.register_nangila_hook is register_nangila_hook
    assert importlib.import_module("nangila_ddp.comm_hook").register_nangila_hook is register_nangila_hook
    assert importlib.import_module("nangila_ddp.train_nano").main is train_nano.main
    assert importlib.import_module("nangila_ddp.examples.minigpt_train").main is minigpt_train.main


def test_plot_scripts_plot_and_summarise(tmp_path, capsys, monkeypatch):
    from nangila_ddp import plot_metrics, plot_train_and_compression

    m = tmp_path / "ddp_metrics.csv"
    m.write_text("ts,100.5,hook_idx,1,bucket_elems,10,raw_bytes,40,comp_bytes,5,ratio,8.0,res_mean_abs,1e-3\n"
                 "ts,101.5,hook_idx,2,bucket_elems,10,raw_bytes,40,comp_bytes,4,ratio,10.0,res_mean_abs,2e-3\n")
    t = tmp_path / "train_log.csv"
    t.write_text("ts,step,loss,lr,tokens_per_sec,step_ms\n100.0,1,4.2,0.0006,1000,10\n101.0,2,4.0,0.0006,1000,10\n")
    monkeypatch.chdir(tmp_path)
    assert plot_metrics.main([str(m)]).endswith("_ratio.png")
    assert plot_train_and_compression.main([str(t), str(m)]) == "train_and_compression.png"
    out = capsys.readouterr().out
    assert "Saved" in out and '"median": 9.0' in out and '"loss"' in out
    assert (tmp_path / "train_and_compression.png").read_bytes()[:8] == b"\x89PNG\r\n\x1a\n"
    empty = tmp_path / "empty.csv"
    empty.write_text("nothing here\n")
    assert plot_metrics.main([str(empty)]) is None


def test_package_metadata_and_lazy_subpackages():
    import sys

    import mini_nangila_b200 as m

    assert m.__version__ == "0.1.0"
    assert m.core.FixedPointBuffer is sys.modules["mini_nangila_b200.core"].FixedPointBuffer
    assert "parallel" in m.__all__
