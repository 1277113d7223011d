"""Model configurations and app defaults agree with the workload dataclasses."""
import inspect

from mini_nangila_b200 import workloads as W
from mini_nangila_b200.models import GPT2Config, LlamaConfig


def test_gpt2_small_matches_workload():
    w, c = W.GPT2SmallDDP(), GPT2Config.small()
    assert (c.n_layer, c.n_embd, c.n_head, c.vocab_size) == (w.n_layer, w.d_model, w.n_head, w.vocab)
    assert (c.n_inner or 4 * c.n_embd) == w.d_ff and c.n_positions >= w.seq


def test_llama_matches_workload():
    w, c = W.Llama1BTopK(), LlamaConfig.b1_1()
    assert (c.n_layer, c.d_model, c.n_head, c.n_kv_head, c.d_ff, c.vocab_size) == (
        w.n_layer, w.d_model, w.n_head, w.n_kv_head, w.d_ff, w.vocab)
    assert c.max_seq >= w.seq


def test_app_defaults_match_workloads():
    from mini_nangila_b200.apps import allreduce_bench, codec_bench, mode_switching

    src = inspect.getsource(codec_bench.main)
    t = W.TrajectoryCodec()
    assert f"default={t.atoms:_}" in src.replace("1_000_000", f"{t.atoms:_}") and f"default={t.steps}" in src
    sw = W.AllReduceSweep()
    src = inspect.getsource(allreduce_bench.main)
    assert ",".join(str(x) for x in sw.sizes_mb) in src and f"default={sw.steps}" in src
    m = W.ModeSwitchingAR1()
    sig = inspect.signature(mode_switching.ar1_gradients)
    assert sig.parameters["rho"].default == m.rho and sig.parameters["sigma"].default == m.sigma
    assert sig.parameters["sigma0"].default == m.sigma0 and sig.parameters["sparse_frac"].default == m.sparse_frac
