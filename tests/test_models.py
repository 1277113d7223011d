"""Model definitions used by the benchmarks (CPU, tiny configs): causal
language models (no position sees a later token), loss equal to the
cross-entropy of the logits, grouped-query attention shapes, and the
reference trainer's TinyGPT (non-causal by default, as the reference)."""
import pytest
import torch
import torch.nn.functional as F

from mini_nangila_b200.models import GPT2, GPT2Config, Llama, LlamaConfig
from mini_nangila_b200.models.tinygpt import TinyGPT


def _model(kind):
    torch.manual_seed(0)
    return GPT2(GPT2Config.tiny()) if kind == "gpt2" else Llama(LlamaConfig.tiny())


@pytest.mark.parametrize("kind", ["gpt2", "llama"])
def test_causal_and_loss(kind):
    m = _model(kind).eval()
    g = torch.Generator().manual_seed(1)
    x = torch.randint(0, 512, (2, 24), generator=g)
    y = torch.randint(0, 512, (2, 24), generator=g)
    with torch.no_grad():
        logits = m(x)
        assert logits.shape == (2, 24, 512)
        x2 = x.clone()
        x2[:, 12:] = torch.randint(0, 512, (2, 12), generator=g)
        logits2 = m(x2)
        # positions before the change see nothing after it
        assert torch.allclose(logits[:, :12], logits2[:, :12], atol=1e-5)
        assert not torch.allclose(logits[:, 12:], logits2[:, 12:])
        loss = m(x, y)
        assert torch.allclose(loss, F.cross_entropy(logits.reshape(-1, 512).float(), y.reshape(-1)), atol=1e-5)


@pytest.mark.parametrize("kind", ["gpt2", "llama"])
def test_backward_reaches_every_parameter(kind):
    m = _model(kind)
    x = torch.randint(0, 512, (2, 16))
    m(x, x).backward()
    assert all(p.grad is not None and torch.isfinite(p.grad).all() for p in m.parameters())


def test_llama_grouped_query_shapes():
    cfg = LlamaConfig.tiny()
    m = Llama(cfg)
    kv = cfg.n_kv_head * (cfg.d_model // cfg.n_head)
    shapes = sorted({tuple(p.shape) for p in m.parameters()})
    assert (kv, cfg.d_model) in shapes and (cfg.d_model, cfg.d_model) in shapes


def test_tinygpt_is_non_causal_by_default_and_causal_on_request():
    torch.manual_seed(0)
    x = torch.randint(0, 100, (1, 10))
    x2 = x.clone()
    x2[0, 9] = (x[0, 9] + 1) % 100
    for causal, first_changes in ((False, True), (True, False)):
        m = TinyGPT(d_model=32, nhead=4, nlayers=1, vocab=100, block_size=16, causal=causal).eval()
        with torch.no_grad():
            a, b = m(x), m(x2)
        assert (not torch.allclose(a[0, 0], b[0, 0], atol=1e-6)) == first_changes
