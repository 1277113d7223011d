"""Error-bounded checkpoints of model / optimizer state (CPU path; the GPU
path is checked for identical bytes in test_tensor_ckpt_gpu)."""
import io

import pytest
import torch

from mini_nangila_b200.checkpoint import tensor_ckpt


def _state():
    torch.manual_seed(0)
    m = torch.nn.Sequential(torch.nn.Linear(64, 128), torch.nn.GELU(), torch.nn.Linear(128, 10))
    opt = torch.optim.AdamW(m.parameters(), lr=1e-3)
    x = torch.randn(32, 64)
    m(x).square().mean().backward()
    opt.step()
    return m, {"model": m.state_dict(), "optimizer": opt.state_dict()}


@pytest.mark.parametrize("codec", ["eb", "bs", "bsrle"])
def test_roundtrip_within_eps(codec, tmp_path):
    _, st = _state()
    eps = 1e-4
    p = tmp_path / "ck.nzt"
    info = tensor_ckpt.save(str(p), st, eps=eps, codec=codec)
    back = tensor_ckpt.load(str(p))
    flat = dict(tensor_ckpt._flatten(st)[0])
    assert set(flat) <= set(back)
    for k, v in flat.items():
        if v.dtype.is_floating_point:
            assert back[k].shape == v.shape and back[k].dtype == v.dtype
            assert float((back[k].float() - v.float()).abs().max()) <= eps * 1.01 + 1e-6, k
        else:
            assert torch.equal(back[k], v), k
    assert back["optimizer/param_groups/0/lr"] == 1e-3
    assert info["compressed"] < info["raw"]


def test_delta_against_previous_checkpoint(tmp_path):
    m, st0 = _state()
    eps = 1e-4
    b0 = io.BytesIO()
    tensor_ckpt.save(b0, st0, eps=eps, codec="bs")
    rec0 = tensor_ckpt.load(b0.getvalue())
    with torch.no_grad():  # a small training update
        for p in m.parameters():
            p.add_(torch.randn_like(p) * 1e-4)
    st1 = {"model": m.state_dict()}
    full = tensor_ckpt.save(io.BytesIO(), st1, eps=eps, codec="bs")
    b1 = io.BytesIO()
    delta = tensor_ckpt.save(b1, st1, eps=eps, codec="bs", base={"model": {k[6:]: v for k, v in rec0.items()
                                                                          if k.startswith("model/")}})
    assert delta["compressed"] < 0.8 * full["compressed"]
    back = tensor_ckpt.load(b1.getvalue(), base={"model": {k[6:]: v for k, v in rec0.items()
                                                           if k.startswith("model/")}})
    for k, v in st1["model"].items():
        assert float((back["model/" + k] - v).abs().max()) <= eps * 1.01 + 1e-6


def test_out_of_range_and_nonfinite_fall_back_to_raw():
    st = {"big": torch.tensor([1000.0, -3.0]), "inf": torch.tensor([float("inf"), 1.0]),
          "half": torch.randn(10).half(), "bf": torch.randn(7).bfloat16(), "step": torch.tensor(5)}
    b = io.BytesIO()
    info = tensor_ckpt.save(b, st, eps=1e-3)
    assert info["fallback_tensors"] == 2
    back = tensor_ckpt.load(b.getvalue())
    assert torch.equal(back["big"], st["big"]) and torch.equal(back["inf"], st["inf"])
    assert torch.equal(back["step"], st["step"])
    assert float((back["half"].float() - st["half"].float()).abs().max()) <= 1e-3 + 1e-3
    assert back["bf"].dtype == torch.bfloat16


def test_bad_magic():
    with pytest.raises(ValueError):
        tensor_ckpt.load(b"XXXX" + bytes(20))


@pytest.mark.gpu
@pytest.mark.parametrize("codec", ["eb", "bs", "bsrle"])
def test_gpu_encode_same_bytes(codec):
    _, st = _state()
    host = io.BytesIO()
    tensor_ckpt.save(host, st["model"], eps=1e-4, codec=codec)
    dev = io.BytesIO()
    tensor_ckpt.save(dev, {k: v.cuda() for k, v in st["model"].items()}, eps=1e-4, codec=codec)
    assert host.getvalue() == dev.getvalue()
    a = tensor_ckpt.load(host.getvalue())
    b = tensor_ckpt.load(host.getvalue(), device="cuda")
    for k in a:
        assert torch.equal(a[k], b[k])
