"""sm_100a fused compressed all-reduce vs the C++ host oracle (bitwise)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

SIZES = [1, 31, 255, 256, 257, 1000, 8 * 256 * 3 + 17, 65536 + 3]


def _ext():
    from mini_nangila_b200 import _ext

    return _ext.host(), _ext.cuda()


def _data(n, seed, scale=1e-3):
    g = np.random.default_rng(seed)
    x = (g.standard_normal(n) * scale).astype(np.float32)
    x[g.random(n) < 0.3] *= 0.01
    return x


def _bits(a):
    return np.asarray(a, dtype=np.float32).view(np.uint32)


@pytest.mark.parametrize("n", SIZES)
@pytest.mark.parametrize("mode", ["int4", "int8", "topk"])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("drop", [0.0, 0.4])
def test_encode_matches_oracle(n, mode, dtype, drop):
    from mini_nangila_b200.parallel.fused import topology

    h, c = _ext()
    topo = topology(n, drop, 11, 5)
    g = torch.from_numpy(_data(n, 1)).to(dtype)
    gf = g.float().numpy()
    pred = _data(n, 2)
    ef = _data(n, 3, 1e-4)
    dev = torch.device("cuda")
    mcode = {"int4": 0, "int8": 1, "topk": 2}[mode]
    k = 13
    out, ef_out = c.product_encode(g.to(dev), torch.from_numpy(pred).to(dev), torch.from_numpy(ef).to(dev),
                                   mcode, k, True, 777, 3, 5, 9, list(topo) if drop else [])
    if mode == "topk":
        wire, e_ref = h.product_topk_encode(gf, pred, ef, k, True, topo)
    else:
        wire, e_ref = h.product_encode(gf, pred, ef, 4 if mode == "int4" else 8, True, True, 777, 3, 5, 9, topo)
    assert bytes(out.cpu().numpy()) == bytes(wire)
    assert np.array_equal(_bits(ef_out.cpu().numpy()), _bits(e_ref))


@pytest.mark.parametrize("n", [257, 1000, 65536 + 3])
@pytest.mark.parametrize("mode", ["int4", "int8", "topk"])
def test_reduce_matches_oracle(n, mode):
    h, c = _ext()
    dev = torch.device("cuda")
    W = 3
    k = 26
    bits = 8 if mode == "int8" else 4
    mcode = {"int4": 0, "int8": 1, "topk": 2}[mode]
    pred = _data(n, 50)
    wires = []
    for r in range(W):
        g = _data(n, 10 + r)
        if mode == "topk":
            wire, _ = h.product_topk_encode(g, pred, None, k, False)
        else:
            wire, _ = h.product_encode(g, pred, None, bits, True, False, 1, r, 0, 0)
        wires.append(wire)
    payloads_dev = [torch.from_numpy(w).to(dev) for w in wires]
    inv = float(np.float32(1.0) / np.float32(W))
    state = torch.from_numpy(pred.copy()).to(dev)
    avg = c.product_reduce(payloads_dev, n, mcode, k, state, 0.9, False, inv, torch.float32)
    if mode == "topk":
        ref = h.product_topk_reduce(wires, n, k, pred, inv)
    else:
        ref = h.product_reduce(wires, n, bits, pred, inv)
    assert np.array_equal(_bits(avg.cpu().numpy()), _bits(ref))
    ema = h.product_ema(pred, ref, 0.9, False)
    assert np.array_equal(_bits(state.cpu().numpy()), _bits(ema))


@pytest.mark.parametrize("mode", ["int4", "int8", "topk"])
@pytest.mark.parametrize("n", [1000, 65536 + 3])
@pytest.mark.parametrize("drop", [0.0, 0.3])
def test_fused_single_rank_matches_oracle(mode, n, drop):
    from mini_nangila_b200.parallel.fused import FusedAllReduce, topology

    h, _ = _ext()
    dev = torch.device("cuda")
    comm = FusedAllReduce(n, device=dev)
    k = 26
    bits = 8 if mode == "int8" else 4
    pred = _data(n, 7)
    ef = _data(n, 8, 1e-4)
    pred_d, ef_d = torch.from_numpy(pred.copy()).to(dev), torch.from_numpy(ef.copy()).to(dev)
    for step in range(3):
        g = _data(n, 100 + step)
        gd = torch.from_numpy(g).to(dev)
        comm.allreduce_(gd, pred_d, ef_d, mode=mode, k=k, seed=42, bucket=2, step=step, beta=0.9, first=(step == 0),
                        topo_drop=drop, topo_seed=17)
        topo = topology(n, drop, 17, 2)
        if mode == "topk":
            rec, e_new = h.product_topk_encode(g, pred, ef, k, True, topo)
            avg = h.product_topk_reduce([rec], n, k, pred, 1.0)
        else:
            wire, e_new = h.product_encode(g, pred, ef, bits, True, True, 42, 0, 2, step, topo)
            avg = h.product_reduce([wire], n, bits, pred, 1.0)
        pred = h.product_ema(pred, avg, 0.9, step == 0)
        ef = e_new
        assert np.array_equal(_bits(gd.cpu().numpy()), _bits(avg)), f"avg mismatch at step {step}"
        assert np.array_equal(_bits(pred_d.cpu().numpy()), _bits(pred))
        assert np.array_equal(_bits(ef_d.cpu().numpy()), _bits(ef))
    comm.check()


def _two_rank_emulation(n, mode, k, bad_tag=False, deliver=True, timeout_s=0.2, drop=0.0):
    """Rank 0 of a 2-rank one-shot all-reduce on one GPU, rank 1's payload
    and column flags pre-delivered (parallel/emulate.py)."""
    from mini_nangila_b200.parallel import emulate

    r = emulate.oneshot(n, mode, k, drop=drop, bad_tag=bad_tag, deliver=deliver, timeout_s=timeout_s)
    return r["status"], r["avg"], r["ref_avg"]


@pytest.mark.parametrize("mode", ["int4", "int8", "topk"])
@pytest.mark.parametrize("drop", [0.0, 0.5])
def test_oneshot_kernel_with_predelivered_peer(mode, drop):
    st, out, ref = _two_rank_emulation(50000, mode, 13, drop=drop)
    assert st[0] == 0, st
    assert np.array_equal(_bits(out), _bits(ref))


def test_wait_times_out_and_reports_status():
    """A flag that nothing sets: the bounded wait gives up, records the status
    and the context stays usable."""
    st, _, _ = _two_rank_emulation(5000, "int4", 13, deliver=False, timeout_s=0.05)
    assert st[0] == 1, st  # timeout waiting for a peer's payload
    x = torch.ones(10, device="cuda")
    assert float(x.sum()) == 10.0


def test_bad_tag_is_reported():
    st, _, _ = _two_rank_emulation(5000, "int4", 13, bad_tag=True)
    assert st[0] == 3, st


@pytest.mark.parametrize("n", [2048, 4096, 65539, 1 << 20])
@pytest.mark.parametrize("grid", [1, 3, 33, 148])
@pytest.mark.parametrize("vec", [False, True])
def test_prefetch_pipeline_copies_every_chunk(n, grid, vec):
    _, c = _ext()
    src = torch.randn(n, device="cuda")
    status = torch.zeros(4, dtype=torch.int32, device="cuda")
    dst = c.pipe_copy(src, grid, status, vec)
    torch.cuda.synchronize()
    assert status.tolist()[0] == 0
    assert torch.equal(dst, src)


def _twoshot_emulation(n, mode, world, drop=0.0, grid_cap=0):
    """Rank 0 of a ``world``-rank two-shot all-reduce on one GPU: ranks
    world-1 .. 1 run first with everything they wait for pre-delivered, and
    their stores fill rank 0's region (parallel/emulate.py)."""
    from mini_nangila_b200.parallel import emulate

    r = emulate.twoshot(n, mode, world, drop, grid_cap)
    return (r["status"], r["avg"], r["pred"], r["ef"]), r["ref_avg"], r["ref_pred"], r["ref_ef"]


@pytest.mark.parametrize("mode", ["int4", "int8"])
@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("n,drop,cap", [(70001, 0.0, 0), (70001, 0.4, 0), (300_000, 0.0, 7)])
def test_twoshot_kernel_with_predelivered_peers(mode, world, n, drop, cap):
    (st, out, pred_out, ef_out), avg, pred_ref, ef_ref = _twoshot_emulation(n, mode, world, drop, cap)
    assert st[0] == 0, st
    assert np.array_equal(_bits(out), _bits(avg)), int(np.sum(_bits(out) != _bits(avg)))
    assert np.array_equal(_bits(pred_out), _bits(pred_ref))
    assert np.array_equal(_bits(ef_out), _bits(ef_ref))


@pytest.mark.parametrize("world", [2, 8])
def test_twoshot_kernel_applies_adamw_in_its_decode_phase(world):
    """AdamW fused into the two-shot kernel's decode phase: with the
    kernel's own averaged gradient (bit-identical to the oracle's), the
    parameters and moments match a float64 AdamW step, on four parameters
    of which one boundary is off the 8-element grid."""
    from mini_nangila_b200.parallel import emulate

    r = emulate.twoshot(70001, "int4", world, optimizer=True)
    assert r["status"][0] == 0
    assert emulate.bit_equal(r["avg"], r["ref_avg"])
    g = r["ref_avg"]
    b1, b2 = r["opt_hyper"][:2]
    ulp = 2.0 ** -24
    for a, b, p, m, v, (p0, m0, v0) in r["opt"]:
        rp, rm, rv = emulate.adamw_reference(p0, m0, v0, g[a:b], r["opt_hyper"])
        gg = np.asarray(g[a:b], np.float64)
        # fp32 error of each moment relative to the size of its two terms:
        # b1*m0 and (1-b1)*g may nearly cancel, so the error bound is a few
        # ulps of the terms, not of the result
        assert np.all(np.abs(m - rm) <= 4 * ulp * (b1 * np.abs(m0) + (1 - b1) * np.abs(gg)) + 1e-30)
        assert np.all(np.abs(v - rv) <= 4 * ulp * (b2 * v0 + (1 - b2) * gg * gg) + 1e-36)
        assert np.allclose(p, rp, rtol=0, atol=1e-7)
        assert np.abs(p - p0).max() > 1e-5  # the step moved the weights (updates are ~5e-5 here)
