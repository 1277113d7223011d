"""CLI apps (ports of the reference's example binaries) and the gRPC twin."""
import os
import struct

import numpy as np
import pytest

from mini_nangila_b200.apps import (checkpoint_demo, cpu_compression_bench, hpc_compress_bench, lammps_compress,
                                    mode_switching, nano_gpt, rotor_twin, throughput_bench, topology_calibration)


def test_mode_switching_ar1_block_int4_deterministic():
    a = mode_switching.run(generator="ar1", train="block-int4", checkpoint_codec="eb", verbose=False)
    b = mode_switching.run(generator="ar1", train="block-int4", checkpoint_codec="eb", verbose=False)
    assert a["determinism_hash"] == b["determinism_hash"]
    assert a["max_checkpoint_err"] <= 1e-3 + 1e-6
    assert 4.0 < a["ratio"] < 12.0


def test_mode_switching_reference_defaults():
    out = mode_switching.run(verbose=False)
    assert out["ratio"] > 4.0 and out["max_checkpoint_err"] <= 1e-3 + 1e-6


def test_lammps_cli_roundtrip(tmp_path):
    p = str(tmp_path / "c.nz")
    d = str(tmp_path / "d.dump")
    lammps_compress.main(["--generate", d, "--particles", "200", "--steps", "4"])
    st = lammps_compress.main(["--input", d, "--output", p, "--use-block-sparse-rle"])
    assert st["max_abs_err"] <= 1e-3 + 1e-6
    vals = lammps_compress.main(["--decompress", "--output", p])
    assert vals.size == 600 * 4
    st2 = lammps_compress.main(["--output", p, "--particles", "5000", "--steps", "5"])
    assert st2["total_raw"] == 5000 * 5 * 4


def test_benches_reach_reference_targets():
    out = cpu_compression_bench.main([])
    assert out["topk"][0] > 18.0 and out["rle"][0] > 50.0
    h = hpc_compress_bench.main(["--particles", "20000", "--steps", "20"])
    assert h["ok"] and h["ratio"] >= 1.9
    t = throughput_bench.main(["--dim", "65536", "--steps", "10"])
    assert t["ratio"] > 7.0


def test_topology_calibration_file(tmp_path):
    p = str(tmp_path / "m.bin")
    m = topology_calibration.main(["--output", p])
    b = open(p, "rb").read()
    assert len(b) == 124 and struct.unpack_from("<Q", b, 0)[0] == len(m.driver_indices) == 9


def test_checkpoint_demo(tmp_path):
    err = checkpoint_demo.main(["--output", str(tmp_path / "c.h5"), "--len", "20000"])
    assert err <= 1e-3 + 1e-6


def test_rotor_twin_and_nano_gpt():
    ratio, rms = rotor_twin.main(["--duration", "2", "--rate-hz", "50", "--no-sleep"])
    assert ratio > 1.4 and rms < 0.05
    r = nano_gpt.main(["--num-steps", "3", "--hidden", "64", "--calibration-steps", "5"])
    assert r > 5.0


def test_grpc_twin_end_to_end(tmp_path):
    grpc = pytest.importorskip("grpc")  # noqa: F841
    from mini_nangila_b200.twin.rotor_net import (Frame, RotorClient, RotorServer, _f32_display, decode_ack, encode_ack,
                                                  imu_sample)

    f = Frame(7, 6, -0.5, b"\x01\x02\x03")
    assert Frame.decode(f.encode()) == f and decode_ack(encode_ack(True)) is True
    for topk in (0.0, 0.5):
        srv = RotorServer(metrics_path=str(tmp_path / f"s{topk}.csv"))
        server, port = srv.serve("127.0.0.1:0")
        try:
            c = RotorClient(f"127.0.0.1:{port}", topk=topk, metrics_path=str(tmp_path / f"c{topk}.csv"))
            for tick in range(40):
                x = imu_sample(tick / 50)
                assert c.send(x, tick)
                # the client's closed loop matches what the server reconstructed
                assert np.array_equal(c.pred.predict().to_f32(), srv.pred.predict().to_f32())
            if topk == 0.0:
                assert np.abs(srv.last - imu_sample(39 / 50)).max() <= 0.05 + 1e-6
            c.close()
        finally:
            server.stop(0)
        assert srv.frames == 40
        lines = open(tmp_path / f"s{topk}.csv").read().splitlines()
        assert lines[0].startswith("tick,0,len,6,raw,24,comp,")
        # the ratio columns as the Rust programs print an f32: "{:.4}" on the
        # server (server.rs:74), "{}" on the client (client.rs:124)
        for line in lines:
            f = line.split(",")
            assert f[9] == f"{float(np.float32(int(f[5])) / np.float32(int(f[7]))):.4f}"
        rows = open(tmp_path / f"c{topk}.csv").read().splitlines()
        assert rows[0] == "tick,len,raw,comp,ratio" and len(rows) == 41
        for row in rows[1:]:
            t, n, raw, comp, ratio = row.split(",")
            assert ratio == _f32_display(np.float32(int(raw)) / np.float32(int(comp)))
            assert not ratio.endswith(".0")
    assert [_f32_display(np.float32(a) / np.float32(b)) for a, b in ((24, 12), (24, 14), (1, 3))] == \
        ["2", "1.7142857", "0.33333334"]


def test_grpc_server_under_concurrent_clients(tmp_path):
    """Frames from several client threads at once (the server's handler runs
    on a thread pool): every frame is counted and every CSV line is whole."""
    pytest.importorskip("grpc")
    import threading

    from mini_nangila_b200.twin.rotor_net import RotorClient, RotorServer, imu_sample

    srv = RotorServer(metrics_path=str(tmp_path / "s.csv"))
    server, port = srv.serve("127.0.0.1:0", max_workers=8)
    errors = []

    def client(k):
        try:
            c = RotorClient(f"127.0.0.1:{port}")
            for tick in range(25):
                assert c.send(imu_sample((100 * k + tick) / 50), 100 * k + tick)
            c.close()
        except Exception as e:  # noqa: BLE001
            errors.append(e)

    try:
        ts = [threading.Thread(target=client, args=(k,)) for k in range(4)]
        for t in ts:
            t.start()
        for t in ts:
            t.join()
    finally:
        server.stop(0)
    assert not errors and srv.frames == 100
    lines = open(tmp_path / "s.csv").read().splitlines()
    assert len(lines) == 100 and all(line.startswith("tick,") and line.count(",") == 9 for line in lines)
    assert sorted(int(line.split(",")[1]) for line in lines) == sorted(100 * k + t for k in range(4) for t in range(25))


def test_grpc_twin_cli_apps(tmp_path):
    """The server and client CLIs with the reference's flags (the client
    takes the reference's ``http://`` address form)."""
    pytest.importorskip("grpc")
    import socket
    import subprocess
    import sys

    from mini_nangila_b200.apps import rotor_twin_client

    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    srv = subprocess.Popen([sys.executable, "-u", "-m", "mini_nangila_b200.apps.rotor_twin_server", "--listen",
                            f"127.0.0.1:{port}", "--metrics", str(tmp_path / "s.csv")], cwd=root,
                           stdout=subprocess.PIPE, text=True)
    try:
        assert "listening" in srv.stdout.readline()
        rotor_twin_client.main(["--server", f"http://127.0.0.1:{port}", "--duration", "1", "--rate-hz", "20",
                                "--metrics", str(tmp_path / "c.csv")])
    finally:
        srv.terminate()
        srv.wait(timeout=30)
    n_client = len(open(tmp_path / "c.csv").read().splitlines())
    n_server = len(open(tmp_path / "s.csv").read().splitlines())
    assert n_client >= 10 and n_server >= 10 and abs(n_client - n_server) <= 1


def test_train_nano_two_cpu_ranks(tmp_path):
    import socket
    import subprocess
    import sys

    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    log = tmp_path / "train_log.csv"
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(port), "-m", "mini_nangila_b200.apps.train_nano",
           "--device", "cpu", "--steps", "3", "--d_model", "32", "--nhead", "2", "--nlayers", "1",
           "--batch_size", "4", "--block_size", "16", "--use_momentum", "--train_log", str(log),
           "--metrics_path", str(tmp_path / "m.csv")]
    env = dict(os.environ, PYTHONPATH=os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=300, env=env)
    assert r.returncode == 0, r.stderr[-2000:]
    rows = log.read_text().splitlines()
    assert rows[0] == "ts,step,loss,lr,tokens_per_sec,step_ms" and len(rows) == 4
    m = (tmp_path / "m.csv").read_text().splitlines()
    assert m and m[0].startswith("ts,") and ",ratio," in m[0]


def test_determinism_hash_app():
    from mini_nangila_b200.apps import determinism_hash

    assert determinism_hash.main([]) == "c18cd836f0cb712247e0ace683d710b8550f3e3f40a6a2998252df59498aab56"


def test_verify_app_reproduces_the_reference_artifacts(tmp_path):
    import json

    from mini_nangila_b200.apps import verify

    out = str(tmp_path / "verification")
    checks = verify.main(["--out", out, "--skip-tests", "--quick"])
    assert all(c["ok"] for c in checks.values())
    assert checks["rotor"]["ratio"] == 1.5 and checks["rotor"]["rms_err"] == 0.02304  # reference: rotor.txt
    assert checks["topology"]["mask_bytes"] == 124
    for f in ("determinism_hash.txt", "ai_throughput.txt", "hpc_bench.txt", "topology.txt", "rotor.txt"):
        assert os.path.getsize(os.path.join(out, f)) > 0
    assert json.load(open(os.path.join(out, "checks.json"))) == json.loads(json.dumps(checks))
    assert open(os.path.join(out, "determinism_hash.txt")).read().strip() == f"Q823_HASH {verify.REFERENCE_HASH}"


def test_analyze_app(tmp_path):
    from mini_nangila_b200.apps import analyze

    tr = tmp_path / "train_log.csv"
    tr.write_text("ts,step,loss,tokens_per_s\n100.0,0,4.2,1000\n101.0,1,3.9,1100\n102.0,2,3.5,1200\n")
    mt = tmp_path / "ddp_metrics.csv"
    mt.write_text("ts,100.5,hook_idx,1,bucket_elems,10,raw_bytes,40,comp_bytes,5,ratio,8.0,res_mean_abs,1e-3\n"
                  "ts,101.5,hook_idx,2,bucket_elems,10,raw_bytes,40,comp_bytes,4,ratio,10.0,res_mean_abs,2e-3\n"
                  "step,3,bucket_elems,10,raw_bytes,40,comp_bytes,4,ratio,10.0\n")
    out = analyze.main(["train", str(tr), str(mt)])
    assert out["loss"]["first"] == 4.2 and out["loss"]["last"] == 3.5 and out["seconds"] == 2.0
    assert out["ratio"]["n"] == 3 and out["ratio"]["max"] == 10.0
    hp = tmp_path / "hpc.log"
    hp.write_text("step 0 ratio 2.00 raw 400 max_err 0.0009\nnoise\nstep 1 ratio 2.5 raw 400 max_err 0.001\n")
    out = analyze.main(["hpc", str(hp)])
    assert out["steps"] == 2 and out["ratio"]["median"] == 2.25
    tw = tmp_path / "client.csv"
    tw.write_text("tick,raw,comp,ratio\n0,24,16,1.5\n1,24,12,2.0\n")
    out = analyze.main(["twin", str(tw)])
    assert out["client"]["ratio"]["mean"] == 1.75
    out = analyze.main(["entropy"])
    assert out["std_reduction"] > 2.0


def test_analyze_reads_checkpoint(tmp_path):
    import numpy as np

    from mini_nangila_b200.apps import analyze
    from mini_nangila_b200.checkpoint import hdf5

    x = np.linspace(-1, 1, 5000, dtype=np.float32)
    p = str(tmp_path / "ck.h5")
    hdf5.write_chunked_dataset(p, "w", x, 1024, 1e-3, "eb")
    out = analyze.main(["checkpoint", p, "w"])
    assert out["n"] == 5000 and abs(out["first"][0] + 1.0) <= 1e-3


def test_rotor_topk_codes_round_half_away_from_zero():
    """The top-k path rounds the f32 quotient as Rust's f32::round does
    (rotor_twin_net client.rs:99): 0.25 / 0.1 is 2.5 in f32 and codes as 3."""
    pytest.importorskip("grpc")
    from mini_nangila_b200.hpc import rle_decode_i16
    from mini_nangila_b200.twin.rotor_net import RotorClient

    for v, h in ((0.25, 2.5), (0.75, 7.5)):
        assert np.float32(v) / np.float32(0.1) == np.float32(h)
    c = RotorClient("127.0.0.1:1", epsilon=0.05, topk=0.5)
    frame, _ = c.encode(np.array([0.25, -0.25, 0.75, 0.0, 0.125, 0.0], np.float32), 0)
    assert frame.scale == -float(np.float32(0.1))
    assert rle_decode_i16(frame.residual).tolist() == [3, -3, 8, 0, 0, 0]
    c.close()
    c = RotorClient("127.0.0.1:1", epsilon=1e-3, topk=0.34)  # k = 2; codes clamp at the i16 ends
    frame, _ = c.encode(np.array([200.0, -200.0, 1.0, 0.0, 0.0, 0.0], np.float32), 0)
    assert rle_decode_i16(frame.residual).tolist() == [32767, -32768, 0, 0, 0, 0]
    c.close()


def test_loss_curves_app_two_cpu_ranks(tmp_path):
    """apps.loss_curves on two gloo ranks with a tiny GPT-2: every setting
    starts from the same loss (same weights and batches) and the summary
    names its difference to the uncompressed all-reduce."""
    import json
    import socket
    import subprocess
    import sys

    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    out = tmp_path / "curves.json"
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(port), "-m", "mini_nangila_b200.apps.loss_curves",
           "--tiny", "--steps", "4", "--micro-batch", "2", "--seq", "16", "--warmup", "2",
           "--settings", "nccl,int4-oneshot,topk5,compat", "--out", str(out), "--log-dir", str(tmp_path)]
    env = dict(os.environ, PYTHONPATH=os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600, env=env)
    assert r.returncode == 0, r.stderr[-3000:]
    res = json.loads(out.read_text())
    curves = res["curves"]
    assert set(curves) == {"nccl", "int4-oneshot", "topk5", "compat"}
    first = {k: v[0] for k, v in curves.items()}
    assert max(first.values()) - min(first.values()) < 1e-5  # same weights, same first batch
    assert res["summary"]["nccl"]["delta_vs_nccl"] == 0.0
    assert (tmp_path / "train_log_topk5.csv").read_text().startswith("ts,step,loss,lr,tokens_per_sec,step_ms")
