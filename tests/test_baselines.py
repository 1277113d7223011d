"""LAMMPS dump I/O in the native host library
(examples/lammps_compress/src/main.rs:324-419) and the compression-baseline
app (benchmarks/run_baselines.sh, benchmarks/plot_baselines.py)."""
import csv
import os

import numpy as np
import pytest

from mini_nangila_b200.apps import baselines
from mini_nangila_b200.checkpoint import lammps, nzcp
from mini_nangila_b200.utils import analysis

HDR = "ITEM: TIMESTEP\n{t}\nITEM: NUMBER OF ATOMS\n{n}\nITEM: BOX BOUNDS xx yy zz\n0 10\n0 10\n0 10\n"


def _dump(rows, fields="id type x y z", t=0):
    return HDR.format(t=t, n=len(rows)) + f"ITEM: ATOMS {fields}\n" + "".join(r + "\n" for r in rows)


def test_columns_located_by_name_and_snapshots_of_any_size():
    text = _dump(["1 1 3 2 1", "2 1 6 5 4"], fields="id type z y x") + "junk line\n" + _dump(["7 2 1.5 2.5 3.5"], t=5)
    snaps = lammps.read_dump_text(text)
    assert [s.tolist() for s in snaps] == [[1, 2, 3, 4, 5, 6], [1.5, 2.5, 3.5]]


def test_float_grammar_is_rusts():
    rows = ["1 1 +2.5 .5 5.", "2 1 1e40 -1e-50 1e-40", "3 1 inf -Infinity NaN"]
    s = lammps.read_dump_text(_dump(rows))[0]
    assert s[:3].tolist() == [2.5, 0.5, 5.0]
    assert s[3] == np.inf and s[4] == 0.0 and np.signbit(s[4]) and s[5] == np.float32(1e-40)
    assert s[6] == np.inf and s[7] == -np.inf and np.isnan(s[8])
    # correctly rounded: same bits as numpy's parse
    vals = ["0.808028", "-0.000001", "3.4028234e38", "1.17549435e-38", "0.1", "123456.789"]
    got = lammps.read_dump_text(_dump([f"1 1 {v} 0 0" for v in vals]))[0][0::3]
    assert np.array_equal(got.view(np.uint32), np.array([np.float32(v) for v in vals]).view(np.uint32))
    for bad in ["0x1p3", "1e", "--1", "+-1", ".", "1.2.3", "1,5", "e5"]:
        with pytest.raises(lammps.DumpFormatError, match="x parse"):
            lammps.read_dump_text(_dump([f"1 1 {bad} 0 0"]))


@pytest.mark.parametrize("text, msg", [
    ("ITEM: TIMESTEP\n0\nITEM: ATOMS\n", "expected NUMBER OF ATOMS line"),
    ("ITEM: TIMESTEP\n0\nITEM: NUMBER OF ATOMS\nx\n", "parse natoms"),
    ("ITEM: TIMESTEP\n0\nITEM: NUMBER OF ATOMS\n-1\n", "parse natoms"),
    ("ITEM: TIMESTEP\n0\nITEM: NUMBER OF ATOMS\n1\nBOX\n", "expected BOX BOUNDS line"),
    (HDR.format(t=0, n=1) + "ATOMS id x y z\n", "expected ATOMS header"),
    (HDR.format(t=0, n=1) + "ITEM: ATOMS id y z\n", "x column not found"),
    (HDR.format(t=0, n=1) + "ITEM: ATOMS id x z\n", "y column not found"),
    (HDR.format(t=0, n=2) + "ITEM: ATOMS id x y z\n1 0 0 0\n", "unexpected EOF reading atoms"),
    (HDR.format(t=0, n=1) + "ITEM: ATOMS id type x y z\n1 1 0 0\n", "z missing"),
    ("ITEM: TIMESTEP\n", "expected NUMBER OF ATOMS line"),
])
def test_malformed_dumps_raise_the_references_errors(text, msg):
    with pytest.raises(lammps.DumpFormatError, match=msg):
        lammps.read_dump_text(text)


def test_timestep_line_is_trimmed_and_other_headers_are_not():
    ok = "   " + _dump(["1 1 1 2 3"])
    assert lammps.read_dump_text(ok)[0].tolist() == [1, 2, 3]
    shifted = _dump(["1 1 1 2 3"]).replace("ITEM: NUMBER OF ATOMS", " ITEM: NUMBER OF ATOMS")
    with pytest.raises(lammps.DumpFormatError, match="NUMBER OF ATOMS"):
        lammps.read_dump_text(shifted)
    assert lammps.read_dump_text("no timestep here\n") == []


def test_writer_layout_and_values(tmp_path):
    p = str(tmp_path / "w.dump")
    lammps.write_dump(p, 4, 2)
    lines = open(p).read().splitlines()
    assert lines[:9] == ["ITEM: TIMESTEP", "0", "ITEM: NUMBER OF ATOMS", "4", "ITEM: BOX BOUNDS xx yy zz",
                         "0 10", "0 10", "0 10", "ITEM: ATOMS id type x y z"]
    assert lines[9] == "1 1 1.000000 0.000000 1.000000"
    assert len(lines) == 2 * (9 + 4) and lines[13] == "ITEM: TIMESTEP" and lines[14] == "1"
    for row in lines[9:13] + lines[22:26]:
        assert all(len(tok.split(".")[1]) == 6 for tok in row.split()[2:])
    snaps = lammps.read_dump(p)
    ph = np.float32(0.1) + np.arange(4, dtype=np.float32) * np.float32(0.001)
    assert np.allclose(snaps[1][0::3], np.cos(ph), atol=1e-6)
    assert np.allclose(snaps[1][1::3], np.sin(ph), atol=1e-6)
    assert np.allclose(snaps[1][2::3], np.cos(ph * np.float32(0.5)), atol=1e-6)
    with pytest.raises(FileNotFoundError):
        lammps.read_dump(str(tmp_path / "missing.dump"))


def test_baselines_app(tmp_path, monkeypatch):
    monkeypatch.chdir(tmp_path)
    monkeypatch.setenv("ZFP_CMD", "cp {in} {out}")
    monkeypatch.setenv("SZ_CMD", "true {in} {out} {eps}")
    rows = baselines.main(["--particles", "300", "--steps", "6"])
    data = os.path.join("baseline_results", "data", "large.dump")
    orig = os.path.getsize(data)
    by = {(r["tool"], r["epsilon"]): r for r in rows}
    assert [r["tool"] for r in rows[:5]] == ["gzip -1 (fast)", "gzip -6 (default)", "gzip -9 (best)", "bzip2", "xz"]
    # the .nz rows are exactly the container the library writes for the parsed dump
    snaps = lammps.read_dump(data)
    x = np.concatenate(snaps)
    for codec, label, eps in baselines.NZ_RUNS:
        blob, _ = nzcp.compress(x, snaps[0].size, len(snaps), codec, eps)
        r = by[(f"Mini-Nangila ({label})", f"{eps:g}")]
        assert r["status"] == "OK" and r["compressed_bytes"] == len(blob) and r["codec"] == label
        assert float(r["ratio"]) == pytest.approx(orig / len(blob), abs=0.006)
    assert by[("ZFP", "0.001")]["ratio"] == "1.00" and by[("SZ", "0.001")]["status"] == "SKIPPED"
    with open(os.path.join("baseline_results", "baseline_comparison.csv"), newline="") as fh:
        rd = csv.DictReader(fh)
        assert rd.fieldnames[:8] == ["tool", "epsilon", "codec", "compressed_bytes", "ratio", "comp_time_s",
                                     "throughput_MBps", "status"]
        assert len(list(rd)) == len(rows) == 5 + len(baselines.NZ_RUNS) + 2
    summary = analysis.summarize_baselines(os.path.join("baseline_results", "baseline_comparison.csv"))
    assert set(summary) == {"general", "0.001", "0.01"}
    assert len(summary["0.001"]["tools"]) == 5  # four codecs and ZFP; the skipped SZ row is left out
    txt = open(os.path.join("baseline_results", "baseline_comparison.txt")).read()
    assert "Original size:" in txt and "Mini-Nangila (BlockSparse+RLE) (eps=0.001):" in txt and "SZ: SKIPPED" in txt


def test_reader_on_random_text_raises_only_format_errors():
    from hypothesis import given, settings
    from hypothesis import strategies as st

    base = _dump(["1 1 0.5 1.5 2.5", "2 1 -1 -2 -3"])
    alphabet = st.sampled_from(list("ITEM: TIMESTEPNUMBEROFATOMSBXyzxyz0123456789.e+-\n \t"))

    @settings(max_examples=300, deadline=None)
    @given(st.integers(0, len(base)), st.lists(alphabet, max_size=120))
    def run(cut, extra):
        text = base[:cut] + "".join(extra)
        try:
            snaps = lammps.read_dump_text(text)
        except lammps.DumpFormatError:
            return
        for s in snaps:
            assert s.dtype == np.float32 and s.size % 3 == 0

    run()
