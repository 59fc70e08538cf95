"""Host-side logic of the benchmark and the workload generator (CPU only)."""
import json
import os
import subprocess
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


def test_topp_rows_drawn_independently(pkg):
    """Any range of global rows equals the same rows of a larger draw, so each
    rank of a multi-GPU batch draws its own shard without the rows before it."""
    whole = pkg.workloads.topp(rows=6, vocab=512)
    part = pkg.workloads.topp(rows=3, vocab=512, first=2)
    assert np.array_equal(part["logits"], whole["logits"][2:5])
    assert np.array_equal(part["topp_rows"], whole["topp_rows"][2:5])


def test_profiled_traffic_needs_matching_digest(tmp_path, monkeypatch):
    """The DRAM traffic of a profile is reported only while its source digest
    matches the current kernel sources; a capture of other sources is ignored."""
    digest = bench.kernel_source_digest(bench.STREAM_SOURCES)
    assert digest == bench.kernel_source_digest(bench.STREAM_SOURCES)
    prof = tmp_path / "profiles"
    prof.mkdir()
    (prof / "good.md").write_text(f"x\nsource_digest: {digest}\ntraffic_bytes_per_launch: 1234\n")
    (prof / "stale.md").write_text("source_digest: 0000000000000000\ntraffic_bytes_per_launch: 99\n")
    (prof / "none.md").write_text(f"source_digest: {digest}\n")
    monkeypatch.setattr(bench, "ROOT", str(tmp_path))
    monkeypatch.setattr(bench, "kernel_source_digest", lambda files: digest)
    assert bench.profiled_traffic("good.md", bench.STREAM_SOURCES) == 1234
    assert bench.profiled_traffic("stale.md", bench.STREAM_SOURCES) is None
    assert bench.profiled_traffic("none.md", bench.STREAM_SOURCES) is None
    assert bench.profiled_traffic("missing.md", bench.STREAM_SOURCES) is None


def test_committed_profiles_match_current_sources():
    """The committed streaming-kernel summary was captured on these sources,
    so the benchmark line carries its measured traffic."""
    assert bench.profiled_traffic("row_stream_kernel_topp_4096x32000.md", bench.STREAM_SOURCES)


def test_host_cpu_reports_count():
    info = bench.host_cpu()
    assert info["nproc"] == os.cpu_count() and info["nproc"] >= 1


def test_reference_arm_prints_one_line():
    """--impl reference runs the reference's own sampler on the host cores and
    prints the contract's JSON line (a small sample of rows here)."""
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "0", "--ref-rows", "16"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["value"] > 0 and line["unit"] == "tokens/s"
    assert line["cpu_baseline"]["kind"] in ("reference", "port") and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
