"""bench.py's reference arm (the oracle port on the host cores) against the JSON line the
benchmark contract asks for: run as a subprocess the way the harness runs it, one JSON
line on stdout, and no work on ranks other than 0.  CPU only."""

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(env_extra, *args):
    env = dict(os.environ, **env_extra)
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                           *args], capture_output=True, text=True, cwd=ROOT, env=env, timeout=300)


def test_reference_arm_prints_one_json_line():
    r = _run({}, "--steps", "1", "--warmup", "0")
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.strip()]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    for k in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
              "higher_is_better", "config", "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["impl"] == "reference" and d["value"] > 0 and d["higher_is_better"] is True
    assert d["unit"] == d["e2e"]["unit"] == d["cpu_baseline"]["unit"] == "words/s"
    assert d["e2e"]["value"] == d["value"] == d["cpu_baseline"]["value"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["cpu_baseline"]["kind"] in ("port", "reference") and d["cpu_baseline"]["cores"] >= 1
    assert "workload" in d["config"]


def test_reference_arm_other_ranks_do_nothing():
    r = _run({"RANK": "1", "WORLD_SIZE": "2"}, "--steps", "1", "--warmup", "0")
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == ""


def test_hbm_peak_falls_back_when_the_measured_peaks_are_absent(tmp_path, monkeypatch):
    """The roofline's HBM peak: MEASURED_PEAKS.json's hbm_gbs when the file is there, the
    recipe's 6650 GB/s (said so in peak_source) when it is absent or unreadable."""
    sys.path.insert(0, ROOT)
    import bench
    monkeypatch.setattr(bench, "PEAKS", str(tmp_path / "missing.json"))
    peak, src = bench.hbm_peak_gbs()
    assert peak == 6650.0 and "fallback" in src
    f = tmp_path / "peaks.json"
    f.write_text(json.dumps({"hbm_gbs": 6545.6}))
    monkeypatch.setattr(bench, "PEAKS", str(f))
    peak, src = bench.hbm_peak_gbs()
    assert peak == 6545.6 and "of measured" in src
    f.write_text("{not json")
    assert bench.hbm_peak_gbs()[0] == 6650.0
