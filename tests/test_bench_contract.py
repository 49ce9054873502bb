"""The bench's reference arm runs on the host cores alone: one JSON line with the keys the driver
reads (the reference arm's line carries impl, cpu_baseline and a host-only e2e), and the process
loads no library of the product (only the oracle's: the reference's host C and the restatement)."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_one_contract_line():
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1", "--warmup", "1"], cwd=ROOT,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for k in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling", "vs_baseline", "dtype",
              "data", "config", "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["impl"] == "reference" and d["steps"] == 1 and d["warmup"] == 1 and d["n_gpus"] == 1
    assert d["value"] > 0 and d["ms_per_step"] > 0 and d["higher_is_better"] is True
    assert "workload" in d["config"]
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    e = d["e2e"]
    assert e["value"] == d["value"] and e["unit"] == d["unit"] and e["h2d_bytes_per_step"] == 0 and e["d2h_bytes_per_step"] == 0
    libs = d["libraries_from_repo"]
    assert libs and all(l.startswith("oracle" + os.sep) for l in libs), libs


def test_host_threads_split_per_rank(monkeypatch):
    sys.path.insert(0, ROOT)
    import bench
    monkeypatch.setenv("LOCAL_WORLD_SIZE", "8")
    n8 = bench.host_threads()
    monkeypatch.setenv("LOCAL_WORLD_SIZE", "1")
    n1 = bench.host_threads()
    assert n1 == (os.cpu_count() or 8) and n8 == max(1, n1 // 8)
