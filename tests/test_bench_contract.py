"""bench.py's output contract, checked on its CPU-only reference arm (no GPU needed): one
JSON line with the metric, value, unit, timing and e2e fields the harness reads."""
import json
import os
import subprocess
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_one_contract_line():
    out = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference",
                          "--workload", "config1", "--steps", "2", "--warmup", "3"],
                         capture_output=True, text=True, timeout=600, cwd=REPO)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config", "e2e",
                "cpu_baseline"):
        assert key in d, key
    assert d["impl"] == "reference" and d["value"] > 0 and d["warmup"] >= 3 and d["steps"] == 2
    assert d["e2e"]["value"] == d["value"] and d["e2e"]["h2d_bytes_per_step"] == 0
    assert d["cpu_baseline"]["kind"] in ("reference", "port") and d["cpu_baseline"]["cores"] >= 1
    assert "workload" in d["config"]


def test_clock_sampler_covers_a_short_region(tmp_path, monkeypatch):
    """A timed region shorter than the sampling interval still gets a clock sample, and a
    throttle reason seen during it is reported (nvidia-smi replaced by a script)."""
    import importlib.util
    import time
    fake = tmp_path / "nvidia-smi"
    fake.write_text("#!/bin/bash\nwhile true; do echo \"0, 1500, 1965, 700.0, 0x4, Not Active, "
                    "Not Active, Not Active, Active\"; sleep 0.05; done\n")
    fake.chmod(0o755)
    monkeypatch.setenv("PATH", f"{tmp_path}:{os.environ['PATH']}")
    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(REPO, "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    c = bench.ClockSampler(0)
    c.start()
    c.begin()
    time.sleep(0.01)
    c.end()
    clk = c.stop()
    assert clk["samples"] >= 1 and clk["sm_mhz"] == 1500.0 and clk["sm_max_mhz"] == 1965.0
    assert clk["reasons"] == ["sw_power_cap"]
