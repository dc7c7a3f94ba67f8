"""bench.py's driver-facing contract on the CPU: the reference arm's JSON line,
the roofline traffic read from the committed ncu summary, and the argument
checks that run before any GPU work."""
import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def test_reference_arm_prints_one_contract_line():
    run = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "3",
                          "--warmup", "3"], cwd=ROOT, capture_output=True, text=True,
                         timeout=600)
    assert run.returncode == 0, run.stderr[-2000:]
    lines = [l for l in run.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    line = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
                "impl", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference" and line["steps"] == 3 and line["warmup"] == 3
    assert line["value"] > 0 and line["higher_is_better"] is True
    assert line["cpu_baseline"]["value"] == line["value"]
    assert line["cpu_baseline"]["kind"] in ("port", "reference")
    assert line["cpu_baseline"]["cores"] >= 1 and line["cpu_baseline"]["sample"]
    assert line["e2e"]["value"] == line["value"] and line["e2e"]["unit"] == line["unit"]
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    assert line["config"]["workload"].startswith("config 1")


def test_roofline_traffic_comes_from_the_committed_profile():
    sys.path.insert(0, str(ROOT))
    import bench
    text = (ROOT / "profiles" / "attn_fwd_bf16_config1.md").read_text()
    want = next(float(l.split(":", 1)[1].split()[0]) for l in text.splitlines()
                if l.startswith("dram_bytes_per_launch:"))
    assert bench.profiled_traffic("attn_fwd_bf16_config1") == want
    assert bench.profiled_traffic("no_such_kernel") is None


def test_ring_refuses_other_precisions_before_gpu_work():
    for extra in (["--fp8"], ["--sparse"], ["--qkv-fp8"]):
        run = subprocess.run([sys.executable, "bench.py", "--ring", "2", *extra], cwd=ROOT,
                             capture_output=True, text=True, timeout=300)
        assert run.returncode == 2 and "ring path" in run.stderr, extra
