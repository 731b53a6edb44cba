"""bench.py's reference arm on the CPU: `--impl reference` times the
reference's own CPU ForwardToken (src/forward.cc:776-807, built into
oracle/_ref) and prints one JSON line with the keys every bench line carries,
plus its cpu_baseline and an e2e entry without host<->device copies. Run here
on the tiny configuration (dim 288, 6 layers, Q8_0) at a short context, so the
line's shape is checked without a GPU."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_line(ref):
    out = subprocess.run(
        [sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--workload",
         "tiny-q8_0", "--ctx", "32", "--steps", "2", "--warmup", "1"],
        cwd=ROOT, capture_output=True, text=True, timeout=300, check=True)
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, out.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and "unavailable" not in d
    assert d["metric"] == "decode tok/s" and d["unit"] == "tok/s"
    assert d["value"] > 0 and d["ms_per_step"] > 0
    assert d["steps"] == 2 and d["warmup"] == 1 and d["n_gpus"] == 1
    assert d["higher_is_better"] is True and d["scaling"] in ("weak", "strong")
    assert d["config"]["workload"] == "tiny-q8_0" and d["config"]["ctx"] == 32
    cb = d["cpu_baseline"]
    assert cb["kind"] == "reference" and cb["cores"] >= 1 and cb["value"] == d["value"]
    assert cb["unit"] == "tok/s" and cb["sample"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == "tok/s"
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    assert len(d["greedy_ids"]) == 3
