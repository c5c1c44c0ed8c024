"""bench.py's contract on CPU: the reference arm's JSON line, the committed
ncu summaries it reads traffic from, and its argument checks."""
import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))


def _run(*args, timeout=300):
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], cwd=ROOT, capture_output=True,
                          text=True, timeout=timeout)


def test_reference_arm_json_line():
    r = _run("--impl", "reference", "--workload", "vit_s", "--steps", "1", "--warmup", "3")
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference"
    assert line["unit"] == "TOPS" and line["value"] > 0 and line["higher_is_better"] is True
    assert line["n_gpus"] == 1 and line["steps"] == 1 and line["warmup"] == 3
    assert line["config"]["workload"] == "vit_s"
    cb = line["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == line["value"] and cb["sample"]
    e2e = line["e2e"]
    assert e2e["value"] == line["value"] and e2e["unit"] == "TOPS"
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


@pytest.mark.parametrize("workload", ["vit_b", "swin_s1", "vit_l"])
def test_profiles_give_traffic(workload):
    import bench
    t = bench.profile_traffic("qfa_fwd", workload)
    assert t is not None and t > 0


def test_warmup_below_three_is_refused():
    r = _run("--warmup", "2", timeout=120)
    assert r.returncode != 0
    assert "--warmup must be >= 3" in r.stderr
