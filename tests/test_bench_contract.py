"""bench.py's reference arm and launch checks, on the CPU.

The reference arm times the reference's CPU implementation of the sweep (the
compiled reference when it was built, else the oracle port) and must print one
JSON line with the same metric, unit and config keys as the GPU arm, plus
impl = "reference", a cpu_baseline block and an e2e block with no host<->device
bytes.  Under torchrun only rank 0 prints; the other ranks exit 0 silently."""
import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def _bench(args, env_extra=None):
    env = dict(os.environ)
    for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK"):
        env.pop(k, None)
    env.update(env_extra or {})
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], cwd=ROOT, env=env,
                          capture_output=True, text=True, timeout=600)


def test_reference_arm_prints_one_contract_line():
    r = _bench(["--impl", "reference", "--steps", "1", "--warmup", "1", "--ref-rows", "256"])
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["unit"] == "GB/s" and d["n_gpus"] == 1
    assert d["higher_is_better"] is True and d["value"] > 0
    assert "workload" in d["config"]
    sys.path.insert(0, str(ROOT))
    import bench
    assert d["config"] == bench.sweep_config(1)  # the GPU arm reports the same config at N=1
    cb = d["cpu_baseline"]
    assert cb["isa"]
    assert cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_reference_arm_other_ranks_exit_silently():
    r = _bench(["--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "1", "--ref-rows", "256"],
               {"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == ""


def test_gpu_count_must_match_the_launch():
    r = _bench(["--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "1"])
    assert r.returncode != 0
    assert "WORLD_SIZE" in (r.stderr + r.stdout)
