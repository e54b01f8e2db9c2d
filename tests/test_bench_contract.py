"""The reference arm of bench.py on CPU: one JSON line with the keys the
driver reads, and silence on ranks other than 0 under a multi-rank launch."""
import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def _run(extra_env=None, *args):
    env = dict(os.environ)
    env.pop("RANK", None)
    env.pop("WORLD_SIZE", None)
    env.pop("LOCAL_RANK", None)
    env.update(extra_env or {})
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference",
                           "--steps", "1", "--warmup", "3", "--tokens", "256", *args],
                          capture_output=True, text=True, timeout=600, env=env, cwd=ROOT)


def test_reference_arm_json_line():
    r = _run()
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"] == "moe_layer_tokens_per_s" and d["unit"] == "tokens/s"
    assert d["value"] > 0 and d["higher_is_better"] is True
    assert d["steps"] == 1 and d["warmup"] == 3
    assert d["config"]["workload"].startswith("moe_layer_")
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["cores"] >= 1 and cb["kind"] in ("port", "reference")
    assert cb["sample"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_reference_arm_other_ranks_are_silent():
    r = _run({"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"}, "--gpus", "2")
    assert r.returncode == 0, r.stderr[-2000:]
    assert not [l for l in r.stdout.splitlines() if l.startswith("{")]


def test_reference_arm_config_is_ours(monkeypatch):
    """Both arms print the same `config` dict for the same arguments (it is a
    function of the arguments alone), so the driver can match the lines."""
    r = _run(None, "--gpus", "2")
    assert r.returncode == 0, r.stderr[-2000:]
    d = json.loads([l for l in r.stdout.splitlines() if l.startswith("{")][0])
    sys.path.insert(0, str(ROOT))
    import bench
    monkeypatch.setattr(sys, "argv", ["bench.py", "--impl", "reference", "--steps", "1",
                                      "--warmup", "3", "--tokens", "256", "--gpus", "2"])
    args = bench.parse()
    assert d["config"] == bench.bench_config(args, 2)
    assert "owner placement" in d["config"]["parallelism"]
