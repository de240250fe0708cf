"""CPU checks of bench.py's output contract where it needs no GPU: the reference arm (the reference's
own compiled C for configs[0], timed on the host cores) prints exactly one JSON line with the keys the
driver reads, and under torchrun only rank 0 prints."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
KEYS = ("metric", "value", "unit", "n_gpus", "steps", "warmup", "higher_is_better", "scaling", "vs_baseline",
        "dtype", "data", "config", "impl", "cpu_baseline", "e2e")


def _bench(args, env=None):
    e = dict(os.environ)
    e.update(env or {})
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py")] + args, capture_output=True, text=True,
                          timeout=600, env=e, cwd=ROOT)


def test_reference_arm_prints_one_contract_line():
    p = _bench(["--impl", "reference", "--workload", "c1", "--steps", "1", "--warmup", "0"])
    assert p.returncode == 0, p.stderr[-2000:]
    lines = [ln for ln in p.stdout.splitlines() if ln.strip().startswith("{")]
    assert len(lines) == 1, p.stdout[-2000:]
    d = json.loads(lines[0])
    assert all(k in d for k in KEYS), [k for k in KEYS if k not in d]
    assert d["impl"] == "reference" and d["value"] > 0 and d["higher_is_better"] is True
    assert d["unit"] == "samples/s" and d["steps"] == 1 and d["warmup"] == 0
    # the reference arm's end-to-end figure is its own value, with no device copies
    assert d["e2e"]["value"] == d["value"] and d["e2e"]["unit"] == d["unit"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    base = d["cpu_baseline"]
    assert base["kind"] == "reference" and base["cores"] >= 1 and base["value"] == d["value"] and base["sample"]


def test_reference_arm_other_ranks_exit_quietly():
    p = _bench(["--impl", "reference", "--workload", "c1", "--steps", "1", "--warmup", "0"],
               env={"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert p.returncode == 0, p.stderr[-2000:]
    assert not p.stdout.strip()
