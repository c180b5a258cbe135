"""bench.py's output contract, checked on CPU through its reference arm (the
oracle timed on the host cores): one JSON line with the driver's keys, the
reference-arm extras, and a zero-copy e2e block.  No GPU needed."""
import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]

KEYS = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
        "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config"}


def run_reference(*args):
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", *args],
                         cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, out.stdout
    return json.loads(lines[0])


def test_reference_arm_line():
    d = run_reference("--workload", "ep", "--steps", "1", "--warmup", "1", "--layers", "48")
    assert KEYS <= set(d), KEYS - set(d)
    assert d["impl"] == "reference"
    assert d["scaling"] == "strong"  # the EP stack's own arm: fixed global batch
    assert d["warmup"] >= 3  # the contract's minimum is enforced
    assert d["value"] > 0 and d["unit"] == "tokens/s" and d["higher_is_better"] is True
    assert isinstance(d["config"], dict) and "workload" in d["config"]
    cb = d["cpu_baseline"]
    assert {"value", "unit", "cores", "kind", "sample"} <= set(cb)
    assert cb["kind"] in ("port", "reference") and cb["value"] == d["value"] and cb["cores"] >= 1
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_reference_arm_other_ranks_print_nothing():
    """Under torchrun only rank 0 runs the CPU reference; the others exit 0."""
    import os

    env = dict(os.environ, RANK="1", WORLD_SIZE="2")
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference",
                          "--workload", "ep", "--steps", "1"], cwd=ROOT, env=env,
                         capture_output=True, text=True, timeout=300)
    assert out.returncode == 0 and not [l for l in out.stdout.splitlines() if l.startswith("{")]
