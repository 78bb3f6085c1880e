"""bench.py contract on one GPU (tiny step counts)."""
import json
import sys

import pytest

from conftest import run

pytestmark = pytest.mark.gpu


def test_bench_json_line(built):
    r = run([sys.executable, "bench.py", "--steps", "3", "--warmup", "3"], timeout=900)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    line = [l for l in r.stdout.splitlines() if l.startswith("{")][-1]
    rec = json.loads(line)
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
              "higher_is_better", "scaling", "dtype", "data", "config", "clocks", "e2e",
              "gpu_launches"):
        assert k in rec, k
    assert rec["n_gpus"] == 1 and rec["value"] > 0 and rec["gpu_launches"] > 0
    assert rec["e2e"]["value"] > 0
