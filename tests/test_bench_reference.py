"""bench.py's reference arm (`--impl reference`) runs the CPU port of the
path and needs no GPU: it must print one JSON line with the molten arm's
metric, unit and direction, a `cpu_baseline` and an `e2e` object, for the
one-GPU default workload (cfg1) and for the prefill workload (cfg3); under
torchrun only rank 0 prints."""
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def run(args, env=None):
    e = dict(os.environ)
    e.update(env or {})
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", *args],
                       capture_output=True, text=True, timeout=240, env=e, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    return [l for l in r.stdout.splitlines() if l.strip().startswith("{")]


@pytest.mark.parametrize("workload,metric_part,unit", [("cfg1", "GB/s", "GB/s"),
                                                        ("cfg3", "tokens/s", "tokens/s")])
def test_reference_arm_prints_one_line(workload, metric_part, unit):
    lines = run(["--workload", workload, "--steps", "2", "--warmup", "1", "--cpu-seconds", "0.5"])
    assert len(lines) == 1, lines
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unit"] == unit and metric_part in d["metric"]
    assert d["higher_is_better"] is True and d["value"] > 0
    assert d["cpu_baseline"]["cores"] >= 1 and d["cpu_baseline"]["kind"] == "port"
    assert d["e2e"]["unit"] == unit and d["e2e"]["h2d_bytes_per_step"] == 0


def test_reference_arm_other_ranks_print_nothing():
    lines = run(["--workload", "cfg1", "--steps", "2", "--warmup", "1", "--cpu-seconds", "0.5"],
                env={"RANK": "1", "WORLD_SIZE": "2"})
    assert lines == []
