"""bench.py's JSON contract on the CPU: the reference arm's line (with the CPU sample stubbed) and the argument
surface the driver uses."""
import json
import subprocess
import sys
import types
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def bench():
    sys.path.insert(0, str(ROOT))
    import bench as B
    return B


@pytest.mark.parametrize("workload", ["e8p12", "scalar"])
def test_reference_arm_line(bench, monkeypatch, workload):
    calls = []

    def fake_sample(wl, rows):
        calls.append((wl, rows))
        return {"value": 12.5, "unit": "s", "cores": 8, "kind": "port", "sample": f"{rows} rows"}

    monkeypatch.setattr(bench, "cpu_sample", fake_sample)
    monkeypatch.delenv("RANK", raising=False)
    args = types.SimpleNamespace(workload=workload, warmup=2, steps=3, cpu_sample_rows=4)
    line = bench.run_reference(args)
    json.dumps(line)
    assert line["impl"] == "reference" and line["value"] == 12.5 and line["higher_is_better"] is False
    assert line["cpu_baseline"]["kind"] == "port" and line["e2e"]["h2d_bytes_per_step"] == 0
    assert len(calls) == 5 and calls[-1] == (workload, 4)


def test_reference_arm_other_ranks_do_nothing(bench, monkeypatch):
    monkeypatch.setenv("RANK", "1")
    assert bench.run_reference(types.SimpleNamespace(workload="e8p12", warmup=1, steps=1, cpu_sample_rows=0)) is None


def test_reference_arm_model_workloads_report_unavailable(bench, monkeypatch):
    monkeypatch.delenv("RANK", raising=False)
    line = bench.run_reference(types.SimpleNamespace(workload="model", warmup=1, steps=1, cpu_sample_rows=0))
    assert line["impl"] == "reference" and "unavailable" in line


def test_bench_help_lists_contract_flags():
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--help"], capture_output=True, text=True,
                         timeout=120).stdout
    for flag in ("--gpus", "--steps", "--warmup", "--impl", "--workload", "--polish-mode"):
        assert flag in out
