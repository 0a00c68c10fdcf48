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
    """Each timed step solves a different row slice; the set-up is timed once; the metric is set-up + per-row time
    x 4096; ms_per_step is the wall time of one step; the config equals the GPU arm's."""
    calls = []

    class FakeOracle:
        cores, t_setup, what = 8, 3.0, "stub"

        def __init__(self, wl, H=None):
            assert wl == workload

        def solve_rows(self, r0, r1):
            calls.append((r0, r1))
            return 0.5 * (r1 - r0), None

    monkeypatch.setattr(bench, "CpuOracle", FakeOracle)
    monkeypatch.delenv("RANK", raising=False)
    monkeypatch.delenv("WORLD_SIZE", raising=False)
    args = types.SimpleNamespace(workload=workload, warmup=2, steps=3, cpu_sample_rows=4, ref_rows=32, block_rows=0,
                                 polish_mode="block_cd")
    line = bench.run_reference(args)
    json.dumps(line)
    assert line["impl"] == "reference" and line["higher_is_better"] is False
    assert line["value"] == pytest.approx(3.0 + 0.5 * 4096)
    assert line["ms_per_step"] == pytest.approx(0.5 * 32 * 1e3)
    assert line["cpu_baseline"]["kind"] == "port" and line["e2e"]["h2d_bytes_per_step"] == 0
    timed = calls[2:]
    assert [r1 - r0 for r0, r1 in calls[:2]] == [1, 1]  # warm-up steps: one row each
    assert timed == [(0, 32), (32, 64), (64, 96)]  # different slices
    assert line["measured"]["rows"] == 96
    assert line["config"] == bench.bench_config(args, 1)
    assert line["config"]["block_rows"] == (128 if workload == "e8p12" else "reference CUDA size (3640 + 456)")


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
