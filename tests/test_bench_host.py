"""Host-side pieces of bench.py that need no GPU: the workload table, the
algorithmic bytes of a checkpoint and the e2e step count."""
import importlib.util
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_module", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_workload_table(bench):
    for name, wk in bench.WORKLOADS.items():
        assert len(wk["layers"]) == len(wk["exit_fractions"]), name
        assert wk["of"] in ("batch", "active"), name
        assert wk.get("dtype", "bf16") in bench.DTYPE_NAMES, name
        assert wk.get("hidden", 4096) % 32 == 0, name
    # the reference's kernel-level case: 4096 fp32 rows of H = 768, one router, 30 % exits
    k = bench.WORKLOADS["kernel_fp32_4096x768"]
    assert (k["rows"], k["hidden"], k["dtype"], k["exit_fractions"]) == (4096, 768, "f32", [0.30])


def test_algorithmic_bytes(bench):
    # every row read and written once, 21 B per row, 12 B per survivor
    n, exits, h = 32768, 1638, 4096
    assert bench.algorithmic_bytes(n, exits, h, 2) == n * 2 * h * 2 + 21 * n + 12 * (n - exits)
    assert bench.algorithmic_bytes(4096, 4096, 768, 4) == 4096 * 2 * 768 * 4 + 21 * 4096


def test_e2e_step_count(bench):
    # the headline sweep copies ~1.6 GB per step: the minimum of 3 steps
    assert bench.e2e_step_count(None, 32768 * 4096 * 2 * 6) == 3
    # a 12.6 MB workload: enough steps for ~2 GB of copies
    assert bench.e2e_step_count(None, 4096 * 768 * 4) == 158
    assert bench.e2e_step_count(None, 1) == 200
    assert bench.e2e_step_count(5, 1) == 5
    assert bench.e2e_step_count(1, 10 ** 12) == 1
