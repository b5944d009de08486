"""bench.py's host-side pieces (CPU): the reference arm's piece schedule covers one whole
sampler step for any step count, and the parallelism labels name the partitioning."""
import importlib.util
from pathlib import Path

import pytest


@pytest.fixture(scope="module")
def bench():
    path = Path(__file__).resolve().parent.parent / "bench.py"
    spec = importlib.util.spec_from_file_location("bench_under_test", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.mark.parametrize("steps", [1, 2, 7, 20, 29, 30, 31, 64])
def test_reference_schedule_covers_one_step(bench, steps):
    sched = bench.reference_schedule(steps, 30)
    assert len(sched) == steps and all(sched)
    flat = [j for plan in sched for j in plan]
    assert set(flat) == set(range(30))
    if steps <= 30:
        assert sorted(flat) == list(range(30))  # every piece exactly once, in order
        assert flat == sorted(flat)


def test_parallelism_labels(bench):
    assert "replicas x8" in bench.parallelism_label(False, 1, 8)
    lab = bench.parallelism_label(True, 1, 1, "peer", 4)
    assert "CFG pair split" in lab and "token rows sharded over 4 GPUs" in lab
    assert "heads and MLP columns sharded over 2" in bench.parallelism_label(True, 2, 1)
