"""GPU: custom_kernel through the evaluator's loops (linalg_kernels_b200.evaluate) with the
device checker: the reference's 17 test shapes in 'test' mode, and the benchmark loop
(distinct inputs per window, L2 flush, recheck of every repeat) on small grid entries."""

import pytest

from linalg_kernels_b200 import evaluate

pytestmark = pytest.mark.gpu


def test_reference_test_shapes_pass_the_test_mode():
    lines = []
    rc = evaluate.run_mode("test", evaluate.reference_test_cases(),
                           lambda k, v: lines.append(f"{k}: {v}"))
    assert rc == 0, [x for x in lines if "error" in x]
    assert lines[0] == "test-count: 17" and lines[-1] == "check: pass"


@pytest.mark.parametrize("index", [0, 1, 2])  # b4096n32, b1024n64, b256n128
def test_benchmark_loop_on_small_grid_entries(index):
    case = evaluate.grid_cases()[index]
    r = evaluate.run_benchmark(case, True, 5, 1e9)
    assert isinstance(r, evaluate.Stats), r
    assert 3 <= r.runs <= 5
    # ns per call; the first window also pays for its fresh outputs' allocations (in the
    # reference's evaluator too), so only the best window is bounded
    assert 0 < r.best <= r.mean <= r.worst and r.best < 1e6
