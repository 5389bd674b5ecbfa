"""CPU: the evaluator loops (linalg_kernels_b200.evaluate) with a host kernel and the
oracle's gates standing in for the GPU kernel and the device checker: case parsing and
seeds, the per-window input count, the seed step between inputs, the statistics, and the
recheck that catches a kernel which writes its input (references/popcorn-eval/eval.py)."""

import math

import pytest
import torch

from linalg_kernels_b200 import evaluate, inputs
from oracle import oracle


def _host_kernel(a):
    return torch.linalg.cholesky_ex(a).L  # a host stand-in for the GPU kernel (test only)


def _host_check(data, out):
    res = oracle.check_factor(data.numpy(), out.numpy())
    return res["ok"], "" if res["ok"] else str(res)


def test_parse_and_seed_pairing():
    cases = evaluate.parse_cases("batch: 4; n: 32; cond: 2; seed: 7\n\nbatch: 1; n: 8; "
                                 "cond: 5; seed: 3; case: diagonal")
    assert [c.args for c in cases] == [
        {"batch": 4, "n": 32, "cond": 2, "seed": 7},
        {"batch": 1, "n": 8, "cond": 5, "seed": 3, "case": "diagonal"}]
    assert evaluate.pair_seed(7, 100) == 7 + 107 * 108 // 2
    seeded = evaluate.parse_cases("batch: 4; n: 32; seed: 7", seed=100)
    assert seeded[0].args["seed"] == evaluate.pair_seed(7, 100)
    with pytest.raises(ValueError):
        evaluate.parse_cases("batch = 4")


def test_builtin_case_lists():
    grid = evaluate.grid_cases()
    assert len(grid) == 15 and len(evaluate.grid_cases(big=False)) == 14
    assert [(c.args["batch"], c.args["n"], c.args["seed"]) for c in grid] == \
        [(c.batch, c.n, c.seed) for c in inputs.GRID.values()]
    tests = evaluate.reference_test_cases()
    assert len(tests) == 17
    assert [c.args.get("case") for c in tests] == [s.case for s in inputs.TEST_SHAPES]


def test_calls_per_window():
    assert evaluate.calls_per_window({"batch": 4096, "n": 32}) == 16  # 16 MiB inputs
    assert evaluate.calls_per_window({"batch": 1, "n": 16384}) == 1
    assert evaluate.calls_per_window({"batch": 2, "n": 8}) == 50


def test_stats():
    s = evaluate.stats([1.0, 2.0, 3.0, 6.0])
    assert s.runs == 4 and s.mean == 3.0 and s.best == 1.0 and s.worst == 6.0
    assert s.std == pytest.approx(math.sqrt(14.0 / 3.0))
    assert s.err == pytest.approx(s.std / 2.0)
    assert evaluate.stats([5.0]).std == 0.0


def test_benchmark_steps_the_seed_and_times(monkeypatch):
    seen = []
    real = evaluate.generate

    def recording(args, device="cuda"):
        seen.append(args["seed"])
        return real(args, device)

    monkeypatch.setattr(evaluate, "generate", recording)
    case = evaluate.parse_cases("batch: 2; n: 24; cond: 2; seed: 1000")[0]
    r = evaluate.run_benchmark(case, True, 5, 1e12, kernel=_host_kernel, check=_host_check,
                               device="cpu")
    assert isinstance(r, evaluate.Stats), r
    assert 3 <= r.runs <= 5 and r.mean > 0
    assert seen == [1000 + 42 * (i + 1) for i in range(50)]
    assert case.args["seed"] == 1000  # the case itself is left as it was


def test_recheck_catches_a_kernel_that_writes_its_input():
    def clobbering(a):
        out = torch.linalg.cholesky_ex(a).L
        a.zero_()
        return out

    case = evaluate.parse_cases("batch: 2; n: 16; cond: 2; seed: 5")[0]
    r = evaluate.run_benchmark(case, True, 5, 1e12, kernel=clobbering, check=_host_check,
                               device="cpu")
    assert isinstance(r, str)
    # without the recheck the timing loop does not look at the outputs
    r = evaluate.run_benchmark(case, False, 3, 1e12, kernel=clobbering, check=_host_check,
                               device="cpu")
    assert isinstance(r, evaluate.Stats)


def test_modes_log_and_exit_codes():
    lines = []
    log = lambda k, v: lines.append(f"{k}: {v}")  # noqa: E731
    cases = evaluate.parse_cases("batch: 3; n: 16; cond: 2; seed: 1\n"
                                 "batch: 2; n: 40; cond: 2; seed: 2; case: tridiagonal")
    kw = dict(kernel=_host_kernel, check=_host_check, device="cpu")
    assert evaluate.run_mode("test", cases, log, **kw) == 0
    assert lines[0] == "test-count: 2" and lines[-1] == "check: pass"
    assert "test.1.status: pass" in lines
    lines.clear()
    assert evaluate.run_mode("benchmark", cases, log, **kw) == 0
    assert "benchmark-count: 2" in lines and any(x.startswith("benchmark.1.mean: ")
                                                 for x in lines)
    lines.clear()
    bad = dict(kw, kernel=lambda a: torch.zeros_like(a))
    assert evaluate.run_mode("leaderboard", cases, log, **bad) == evaluate.FAIL_EXIT
    assert lines[-1] == "check: fail" and "benchmark.0.status: fail" in lines
