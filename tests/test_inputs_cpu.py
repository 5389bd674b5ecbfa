"""CPU: the benchmark grid and test-shape tables, and their generators against the oracle.

The grid is the reference's 15 benchmark entries (AGENTS.md:66-81) and the test shapes its
17 correctness entries (AGENTS.md:83-100); bench.py carries the reference's published time
for every grid entry."""

import numpy as np
import pytest

import bench
from linalg_kernels_b200 import inputs
from oracle import oracle


def test_grid_holds_the_configs_and_the_published_times():
    assert len(inputs.GRID) == 15
    assert set(inputs.CONFIGS) <= set(inputs.GRID)
    for name, cfg in inputs.GRID.items():
        assert name == f"b{cfg.batch}n{cfg.n}"
        assert name in bench.REFERENCE_PUBLISHED_S
    # the low-batch entries from n = 32 to 1024 hold 2^22 elements each (AGENTS.md:58-61)
    for name in ("b4096n32", "b1024n64", "b256n128", "b64n256", "b16n512", "b4n1024"):
        cfg = inputs.GRID[name]
        assert cfg.batch * cfg.n * cfg.n == 1 << 22


def test_grid_summary_is_the_geometric_mean():
    # the compact shape rows: [ms per call, published ms, ratio, roofline fraction]
    shapes = {"cols": ["ms", "ref_ms", "vs_ref", "frac"], "frac": "note",
              "b4096n32": [0.01, 0.0157, 1.57, 0.5], "b1n16384": [10.0, 15.1, 1.51, 0.2]}
    g = bench._grid_summary("b1024n64", 0.02, shapes)
    assert g["entries"] == 3
    assert g["geomean_ms"] == pytest.approx((0.01 * 10.0 * 0.02) ** (1 / 3), rel=1e-3)
    ref = (15.7e-3 * 15.1 * 24.1e-3) ** (1 / 3)
    assert g["reference_geomean_ms"] == pytest.approx(ref, rel=1e-3)
    assert g["vs_reference_published"] == pytest.approx(ref / g["geomean_ms"], rel=1e-3)


def test_test_shapes_table():
    assert len(inputs.TEST_SHAPES) == 17
    assert len({(s.batch, s.n, s.seed) for s in inputs.TEST_SHAPES}) == 17
    for s in inputs.TEST_SHAPES:
        assert s.case is None or s.case in inputs.CASES


@pytest.mark.parametrize("spec", [s for s in inputs.TEST_SHAPES if s.n <= 512],
                         ids=lambda s: f"b{s.batch}n{s.n}-{s.case or 'family'}-{s.seed}")
def test_test_shape_inputs_are_spd(spec):
    """Each generated input is symmetric up to FP32 roundoff (the factor reads only the lower
    triangle) and SPD: the oracle factors it with info 0 and a residual within the
    north-star bound."""
    a = inputs.spec_input(spec)
    assert a.shape == (spec.batch, spec.n, spec.n) and a.is_contiguous()
    a = a.numpy()
    asym = np.abs(a - np.swapaxes(a, 1, 2)).max()
    assert asym <= 4 * np.finfo(np.float32).eps * np.abs(a).max(), asym
    l, info = oracle.potrf(a)
    assert (info == 0).all()
    res = oracle.check_factor(a, l)
    assert res["ok"], res


def test_generate_input_follows_the_grid_families():
    """generate_input(batch, n, seed) gives the grid entry's own input at its shape."""
    for name in ("b4096n32", "b256n128", "b16n512", "b2n2048"):
        cfg = inputs.GRID[name]
        b = min(cfg.batch, 2)
        want, _ = inputs.config_input(cfg, batch=b)
        got = inputs.generate_input(b, cfg.n, cfg.seed)
        assert np.array_equal(got.numpy(), want.numpy()), name
