"""CPU: the host side of the schedule choice, through the C ABI without a GPU.

chol_launch_count and chol_workspace_bytes are pure host logic; they follow the schedules
the blocked path picks: one small-kernel launch for n <= 64, one shared-memory-kernel launch
for n <= 128, one wide-kernel launch for a ragged 128 < n <= 256 (small batches); for one panel, the whole matrix
in one diagonal-block launch while batch * n^3 is small, else the left-looking chain (a zero
fill, then per block column a factor, a left-looking update and a solve; 128-wide block
columns when n % 128 == 0, 64-wide otherwise or with CHOL_OPT_CHAIN_WIDTH = 64); for several
512-wide
panels, per panel the diagonal block, the solve GEMM, the split and the trailing update.
Also the reference arm of bench.py (the reference's CPU path) prints its JSON line."""

import json
import subprocess
import sys
from pathlib import Path

import pytest

from linalg_kernels_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.parametrize("batch,n,launches", [
    (1, 32, 1), (4096, 32, 1), (1024, 64, 1),
    (4, 256, 2),            # one diagonal-block launch (+ copy)
    (640, 512, 10),         # 128-wide chain: 4 factors (with the zero fill) + 3 updates + 3 solves
    (60, 1024, 47),         # batch < 256: 64-wide chain: 1 + 16 + 15 + 15
    (256, 1024, 22),        # 128-wide chain: 8 + 7 + 7
    (400, 320, 14),         # n % 128 != 0: 64-wide chain: 1 + 5 + 4 + 4
    (3, 200, 1),            # ragged 128 < n <= 256, small batch: one wide-kernel launch
    (600, 200, 11),         # the same n at a large batch: the 64-wide chain, 1 + 4 + 3 + 3
    (1024, 130, 1),         # n < 144: the wide kernel at any batch
    (64, 192, 2),           # n % 64 == 0: the one-launch diagonal-block path (+ copy)
    (1, 2048, 16),          # 3 x (block, solve, split, trailing) + last block + copy,
                            # + 2 look-ahead splits (automatic for n <= 8192)
    (1, 2100, 35),          # 768-wide panels: 2 full ones (block, solve, split, trailing; one
                            # look-ahead split) + a 564-wide last panel as a 64-wide chain
                            # (9 factors, 8 updates, 8 solves) + copy
    (1, 16384, 86),         # 768-wide panels: 21 x 4 + a 256-wide last block + copy
    (2, 1030, 50),          # rows not 16-byte multiples: the 64-wide steps in each panel
])
def test_launch_counts_follow_the_schedule(batch, n, launches):
    assert int(_lib.load().chol_launch_count(batch, n)) == launches


def test_lookahead_option():
    lib = _lib.load()
    assert lib.chol_set_option(_lib.CHOL_OPT_LOOKAHEAD, 2) == _lib.CHOL_ERR_INVALID_ARG
    try:
        assert lib.chol_set_option(_lib.CHOL_OPT_LOOKAHEAD, 0) == _lib.CHOL_OK
        assert int(lib.chol_launch_count(1, 2048)) == 14
        assert lib.chol_set_option(_lib.CHOL_OPT_LOOKAHEAD, 1) == _lib.CHOL_OK
        assert int(lib.chol_launch_count(1, 16384)) > 86
    finally:
        lib.chol_set_option(_lib.CHOL_OPT_LOOKAHEAD, -1)
    assert int(lib.chol_launch_count(1, 16384)) == 86    # automatic: off above n = 8192


def test_chain_width_option():
    lib = _lib.load()
    assert lib.chol_set_option(_lib.CHOL_OPT_CHAIN_WIDTH, 96) == _lib.CHOL_ERR_INVALID_ARG
    assert lib.chol_set_option(_lib.CHOL_OPT_CHAIN_WIDTH, 64) == _lib.CHOL_OK
    try:
        assert int(lib.chol_launch_count(640, 512)) == 23   # 64-wide chain: 1 + 8 + 7 + 7
        assert int(lib.chol_launch_count(256, 1024)) == 47  # 1 + 16 + 15 + 15
    finally:
        lib.chol_set_option(_lib.CHOL_OPT_CHAIN_WIDTH, 128)
    assert int(lib.chol_launch_count(640, 512)) == 10


def test_mid_sizes_take_one_launch_and_no_workspace():
    """64 < n <= 128: one launch of the shared-memory kernel, no workspace; the same for the
    wide kernel's ragged 128 < n <= 256; with CHOL_OPT_MID_KERNEL = 0 the blocked schedule
    (and its workspace) comes back."""
    lib = _lib.load()
    for b, n in ((256, 128), (7, 65), (33, 100), (256, 130), (296, 255), (2048, 143)):
        assert int(lib.chol_launch_count(b, n)) == 1
        assert int(lib.chol_workspace_bytes(b, n)) == 0
    assert lib.chol_set_option(_lib.CHOL_OPT_MID_KERNEL, 2) == _lib.CHOL_ERR_INVALID_ARG
    assert lib.chol_set_option(_lib.CHOL_OPT_MID_KERNEL, 0) == _lib.CHOL_OK
    try:
        assert int(lib.chol_launch_count(256, 128)) == 2    # diagonal-block launch + copy
        assert int(lib.chol_workspace_bytes(256, 128)) > 0
        assert int(lib.chol_launch_count(7, 100)) > 1
        assert int(lib.chol_launch_count(7, 200)) > 1
    finally:
        lib.chol_set_option(_lib.CHOL_OPT_MID_KERNEL, 1)
    assert int(lib.chol_launch_count(297, 255)) > 1           # past the wide kernel's batches
    assert int(lib.chol_launch_count(8, 256)) > 1             # n % 64 == 0: blocked
    assert int(lib.chol_launch_count(8, 257)) > 1             # past n = 256


def test_workspace_regions():
    lib = _lib.load()
    ws = lambda b, n: int(lib.chol_workspace_bytes(b, n))
    assert ws(1024, 64) == 0                           # small kernel: no workspace
    # required region: one 64 x 64 inverse block per matrix
    required = lambda b: b * 64 * 64 * 4
    # one panel, large batch, n % 128 == 0 (128-wide chain): + one 128 x 128 inverse per matrix
    assert ws(640, 512) == required(640) + 640 * 128 * 128 * 4
    # ... n % 128 != 0 (64-wide chain): only the required region
    assert ws(400, 320) == required(400)
    # one panel, small batch (diagonal-block kernel): + n/64 inverse blocks and the tile
    # flags per matrix, + a ticket counter
    assert ws(4, 256) == required(4) + 4 * (4 * 64 * 64 * 4 + 768 * 4) + 256
    # several panels: + panel buffer (n x 512), V (512 x 512), flags, one ticket per panel
    n = 2048
    assert ws(1, n) == required(1) + n * 512 * 4 + 512 * 512 * 4 + 768 * 4 + 256
    # rows that are not 16-byte multiples: only the required region
    assert ws(2, 1030) == required(2)


def test_reference_arm_prints_its_line():
    out = subprocess.run(
        [sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "3",
         "--warmup", "3", "--cpu-budget", "0.5"],
        capture_output=True, text=True, timeout=300, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["metric"] == "matrices/s" and line["value"] > 0
    assert line["cpu_baseline"]["kind"] == "reference"
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
