"""Generate tests/golden/golden.npz from the reference implementation itself.

Imports the reference's ``cholesky/cholesky.py`` (Mark123M/linalg-kernels) with a stub
``task`` module, exactly as the reference's own harness does
(cholesky/b4096n32/cholesky_b4096n32_modal.py:201-209), and calls its ``custom_kernel`` on
CPU tensors. For CPU input the reference takes its fallback branch,
``torch.linalg.cholesky_ex(data, check_errors=False).L`` (cholesky/cholesky.py:5850), i.e.
LAPACK SPOTRF from the MKL bundled with torch. The outputs L (and info from
``torch.linalg.cholesky_ex``) are stored next to the inputs.

Run in the build container (the reference tree is not present on GPU boxes):
    python tests/golden/make_golden.py /path/to/reference
"""

from __future__ import annotations

import importlib.util
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from linalg_kernels_b200 import inputs  # noqa: E402


def load_reference(root: Path):
    task = types.ModuleType("task")
    task.input_t = torch.Tensor
    task.output_t = torch.Tensor
    sys.modules.setdefault("task", task)
    spec = importlib.util.spec_from_file_location("reference_cholesky",
                                                  root / "cholesky" / "cholesky.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def cases():
    """(name, A float32 (b,n,n), cond per matrix) — small, seeded, CPU-generated."""
    out = []
    # the benchmark families at small batch
    for b, n, lam, seed in [(8, 32, 1e2, 41032), (4, 64, 1e3, 41064), (1, 256, 1e3, 41256)]:
        a, cond = inputs.spectral(b, n, lam, seed)
        out.append((f"spectral_b{b}n{n}", a, cond))
    for b, n, shift, seed in [(1, 192, 1.0, 510512), (1, 130, 0.5, 48284)]:
        a, cond = inputs.covariance(b, n, shift, seed)
        out.append((f"covariance_b{b}n{n}", a, cond))
    # structural case families (the reference harness's set, our constants)
    for name, b, n, seed in [("diagonal", 4, 32, 1203), ("tridiagonal", 2, 64, 32526),
                             ("lowrank", 3, 48, 32524), ("spectrum", 4, 32, 1202),
                             ("rowscale", 2, 64, 32525), ("dense", 2, 16, 53124),
                             ("spectrum", 2, 128, 1200), ("diagonal", 1, 128, 1201)]:
        a = inputs.case(name, b, n, seed)
        ev = torch.linalg.eigvalsh(a.double())
        out.append((f"{name}_b{b}n{n}", a, ev[:, -1] / ev[:, 0]))
    # ragged / edge sizes
    for n in (1, 2, 3, 5, 7, 17, 31, 33, 63, 65, 100, 127, 129):
        b = 3 if n < 64 else 1
        a, _ = inputs.spectral(b, n, 50.0, 7000 + n)
        ev = torch.linalg.eigvalsh(a.double())
        out.append((f"edge_b{b}n{n}", a, ev[:, -1] / ev[:, 0]))
    # only the lower triangle may be read: garbage above the diagonal
    a, cond = inputs.spectral(2, 40, 30.0, 99)
    g = torch.Generator().manual_seed(5)
    junk = torch.randn(2, 40, 40, generator=g) * 1e3
    a_junk = torch.where(torch.ones(40, 40, dtype=torch.bool).triu(1), junk, a)
    out.append(("upper_garbage_b2n40", a_junk.contiguous(), cond))
    return out


def not_spd_cases():
    """Inputs with a non-positive leading minor; only info is compared."""
    out = []
    a, _ = inputs.spectral(3, 24, 10.0, 123)
    a = a.clone()
    a[1, 10, 10] = -1.0  # matrix 1 fails at column 11 at the latest
    a[2, 0, 0] = 0.0  # matrix 2 fails at column 1
    out.append(("notspd_b3n24", a))
    a, _ = inputs.covariance(1, 96, 1.0, 321)
    a = a.clone()
    a[0, 80, 80] = -5.0
    out.append(("notspd_b1n96", a))
    return out


def main(argv):
    if len(argv) < 2:
        raise SystemExit("usage: python tests/golden/make_golden.py <path to the reference tree>")
    root = Path(argv[1])
    ref = load_reference(root)
    store: dict[str, np.ndarray] = {}
    names = []
    for name, a, cond in cases():
        l_ref = ref.custom_kernel(a)
        store[f"{name}/A"] = a.numpy()
        store[f"{name}/L"] = l_ref.numpy()
        store[f"{name}/cond"] = np.asarray(cond, dtype=np.float64)
        names.append(name)
    bad = []
    for name, a in not_spd_cases():
        res = torch.linalg.cholesky_ex(a, check_errors=False)
        store[f"{name}/A"] = a.numpy()
        store[f"{name}/info"] = res.info.numpy().astype(np.int32)
        bad.append(name)
    store["_names"] = np.array(names)
    store["_notspd"] = np.array(bad)
    store["_torch"] = np.array(torch.__version__)
    store["_lapack"] = np.array("MKL 2024.2 via torch.linalg.cholesky_ex (reference fallback)")
    np.savez_compressed(HERE / "golden.npz", **store)
    print(f"wrote {HERE / 'golden.npz'}: {len(names)} factor cases, {len(bad)} non-SPD cases")


if __name__ == "__main__":
    main(sys.argv)
