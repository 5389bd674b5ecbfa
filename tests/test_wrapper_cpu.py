"""CPU: the Python drop-in wrapper's host logic (no GPU work)."""

import re
from pathlib import Path

import pytest
import torch

from linalg_kernels_b200 import cholesky as chol_mod
from linalg_kernels_b200 import submission

ROOT = Path(__file__).resolve().parents[1]


def test_cpu_input_raises_no_fallback():
    a = torch.eye(4).expand(2, 4, 4).contiguous()
    with pytest.raises(TypeError, match="GPU only"):
        chol_mod.custom_kernel(a)
    with pytest.raises(TypeError):
        submission.custom_kernel(a)


def test_non_tensor_rejected():
    with pytest.raises(TypeError):
        chol_mod.custom_kernel([[1.0]])


def test_no_torch_linalg_fallback_in_product_path():
    """The product modules never call torch.linalg.cholesky* or the oracle."""
    for f in (ROOT / "linalg_kernels_b200").glob("*.py"):
        text = f.read_text()
        assert not re.search(r"torch\.linalg\.cholesky\w*\s*\(", text), f
        assert "import oracle" not in text and "from oracle" not in text, f


def test_submission_files_avoid_banned_token():
    """The evaluator rejects any submission source containing the word spelled
    s-t-r-e-a-m (reference AGENTS.md:28); the drop-in modules stay clean of it."""
    token = "".join(["s", "t", "r", "e", "a", "m"])
    for name in ("cholesky.py", "submission.py"):
        text = (ROOT / "linalg_kernels_b200" / name).read_text().lower()
        assert token not in text, name


def test_signature_matches_reference():
    import inspect

    params = list(inspect.signature(submission.custom_kernel).parameters)
    assert params == ["data"]
