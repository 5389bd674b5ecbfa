"""Evaluator-facing module with the reference's submission signature.

Reference: submission.py:1-7 (``custom_kernel(data: input_t) -> output_t``), imported by
the evaluator as ``from submission import custom_kernel``
(references/popcorn-eval/eval.py:126-133). ``input_t``/``output_t`` come from the
evaluator's ``task`` module when present, else they are ``torch.Tensor``.
"""

import torch

try:  # the evaluator provides `task`; outside it the types are plain tensors
    from task import input_t, output_t  # type: ignore
except ImportError:  # pragma: no cover - depends on the caller's environment
    input_t = output_t = torch.Tensor

from .cholesky import custom_kernel as _custom_kernel


def custom_kernel(data: input_t) -> output_t:
    return _custom_kernel(data)
