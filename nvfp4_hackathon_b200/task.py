"""Input/output types of the two drop-in entry points.

Same tuple layouts as the reference's task contracts:
kernels/gemm/task.py:4-5 (7-tuple) and kernels/group_gemm/task.py:4-5 (4-tuple of lists).
"""
from typing import TypeVar

import torch

# (a, b, sfa, sfb, sfa_permuted, sfb_permuted, c)
gemm_input_t = TypeVar(
    "gemm_input_t",
    bound=tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor,
                torch.Tensor, torch.Tensor])
gemm_output_t = TypeVar("gemm_output_t", bound=torch.Tensor)

# ([(a, b, c)], [(sfa, sfb)], [(sfa_permuted, sfb_permuted)], [(m, n, k, l)])
group_input_t = TypeVar(
    "group_input_t",
    bound=tuple[list[tuple[torch.Tensor, torch.Tensor, torch.Tensor]],
                list[tuple[torch.Tensor, torch.Tensor]],
                list[tuple[torch.Tensor, torch.Tensor]],
                list[tuple[int, int, int, int]]])
group_output_t = TypeVar("group_output_t", bound=list[torch.Tensor])

