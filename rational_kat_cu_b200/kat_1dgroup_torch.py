"""Explicit PyTorch (CPU-capable) formulation: KAT_Group_Torch and KAT_Group(device="cpu").

The reference exports a pure-PyTorch module next to the CUDA one
(kat_rational/kat_1dgroup_torch.py:27-155, exported at kat_rational/__init__.py:4).  This
file keeps that API: `Rational_CUDA_A_1DGroup(x, weight_numerator, weight_denominator,
group)` on [B, L, D] input, and `KAT_Group_Torch(num_groups, mode)`.  It evaluates the same
formula, y = P(x) / (1 + sum |b_i| x^i), by Horner's rule on grouped views with torch
autograd for the backward.  It is selected only on explicit request (device="cpu" or this
class); the CUDA modules never route through it.
"""

from __future__ import annotations

import json

import torch
from torch import nn

from ._init_table import INIT_JSON


def Rational_CUDA_A_1DGroup(x: torch.Tensor, weight_numerator: torch.Tensor,
                            weight_denominator: torch.Tensor, group: int) -> torch.Tensor:
    """P(x)/Q(x) per channel group on x [B, L, D]; weight_numerator [group, len_num],
    weight_denominator [group, len_den]."""
    B, L, D = x.shape
    z = x.view(B, L, group, D // group)
    a = weight_numerator.view(group, -1).unsqueeze(-1)          # [G, n, 1]
    c = weight_denominator.view(group, -1).abs().unsqueeze(-1)  # [G, m, 1]
    p = a[:, -1]
    for k in range(a.shape[1] - 2, -1, -1):
        p = p * z + a[:, k]
    q = c[:, -1]
    for i in range(c.shape[1] - 2, -1, -1):
        q = q * z + c[:, i]
    q = q * z + 1.0
    return (p / q).view(B, L, D)


class KAT_Group_Torch(nn.Module):
    def __init__(self, num_groups: int = 8, mode: str = "gelu"):
        super().__init__()
        self.order = (5, 4)
        self.num_groups = num_groups
        self.initialize(mode=mode)

    def init_info(self) -> dict:
        with open(INIT_JSON) as json_file:
            return json.load(json_file)

    def initialize(self, mode: str = "gelu") -> None:
        try:
            with open(INIT_JSON) as json_file:
                data = json.load(json_file)
            weight_numerator = torch.tensor(data[mode]["init_w_numerator"]).view(1, -1)
            weight_denominator = torch.tensor(data[mode]["init_w_denominator"])
            weight_denominator = torch.cat([weight_denominator] * self.num_groups).view(
                self.num_groups, -1)
            self.weight_numerator = nn.Parameter(weight_numerator.float(), requires_grad=True)
            self.weight_denominator = nn.Parameter(weight_denominator.float(), requires_grad=True)
        except FileNotFoundError:
            print("Initialization JSON file not found.")
        except json.JSONDecodeError:
            print("Error decoding JSON.")

    def forward(self, input: torch.Tensor) -> torch.Tensor:
        assert input.dim() == 3, "Input tensor must be 3D. Of size (batch, length, channels)."
        weight_numerator = self.weight_numerator.repeat(self.num_groups, 1)
        return Rational_CUDA_A_1DGroup(input, weight_numerator, self.weight_denominator,
                                       self.num_groups)

    def extra_repr(self) -> str:
        return f"num_groups={self.num_groups}, order={self.order}"
