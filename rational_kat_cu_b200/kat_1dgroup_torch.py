"""Explicit PyTorch (CPU-capable) formulation: KAT_Group_Torch and KAT_Group(device="cpu").

The reference exports a pure-PyTorch module next to the CUDA one
(kat_rational/kat_1dgroup_torch.py:27-155, exported at kat_rational/__init__.py:4).  This
file keeps that API: `Rational_CUDA_A_1DGroup(x, weight_numerator, weight_denominator,
group)` on [B, L, D] input, and `KAT_Group_Torch(num_groups, mode)`.  Its results are defined
by a sequence of tensor operations, so this file performs the same sequence — group-major
copy, a table of powers built by repeated products, one batched matrix product per
polynomial with the denominator's coefficients padded and made non-negative, the quotient,
the layout restored — and torch autograd differentiates it: on the same machine the values and
gradients equal the reference's bit for bit.  It is selected only on explicit request
(device="cpu" or this class); the CUDA modules never route through it.
"""

from __future__ import annotations

import json

import torch
from torch import nn

from ._init_table import INIT_JSON


def _power_table(z: torch.Tensor, count: int) -> torch.Tensor:
    """[G, count, M]: z**0 .. z**(count - 1) for z [G, M], each power the previous one times z
    (kat_1dgroup_torch.py:7-24 builds its table the same way)."""
    cols = [torch.ones_like(z), z]
    while len(cols) < count:
        cols.append(cols[-1] * z)
    return torch.stack(cols[:count], dim=1)


def Rational_CUDA_A_1DGroup(x: torch.Tensor, weight_numerator: torch.Tensor,
                            weight_denominator: torch.Tensor, group: int) -> torch.Tensor:
    """P(x)/Q(x) per channel group on x [B, L, D]; weight_numerator [group, n],
    weight_denominator [group, m]; Q = 1 + sum_i |b_i| x^i (kat_1dgroup_torch.py:27-78)."""
    B, L, D = x.shape
    per = D // group
    n, m = weight_numerator.size(1), weight_denominator.size(1)
    # One row per group: [G, B*L*per], channels of a group contiguous.
    z = x.view(B, L, group, per).permute(2, 0, 1, 3).contiguous().view(group, B * L * per)
    table = _power_table(z, max(n, m))
    num = torch.bmm(weight_numerator.unsqueeze(1), table).squeeze(1)
    den_coef = torch.cat([
        torch.ones(group, 1, device=x.device, dtype=weight_denominator.dtype),
        weight_denominator,
        torch.zeros(group, max(0, n - m - 1), device=x.device, dtype=weight_denominator.dtype),
    ], dim=1).abs()
    den = torch.bmm(den_coef.unsqueeze(1), table).squeeze(1)
    out = num.div(den)
    return out.view(group, B, L, per).permute(1, 2, 0, 3).contiguous().view(B, L, D)


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
