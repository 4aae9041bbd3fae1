"""KAT_Group2D: group-rational activation for NCHW input ([B, C, H, W]).

Drop-in for the reference's kat_rational/kat_2dgroup_triton.py:8-95: same constructor,
parameters and init.json presets; forward calls RationalCUDA2D (sm_100a kernels).  As in
the reference (kat_2dgroup_triton.py:31), device="cpu" is rejected.
"""

from __future__ import annotations

import json

import torch
import torch.nn as nn

from ._init_table import INIT_JSON
from .rational_cuda import SHARED_ROW_MAX_GROUPS, KatGroupFunction, RationalCUDA2D


class KAT_Group2D(nn.Module):
    def __init__(self, num_groups: int = 8, mode: str = "gelu", device: str = "cuda"):
        super().__init__()
        assert device in ["cuda", "cpu"], "Device must be either 'cuda' or 'cpu'."
        self.order = (5, 4)
        self.num_groups = num_groups
        self.initialize(mode=mode)
        if device == "cuda":
            self.rational = RationalCUDA2D.apply
        else:
            assert False, "Only CUDA is supported for 2D group-wise processing."

    def init_info(self) -> dict:
        with open(INIT_JSON) as json_file:
            return json.load(json_file)

    def initialize(self, mode: str = "gelu") -> None:
        """Set the coefficients from an init.json preset (kat_2dgroup_triton.py:45-69)."""
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
        assert input.dim() == 4, "Input tensor must be 4D (batch, channels, height, width)."
        exchange = getattr(self, "exchange", None)
        if exchange is not None or self.rational == RationalCUDA2D.apply:
            # up to SHARED_ROW_MAX_GROUPS groups the numerator row goes to the kernels as is
            # (no repeat / sum launches); the same choice with and without the exchange
            shared = self.num_groups <= SHARED_ROW_MAX_GROUPS
            num = (self.weight_numerator if shared
                   else self.weight_numerator.repeat(self.num_groups, 1))
            return KatGroupFunction.apply(input, num, self.weight_denominator, self.num_groups,
                                          True, exchange, shared)
        weight_numerator = self.weight_numerator.repeat(self.num_groups, 1)
        return self.rational(input, weight_numerator, self.weight_denominator, self.num_groups)

    def enable_data_parallel(self, group=None, average: bool = True,
                             timeout_ms: int = 5000) -> None:
        """Exchange this module's coefficient gradients with the other ranks of `group`
        inside the backward's reduction kernel (NVLink peer memory, one node, up to 8 ranks):
        every rank then holds the same rank-order sum (average by default).  Collective: call
        it on every rank, in the same module order."""
        from .distributed import PeerExchange

        self.exchange = PeerExchange(self.num_groups, group=group, average=average,
                                     timeout_ms=timeout_ms,
                                     device=self.weight_denominator.device)

    def disable_data_parallel(self) -> None:
        """Collective: release the exchange buffers enable_data_parallel set up (call it on
        every rank, after the last backward through them) and return to the local backward."""
        exchange = getattr(self, "exchange", None)
        self.exchange = None
        if exchange is not None:
            exchange.close()

    def extra_repr(self) -> str:
        return f"num_groups={self.num_groups}, order={self.order}"
