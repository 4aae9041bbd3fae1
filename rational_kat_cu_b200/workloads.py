"""Seeded synthetic workloads of the group-rational benchmark configurations.

No public dataset is involved: each configuration is a tensor shape, a dtype, an input
distribution and a coefficient preset, generated from fixed seeds:

  kat_group_f32      KAT_Group fp32, x[8,197,768] ~ N(0,1) seed 0, grad_out seed 1,
                     G=8, 'gelu' coefficients
  kat_group_vitb_bf16  KAT_Group bf16 at the ViT-B MLP-hidden shape x[128,197,3072]
                     ~ N(0,1) seed 0, grad_out seed 1, G=8, 'gelu' coefficients plus
                     N(0, 0.01) perturbations (numerator then denominator, seed 2)
  kat_group2d_f32    KAT_Group2D fp32 NCHW x[64,256,56,56] ~ N(0,1) seed 0, grad_out
                     seed 1, G=8, 'identity' coefficients
  sweep(C, G, N, dtype)  x[N/C, C] ~ N(0, 2), grad_out ~ N(0, 1), numerator [1,6] and
                     denominator [G,4] ~ N(0, 0.5) (seed 3); N rounded down to a multiple of C
  rat_cuda_vitb_bf16 the abs-after-sum formula (rat_cuda) at the same ViT-B MLP-hidden shape
                     x[128,197,3072] bf16 ~ N(0,1), G=8, numerator [6] and denominator [G,4]
                     ~ N(0, 0.5) (seed 3)
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional, Tuple

import torch

from ._init_table import load_table

DTYPES = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}


@dataclass
class Workload:
    name: str
    shape: Tuple[int, ...]
    layout: str            # "blc" (channels-last) or "nchw"
    groups: int
    dtype: str             # "f32", "bf16", "f16"
    mode: str              # init.json preset, or "random"
    x_std: float = 1.0
    perturb: float = 0.0
    coef_seed: int = 2
    x_seed: int = 0
    gy_seed: int = 1
    formula: int = 0       # 0: KAT (Q = 1 + sum |b_i| x^i), 1: abs after sum (rat_cuda)
    meta: dict = field(default_factory=dict)

    @property
    def numel(self) -> int:
        n = 1
        for s in self.shape:
            n *= s
        return n

    def coefficients(self) -> Tuple[torch.Tensor, torch.Tensor]:
        """(numerator [1, 6], denominator [G, 4]) fp32 on the CPU."""
        G = self.groups
        if self.mode == "random":
            gen = torch.Generator().manual_seed(self.coef_seed)
            return (torch.randn(1, 6, generator=gen) * 0.5, torch.randn(G, 4, generator=gen) * 0.5)
        table = load_table()[self.mode]
        num = torch.tensor(table["init_w_numerator"], dtype=torch.float32).view(1, 6)
        den = torch.tensor(table["init_w_denominator"], dtype=torch.float32).repeat(G, 1)
        if self.perturb:
            gen = torch.Generator().manual_seed(self.coef_seed)
            num = num + torch.randn(1, 6, generator=gen) * self.perturb
            den = den + torch.randn(G, 4, generator=gen) * self.perturb
        return num, den

    def inputs(self, device: Optional[torch.device] = None):
        """(x, grad_out) in the workload dtype.  Generated on the CPU with torch.Generator
        (reproducible anywhere) unless `device` is a CUDA device, where a seeded CUDA
        generator is used (faster for the large sweep points)."""
        dt = DTYPES[self.dtype]
        if device is not None and device.type == "cuda":
            gx = torch.Generator(device=device).manual_seed(self.x_seed)
            gg = torch.Generator(device=device).manual_seed(self.gy_seed)
            x = torch.randn(self.shape, generator=gx, device=device, dtype=torch.float32)
            if self.x_std != 1.0:
                x.mul_(self.x_std)
            x = x.to(dt)
            gy = torch.randn(self.shape, generator=gg, device=device, dtype=torch.float32).to(dt)
            return x, gy
        x = torch.randn(self.shape, generator=torch.Generator().manual_seed(self.x_seed))
        if self.x_std != 1.0:
            x.mul_(self.x_std)
        gy = torch.randn(self.shape, generator=torch.Generator().manual_seed(self.gy_seed))
        return x.to(dt), gy.to(dt)

    def dims(self) -> Tuple[int, int, int]:
        """(batch, channels, inner) of the contiguous tensor."""
        if self.layout == "nchw":
            B, C, H, W = self.shape
            return B, C, H * W
        C = self.shape[-1]
        return self.numel // C, C, 1


def kat_group_f32() -> Workload:
    return Workload("kat_group_f32", (8, 197, 768), "blc", 8, "f32", "gelu")


def kat_group_vitb_bf16() -> Workload:
    return Workload("kat_group_vitb_bf16", (128, 197, 3072), "blc", 8, "bf16", "gelu",
                    perturb=0.01, coef_seed=2)


def kat_group2d_f32() -> Workload:
    return Workload("kat_group2d_f32", (64, 256, 56, 56), "nchw", 8, "f32", "identity")


def sweep(channels: int, groups: int, numel: int, dtype: str) -> Workload:
    rows = max(1, numel // channels)
    return Workload(f"sweep_c{channels}_g{groups}_n{rows * channels}_{dtype}", (rows, channels),
                    "blc", groups, dtype, "random", x_std=2.0, coef_seed=3)


def rat_cuda_vitb_bf16() -> Workload:
    return Workload("rat_cuda_vitb_bf16", (128, 197, 3072), "blc", 8, "bf16", "random",
                    coef_seed=3, formula=1)


BY_NAME = {
    "kat_group_f32": kat_group_f32,
    "kat_group_vitb_bf16": kat_group_vitb_bf16,
    "kat_group2d_f32": kat_group2d_f32,
    "rat_cuda_vitb_bf16": rat_cuda_vitb_bf16,
}


def get(name: str) -> Workload:
    """A workload by name: one of BY_NAME, or "sweep:C:G:N:dtype" for a sweep point."""
    if name.startswith("sweep:"):
        _, c, g, n, dt = name.split(":")
        return sweep(int(c), int(g), int(n), dt)
    return BY_NAME[name]()


def sweep_points():
    """The bandwidth-sweep points bench.py --sweep measures: C in {768, 3072, 8192},
    G in {8, 16, 64}, N = 2^20 .. 2^30 elements, bf16 / fp32 / fp16, plus 2^31 elements at
    C = 3072, G = 8 in bf16 and fp32."""
    pts = []
    for dt in ("bf16", "f32", "f16"):
        for c in (768, 3072, 8192):
            for g in (8, 16, 64):
                for logn in (20, 24, 28, 30):
                    pts.append((c, g, 1 << logn, dt))
    for dt in ("bf16", "f32"):
        pts.append((3072, 8, 1 << 31, dt))
    return pts
