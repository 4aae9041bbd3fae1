"""GR-KAN ViT-B/16: the Vision Transformer whose MLP blocks use the group-rational
activation, and its data-parallel training step.

This is the caller of the KAT_Group kernels in a real model.  The reference ships only the
KAN MLP block (README.md:20-51): act1 = KAT_Group('identity') on the block input, dropout,
fc1, act2 = KAT_Group('gelu') on the hidden activations, dropout, fc2.  The scaffolding
around it is the standard ViT-B/16 layout, written here in plain PyTorch (no timm):

  16x16 patch embedding (a stride-16 convolution) -> class token + learned position
  embedding (197 tokens for a 224x224 image) -> 12 pre-norm blocks
  (LayerNorm -> multi-head self-attention, 12 heads of 64 -> residual;
   LayerNorm -> KAN MLP 768 -> 3072 -> 768 -> residual) -> LayerNorm -> linear head on the
  class token (1000 classes).

At batch 128, act1 sees [128, 197, 768] and act2 [128, 197, 3072] in every block.  Attention
uses torch's scaled_dot_product_attention; the linear layers are cuBLAS GEMMs, except that with
`fused_gemm=True` the KAN block's fc1 -> act2 -> fc2 runs on the tcgen05 GEMMs with act2 in
their epilogues (fused_gemm.KANMlpFused: act2's forward in fc1's epilogue, its backward in the
epilogue of fc2's input-gradient GEMM).

Training step: cross-entropy on the class logits, backward, optimizer step.  Data parallel
is one process per GPU with DistributedDataParallel over NCCL; the KAT coefficient
gradients either ride DDP's buckets (kat_exchange="ddp") or are left out of DDP and
exchanged inside each KAT backward kernel over NVLink peer memory (kat_exchange="fused",
KAT_Group.enable_data_parallel).
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import List, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import fused_gemm
from .kat_1dgroup import KAT_Group


@dataclass
class ViTConfig:
    image_size: int = 224
    patch_size: int = 16
    in_chans: int = 3
    num_classes: int = 1000
    embed_dim: int = 768
    depth: int = 12
    num_heads: int = 12
    mlp_ratio: float = 4.0
    num_groups: int = 8          # KAT_Group groups
    drop: float = 0.0
    act: str = "kat"             # "kat" (GR-KAN) or "gelu" (plain ViT MLP)
    fused_gemm: bool = False     # KAN block: act2 in the fc1 / fc2-dgrad GEMM epilogues

    @property
    def num_tokens(self) -> int:
        return (self.image_size // self.patch_size) ** 2 + 1


def vit_b16(**overrides) -> ViTConfig:
    """ViT-B/16 at 224x224: 12 layers, width 768, MLP 3072, 12 heads."""
    return ViTConfig(**overrides)


class KAN(nn.Module):
    """The KAN MLP block of the reference README (README.md:20-51):
    act1 -> drop -> fc1 -> act2 -> drop -> fc2, act1 initialised 'identity', act2 'gelu'."""

    def __init__(self, in_features: int, hidden_features: int, num_groups: int = 8,
                 act_init=("identity", "gelu"), drop: float = 0.0, device: str = "cuda",
                 fused_gemm: bool = False):
        super().__init__()
        self.act1 = KAT_Group(num_groups=num_groups, mode=act_init[0], device=device)
        self.drop1 = nn.Dropout(drop)
        self.fc1 = nn.Linear(in_features, hidden_features)
        self.act2 = KAT_Group(num_groups=num_groups, mode=act_init[1], device=device)
        self.drop2 = nn.Dropout(drop)
        self.fc2 = nn.Linear(hidden_features, in_features)
        self.fused_gemm = fused_gemm

    def _fusable(self, x: torch.Tensor) -> bool:
        """The fused GEMM path applies to bf16 CUDA activations and weights, without dropout
        between act2 and fc2 and without act2's in-kernel gradient exchange."""
        return (self.fused_gemm and x.is_cuda and x.dtype == torch.bfloat16
                and self.fc1.weight.dtype == torch.bfloat16
                and self.fc2.weight.dtype == torch.bfloat16
                and (self.drop2.p == 0.0 or not self.training)
                and getattr(self.act2, "exchange", None) is None
                and fused_gemm.supports(x.numel() // x.shape[-1], self.fc1.out_features,
                                        self.fc1.in_features, self.act2.num_groups))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x = self.act1(x)
        x = self.drop1(x)
        if self._fusable(x):
            return fused_gemm.kan_mlp_fused(x, self.fc1, self.act2, self.fc2)
        x = self.fc1(x)
        x = self.act2(x)
        x = self.drop2(x)
        return self.fc2(x)


class GeluMLP(nn.Module):
    """The plain ViT MLP (fc1 -> GELU -> fc2), for comparison runs."""

    def __init__(self, in_features: int, hidden_features: int, drop: float = 0.0):
        super().__init__()
        self.fc1 = nn.Linear(in_features, hidden_features)
        self.fc2 = nn.Linear(hidden_features, in_features)
        self.drop = nn.Dropout(drop)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.fc2(self.drop(F.gelu(self.fc1(x))))


class Attention(nn.Module):
    def __init__(self, dim: int, num_heads: int):
        super().__init__()
        self.num_heads = num_heads
        self.qkv = nn.Linear(dim, dim * 3)
        self.proj = nn.Linear(dim, dim)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        B, L, C = x.shape
        qkv = self.qkv(x).view(B, L, 3, self.num_heads, C // self.num_heads).permute(2, 0, 3, 1, 4)
        q, k, v = qkv.unbind(0)   # (indexing would make its backward zero-fill the whole qkv)
        o = F.scaled_dot_product_attention(q, k, v)
        return self.proj(o.transpose(1, 2).reshape(B, L, C))


class Block(nn.Module):
    def __init__(self, cfg: ViTConfig, kat_device: str):
        super().__init__()
        dim = cfg.embed_dim
        hidden = int(dim * cfg.mlp_ratio)
        self.norm1 = nn.LayerNorm(dim, eps=1e-6)
        self.attn = Attention(dim, cfg.num_heads)
        self.norm2 = nn.LayerNorm(dim, eps=1e-6)
        if cfg.act == "kat":
            self.mlp = KAN(dim, hidden, cfg.num_groups, drop=cfg.drop, device=kat_device,
                           fused_gemm=cfg.fused_gemm)
        else:
            self.mlp = GeluMLP(dim, hidden, cfg.drop)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x = x + self.attn(self.norm1(x))
        return x + self.mlp(self.norm2(x))


class GRKANViT(nn.Module):
    """ViT with KAN MLP blocks.  `kat_device` is the KAT_Group device argument ("cuda" for
    the sm_100a kernels, "cpu" for the PyTorch formulation)."""

    def __init__(self, cfg: Optional[ViTConfig] = None, kat_device: str = "cuda"):
        super().__init__()
        cfg = cfg or ViTConfig()
        self.cfg = cfg
        dim = cfg.embed_dim
        self.patch_embed = nn.Conv2d(cfg.in_chans, dim, cfg.patch_size, cfg.patch_size)
        self.cls_token = nn.Parameter(torch.zeros(1, 1, dim))
        self.pos_embed = nn.Parameter(torch.zeros(1, cfg.num_tokens, dim))
        self.blocks = nn.ModuleList([Block(cfg, kat_device) for _ in range(cfg.depth)])
        self.norm = nn.LayerNorm(dim, eps=1e-6)
        self.head = nn.Linear(dim, cfg.num_classes)
        self.reset_parameters()

    @torch.no_grad()
    def reset_parameters(self) -> None:
        """Truncated-normal(0.02) linear weights and embeddings, zero biases, unit LayerNorm;
        the KAT coefficients keep their init.json presets."""
        nn.init.trunc_normal_(self.pos_embed, std=0.02)
        nn.init.trunc_normal_(self.cls_token, std=0.02)
        fan_in = self.patch_embed.in_channels * self.patch_embed.kernel_size[0] ** 2
        nn.init.trunc_normal_(self.patch_embed.weight, std=math.sqrt(1.0 / fan_in))
        nn.init.zeros_(self.patch_embed.bias)
        for m in self.modules():
            if isinstance(m, nn.Linear):
                nn.init.trunc_normal_(m.weight, std=0.02)
                nn.init.zeros_(m.bias)
            elif isinstance(m, nn.LayerNorm):
                nn.init.ones_(m.weight)
                nn.init.zeros_(m.bias)

    def kat_modules(self) -> List[KAT_Group]:
        return [m for m in self.modules() if isinstance(m, KAT_Group)]

    def forward(self, images: torch.Tensor) -> torch.Tensor:
        x = self.patch_embed(images).flatten(2).transpose(1, 2)
        x = torch.cat([self.cls_token.expand(x.shape[0], -1, -1), x], dim=1) + self.pos_embed
        for blk in self.blocks:
            x = blk(x)
        return self.head(self.norm(x)[:, 0])


def coefficient_names(model: nn.Module) -> List[str]:
    """Parameter names of every KAT coefficient tensor in `model`."""
    return [n for n, _ in model.named_parameters()
            if n.endswith("weight_numerator") or n.endswith("weight_denominator")]


def wrap_data_parallel(model: nn.Module, kat_exchange: str = "ddp", device_ids=None,
                       timeout_ms: int = 20000, **ddp_kwargs) -> nn.Module:
    """DistributedDataParallel around `model` (process group already initialised).

    kat_exchange="ddp": every parameter, KAT coefficients included, is averaged by DDP's
    bucketed all-reduce.  kat_exchange="fused": DDP skips the KAT coefficients and each
    KAT_Group exchanges them inside its backward kernel (rank-order fp64 average over NVLink
    peer memory, KAT_Group.enable_data_parallel); one node, CUDA only."""
    from torch.nn.parallel import DistributedDataParallel as DDP

    if kat_exchange not in ("ddp", "fused"):
        raise ValueError(f"kat_exchange must be 'ddp' or 'fused', got {kat_exchange!r}")
    if kat_exchange == "fused":
        DDP._set_params_and_buffers_to_ignore_for_model(model, coefficient_names(model))
        for m in model.modules():
            if isinstance(m, KAT_Group):
                m.enable_data_parallel(timeout_ms=timeout_ms)
    return DDP(model, device_ids=device_ids, **ddp_kwargs)


def make_optimizer(model: nn.Module, lr: float = 1e-4, weight_decay: float = 0.05,
                   capturable: bool = False):
    """AdamW; the fused CUDA implementation when the parameters are on a GPU (capturable=True
    for use inside a CUDA graph)."""
    params = list(model.parameters())
    fused = bool(params) and params[0].is_cuda
    return torch.optim.AdamW(params, lr=lr, weight_decay=weight_decay, fused=fused,
                             capturable=capturable and fused)


def train_step(model: nn.Module, optimizer, images: torch.Tensor,
               labels: torch.Tensor) -> torch.Tensor:
    """One training step: forward, cross-entropy, backward, optimizer step.  Returns the
    (detached) loss on the device."""
    logits = model(images)
    loss = F.cross_entropy(logits.float(), labels)
    optimizer.zero_grad(set_to_none=True)
    loss.backward()
    optimizer.step()
    return loss.detach()


class GraphedTrainStep:
    """The whole training step — forward, loss, backward and the optimizer update — captured
    once in a CUDA graph and replayed, so a step costs its kernels and not the ~800 Python-side
    launches of an eager step.  Inputs are copied into static device buffers before each replay.
    The optimizer must be capturable (make_optimizer(capturable=True)).  One process per GPU,
    no DistributedDataParallel inside (the fused KAT coefficient exchange may be inside)."""

    def __init__(self, model: nn.Module, optimizer, images: torch.Tensor, labels: torch.Tensor,
                 warmup: int = 3):
        self.model, self.optimizer = model, optimizer
        self.images = images.detach().clone()
        self.labels = labels.detach().clone()
        side = torch.cuda.Stream(self.images.device)
        side.wait_stream(torch.cuda.current_stream(self.images.device))
        with torch.cuda.stream(side):
            for _ in range(warmup):
                train_step(model, optimizer, self.images, self.labels)
        torch.cuda.current_stream(self.images.device).wait_stream(side)
        optimizer.zero_grad(set_to_none=True)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            logits = model(self.images)
            self.loss = F.cross_entropy(logits.float(), self.labels)
            self.loss.backward()
            optimizer.step()

    def __call__(self, images: torch.Tensor = None, labels: torch.Tensor = None) -> torch.Tensor:
        """Replay one step (after copying new inputs in, if given); returns the loss tensor
        (device, overwritten by the next replay)."""
        if images is not None:
            self.images.copy_(images, non_blocking=True)
        if labels is not None:
            self.labels.copy_(labels, non_blocking=True)
        self.graph.replay()
        return self.loss


def synthetic_batch(batch: int, cfg: ViTConfig, dtype=torch.bfloat16, seed: int = 0,
                    device: Optional[torch.device] = None):
    """Images ~ N(0, 1) [batch, 3, H, W] in `dtype` and uniform labels in [0, classes),
    generated on the CPU from `seed` (pinned when a CUDA device will consume them)."""
    gen = torch.Generator().manual_seed(seed)
    images = torch.randn(batch, cfg.in_chans, cfg.image_size, cfg.image_size,
                         generator=gen).to(dtype)
    labels = torch.randint(0, cfg.num_classes, (batch,), generator=gen)
    if device is not None and device.type == "cuda":
        images, labels = images.pin_memory(), labels.pin_memory()
    return images, labels
