"""The fused-GEMM host layer on the CPU: which shapes the kernels take, the errors for tensors
they cannot take (raised before anything reaches the library), and the KAN block's choice
between the fused GEMMs and the unfused layers."""

import pytest
import torch

from rational_kat_cu_b200 import fused_gemm as fg
from rational_kat_cu_b200 import grkan_vit as gv


@pytest.mark.parametrize("m,n,k,g,ok", [
    (25216, 3072, 768, 8, True),      # ViT-B/16 MLP, act2
    (1, 256, 64, 1, True),
    (1000, 768, 256, 8, True),        # 96 columns per group
    (128, 3072, 768, 64, False),      # 48 columns per group: not a multiple of 32
    (128, 300, 64, 1, False),         # N not a multiple of 256
    (128, 256, 100, 1, False),        # K not a multiple of 64
    (0, 256, 64, 1, True),           # empty batch: a no-op
    (-1, 256, 64, 1, False),
    (128, 512, 64, 3, False),         # groups do not divide N
])
def test_supported_shapes(m, n, k, g, ok):
    assert fg.supports(m, n, k, g) is ok


def test_cpu_tensors_are_rejected():
    a = torch.zeros(128, 64, dtype=torch.bfloat16)
    b = torch.zeros(256, 64, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        fg.gemm_bf16(a, b)
    with pytest.raises(RuntimeError, match="CUDA"):
        fg.gemm_rational_fwd(a, b, None, torch.zeros(1, 6), torch.zeros(1, 4), 1)
    with pytest.raises(RuntimeError, match="CUDA"):
        fg.gemm_rational_bwd(a, b, torch.zeros(128, 256, dtype=torch.bfloat16),
                             torch.zeros(1, 6), torch.zeros(1, 4), 1)


def test_kan_block_uses_unfused_layers_where_fusion_does_not_apply():
    torch.manual_seed(0)
    kan = gv.KAN(128, 512, num_groups=8, device="cpu", fused_gemm=True)
    x = torch.randn(2, 5, 128)
    assert not kan._fusable(x)                    # CPU tensor
    ref = gv.KAN(128, 512, num_groups=8, device="cpu", fused_gemm=False)
    ref.load_state_dict(kan.state_dict())
    torch.testing.assert_close(kan(x), ref(x))
    kan.drop2.p = 0.1
    kan.train()
    assert not kan._fusable(x)
    cfg = gv.ViTConfig(image_size=32, patch_size=16, num_classes=10, embed_dim=128, depth=1,
                       num_heads=4, fused_gemm=True)
    model = gv.GRKANViT(cfg, kat_device="cpu")
    assert all(b.mlp.fused_gemm for b in model.blocks)
