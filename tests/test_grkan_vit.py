"""GR-KAN ViT (the model that calls KAT_Group) on the CPU: the ViT-B/16 configuration has the
shapes the activation kernels are benchmarked on, the KAN block follows the reference
README's layer order, a training step runs with the CPU KAT formulation, and a
DistributedDataParallel step over two gloo ranks reproduces the single-process gradients."""

import os
import socket
import subprocess
import sys
import tempfile

import pytest
import torch

from rational_kat_cu_b200 import KAT_Group
from rational_kat_cu_b200 import grkan_vit as gv

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def tiny_cfg(**kw):
    base = dict(image_size=32, patch_size=16, num_classes=10, embed_dim=64, depth=2,
                num_heads=2, num_groups=4)
    base.update(kw)
    return gv.ViTConfig(**base)


def test_vit_b16_configuration():
    cfg = gv.vit_b16()
    assert (cfg.depth, cfg.embed_dim, cfg.num_heads, int(cfg.embed_dim * cfg.mlp_ratio)) == \
        (12, 768, 12, 3072)
    assert cfg.num_tokens == 197
    with torch.device("meta"):
        model = gv.GRKANViT(cfg, kat_device="cpu")
    kats = model.kat_modules()
    assert len(kats) == 24
    # act1 'identity', act2 'gelu' in every block; 8 groups
    for blk in model.blocks:
        assert isinstance(blk.mlp.act1, KAT_Group) and isinstance(blk.mlp.act2, KAT_Group)
        assert blk.mlp.act1.num_groups == 8
    n_params = sum(p.numel() for p in model.parameters())
    # ViT-B/16 has 86.57 M parameters; the KAN MLP adds 24 x (6 + 8 * 4) coefficients.
    assert n_params == 86567656 + 24 * (6 + 32)


def test_kan_block_layer_order():
    """act1 -> drop -> fc1 -> act2 -> drop -> fc2 (README.md:44-51)."""
    kan = gv.KAN(16, 64, num_groups=4, device="cpu")
    order = [name for name, _ in kan.named_children()]
    assert order == ["act1", "drop1", "fc1", "act2", "drop2", "fc2"]
    calls = []
    for name, mod in kan.named_children():
        mod.register_forward_hook(lambda m, i, o, name=name: calls.append(name))
    kan(torch.randn(2, 3, 16))
    assert calls == order
    # act1 starts as the identity, act2 as the GELU fit
    x = torch.randn(4, 16)
    assert torch.allclose(kan.act1(x), x, atol=1e-6)


def test_training_step_cpu_formulation():
    torch.manual_seed(0)
    cfg = tiny_cfg()
    model = gv.GRKANViT(cfg, kat_device="cpu")
    opt = gv.make_optimizer(model, lr=1e-3)
    images, labels = gv.synthetic_batch(4, cfg, dtype=torch.float32, seed=1)
    before = [p.detach().clone() for p in model.parameters()]
    losses = [gv.train_step(model, opt, images, labels).item() for _ in range(5)]
    assert all(torch.isfinite(torch.tensor(losses)))
    assert losses[-1] < losses[0]
    for b, p in zip(before, model.parameters()):
        assert p.grad is not None
    # the KAT coefficients are trained too
    k = model.kat_modules()[1]
    assert k.weight_denominator.grad is not None and k.weight_denominator.grad.abs().sum() > 0


def test_synthetic_batch_is_seeded():
    cfg = tiny_cfg()
    a = gv.synthetic_batch(3, cfg, dtype=torch.bfloat16, seed=5)
    b = gv.synthetic_batch(3, cfg, dtype=torch.bfloat16, seed=5)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
    assert a[0].dtype == torch.bfloat16 and a[0].shape == (3, 3, 32, 32)
    assert int(a[1].max()) < cfg.num_classes


def test_wrap_rejects_unknown_exchange():
    with pytest.raises(ValueError):
        gv.wrap_data_parallel(torch.nn.Linear(2, 2), kat_exchange="nccl")


def test_coefficient_names():
    model = gv.GRKANViT(tiny_cfg(), kat_device="cpu")
    names = gv.coefficient_names(model)
    assert len(names) == 2 * len(model.kat_modules())
    assert names[0] == "blocks.0.mlp.act1.weight_numerator"


WORKER = r'''
import os, sys, datetime
sys.path.insert(0, {repo!r})
import torch, torch.distributed as dist
from rational_kat_cu_b200 import grkan_vit as gv
rank, world, out = int(sys.argv[1]), int(sys.argv[2]), sys.argv[3]
dist.init_process_group("gloo", init_method="tcp://127.0.0.1:{port}", rank=rank,
                        world_size=world, timeout=datetime.timedelta(seconds=30))
cfg = gv.ViTConfig(image_size=32, patch_size=16, num_classes=10, embed_dim=64, depth=2,
                   num_heads=2, num_groups=4)
torch.manual_seed(0)
model = gv.GRKANViT(cfg, kat_device="cpu")
images, labels = gv.synthetic_batch(8, cfg, dtype=torch.float32, seed=3)
ddp = gv.wrap_data_parallel(model, kat_exchange="ddp")
lo, hi = 8 * rank // world, 8 * (rank + 1) // world
loss = torch.nn.functional.cross_entropy(ddp(images[lo:hi]), labels[lo:hi])
loss.backward()
torch.save({{n: p.grad for n, p in model.named_parameters()}}, f"{{out}}.{{rank}}.pt")
dist.destroy_process_group()
'''


def test_ddp_step_matches_single_process():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    code = WORKER.format(repo=REPO, port=port)
    with tempfile.TemporaryDirectory() as td:
        out = os.path.join(td, "g")
        env = dict(os.environ, MASTER_ADDR="127.0.0.1", OMP_NUM_THREADS="2")
        procs = [subprocess.Popen([sys.executable, "-c", code, str(r), "2", out],
                                  stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True,
                                  env=env) for r in range(2)]
        for p in procs:
            try:
                so, se = p.communicate(timeout=240)
            except subprocess.TimeoutExpired:
                p.kill()
                so, se = p.communicate()
            assert p.returncode == 0, se[-3000:]
        g0 = torch.load(out + ".0.pt")
        g1 = torch.load(out + ".1.pt")
    cfg = tiny_cfg()
    torch.manual_seed(0)
    model = gv.GRKANViT(cfg, kat_device="cpu")
    images, labels = gv.synthetic_batch(8, cfg, dtype=torch.float32, seed=3)
    torch.nn.functional.cross_entropy(model(images), labels).backward()
    for n, p in model.named_parameters():
        assert torch.equal(g0[n], g1[n]), n           # every rank holds the same average
        scale = p.grad.abs().max().item() + 1e-12
        assert (g0[n] - p.grad).abs().max().item() <= 1e-5 * scale, n
