"""GR-KAN ViT on the GPU: the model with the sm_100a KAT kernels against the same model whose
activations are the oracle's restatement of the reference formulation (same weights, same
inputs, every other layer identical), a bf16 training run, and the data-parallel wrapper's
two coefficient-gradient exchanges agreeing bit for bit at world size 1."""

import copy
import os
import socket
import subprocess
import sys

import pytest
import torch

from oracle import kat_torch_oracle
from rational_kat_cu_b200 import grkan_vit as gv

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def small_cfg(**kw):
    base = dict(image_size=64, patch_size=16, num_classes=10, embed_dim=128, depth=2,
                num_heads=4, num_groups=8)
    base.update(kw)
    return gv.ViTConfig(**base)


def oracle_model(model):
    """A copy of `model` whose KAT modules evaluate the oracle's formulation."""
    ref = copy.deepcopy(model)
    for m in ref.kat_modules():
        m.rational = kat_torch_oracle.rational_1dgroup
    return ref


@pytest.fixture
def strict_fp32():
    old = (torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32)
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = old


def _step(model, images, labels):
    logits = model(images)
    loss = torch.nn.functional.cross_entropy(logits, labels)
    loss.backward()
    return logits.detach(), loss.detach(), {n: p.grad for n, p in model.named_parameters()}


def test_vit_step_matches_oracle_activations(cuda_device, strict_fp32):
    """Logits, loss and every parameter gradient of one step, from the model with the
    sm_100a KAT kernels and from the same model with the oracle's fp32 activations, are both
    compared with the same model run entirely in float64: the kernel model's error may not
    exceed a small multiple of the oracle model's own fp32 error."""
    from torch.nn.attention import SDPBackend, sdpa_kernel

    torch.manual_seed(0)
    cfg = small_cfg()
    model = gv.GRKANViT(cfg).to(cuda_device)
    # perturb the coefficients away from their presets so every term is exercised
    g = torch.Generator().manual_seed(4)
    with torch.no_grad():
        for m in model.kat_modules():
            m.weight_numerator.add_(0.05 * torch.randn(1, 6, generator=g).to(cuda_device))
            m.weight_denominator.add_(0.05 * torch.randn(8, 4, generator=g).to(cuda_device))
    ref32 = oracle_model(model)
    ref64 = oracle_model(model).double()
    images, labels = gv.synthetic_batch(6, cfg, dtype=torch.float32, seed=2)
    images, labels = images.to(cuda_device), labels.to(cuda_device)
    with sdpa_kernel(SDPBackend.MATH):
        ours = _step(model, images, labels)
        o32 = _step(ref32, images, labels)
        o64 = _step(ref64, images.double(), labels)

    def err(a, b):
        return (a.double() - b).abs().max().item()

    report = []
    pairs = [("logits", ours[0], o32[0], o64[0]), ("loss", ours[1], o32[1], o64[1])]
    pairs += [(n, ours[2][n], o32[2][n], o64[2][n]) for n in o64[2]]
    assert len(pairs) == 2 + len(list(model.parameters()))
    bad = []
    for name, a, b, t in pairs:
        assert a is not None, name
        scale = t.abs().max().item()
        e_ours, e_ref = err(a, t), err(b, t)
        report.append((name, e_ours, e_ref, scale))
        if e_ours > max(4.0 * e_ref, 1e-5 * scale, 1e-12):
            bad.append((name, e_ours, e_ref, scale))
    worst = max(report, key=lambda r: r[1] / (r[3] + 1e-30))
    print("worst relative error (ours, oracle fp32):", worst)
    assert not bad, bad


def test_vit_bf16_training_decreases_loss(cuda_device):
    torch.manual_seed(0)
    cfg = small_cfg()
    model = gv.GRKANViT(cfg).to(cuda_device, dtype=torch.bfloat16)
    opt = gv.make_optimizer(model, lr=1e-3)
    images, labels = gv.synthetic_batch(16, cfg, dtype=torch.bfloat16, seed=7)
    images, labels = images.to(cuda_device), labels.to(cuda_device)
    losses = [gv.train_step(model, opt, images, labels).item() for _ in range(12)]
    assert all(torch.isfinite(torch.tensor(losses)))
    assert losses[-1] < 0.8 * losses[0]
    for m in model.kat_modules():
        assert m.weight_numerator.dtype == torch.bfloat16
        assert torch.isfinite(m.weight_denominator).all()


def test_graphed_train_step_tracks_eager(cuda_device):
    """The CUDA-graph step (forward, backward, fused AdamW replayed) follows the eager step's
    loss trajectory on the same model, data and optimizer settings."""
    cfg = small_cfg()
    images, labels = gv.synthetic_batch(16, cfg, dtype=torch.bfloat16, seed=11)
    images, labels = images.to(cuda_device), labels.to(cuda_device)
    losses = {}
    for mode in ("eager", "graph"):
        torch.manual_seed(0)
        model = gv.GRKANViT(cfg).to(cuda_device, dtype=torch.bfloat16)
        opt = gv.make_optimizer(model, lr=1e-3, capturable=(mode == "graph"))
        if mode == "graph":
            # the three warm-up steps before capture are ordinary training steps
            step = gv.GraphedTrainStep(model, opt, images, labels, warmup=3)
            losses[mode] = [step().item() for _ in range(8)]
        else:
            all_losses = [gv.train_step(model, opt, images, labels).item() for _ in range(11)]
            losses[mode] = all_losses[3:]
    torch.testing.assert_close(torch.tensor(losses["graph"]), torch.tensor(losses["eager"]),
                               rtol=2e-2, atol=2e-2)
    assert losses["graph"][-1] < losses["graph"][0]


WORKER = r'''
import os, sys, datetime
sys.path.insert(0, {repo!r})
import torch, torch.distributed as dist
from rational_kat_cu_b200 import grkan_vit as gv
dist.init_process_group("nccl", init_method="tcp://127.0.0.1:{port}", rank=0, world_size=1,
                        timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", 0))
torch.cuda.set_device(0)
cfg = gv.ViTConfig(image_size=64, patch_size=16, num_classes=10, embed_dim=128, depth=2,
                   num_heads=4, num_groups=8)
images, labels = gv.synthetic_batch(8, cfg, dtype=torch.float32, seed=3)
images, labels = images.cuda(), labels.cuda()
grads = {{}}
for mode in ("ddp", "fused"):
    torch.manual_seed(0)
    model = gv.GRKANViT(cfg).cuda()
    ddp = gv.wrap_data_parallel(model, kat_exchange=mode, device_ids=[0], timeout_ms=5000)
    torch.nn.functional.cross_entropy(ddp(images), labels).backward()
    torch.cuda.synchronize()
    grads[mode] = {{n: p.grad.detach().clone() for n, p in model.named_parameters()}}
    for m in model.kat_modules():
        if getattr(m, "exchange", None) is not None:
            m.exchange.close()
    del ddp, model
bad = [n for n in grads["ddp"] if not torch.equal(grads["ddp"][n], grads["fused"][n])]
print("MISMATCH", bad if bad else "none")
dist.destroy_process_group()
'''


def test_fused_and_ddp_exchange_agree_at_world_one(cuda_device):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    env = dict(os.environ, MASTER_ADDR="127.0.0.1", NCCL_NVLS_ENABLE="0")
    p = subprocess.run([sys.executable, "-c", WORKER.format(repo=REPO, port=port)],
                       capture_output=True, text=True, timeout=300, env=env)
    assert p.returncode == 0, p.stderr[-3000:]
    assert "MISMATCH none" in p.stdout, p.stdout[-2000:]


def test_fused_gemm_blocks_match_unfused(cuda_device):
    """KAN blocks with fc1 -> act2 -> fc2 on the fused tcgen05 GEMMs against the same blocks on
    torch linears + the activation kernels: same weights and inputs, bf16; logits, loss and
    every gradient agree to bf16 accuracy, and a graphed fused training run learns."""
    cfg = small_cfg()
    images, labels = gv.synthetic_batch(16, cfg, dtype=torch.bfloat16, seed=5)
    images, labels = images.to(cuda_device), labels.to(cuda_device)
    out = {}
    for fused in (False, True):
        torch.manual_seed(0)
        model = gv.GRKANViT(small_cfg(fused_gemm=fused)).to(cuda_device, dtype=torch.bfloat16)
        assert all(b.mlp._fusable(torch.empty(1, 1, cfg.embed_dim, device=cuda_device,
                                              dtype=torch.bfloat16)) == fused
                   for b in model.blocks)
        out[fused] = _step(model, images, labels)
    (lu, su, gu), (lf, sf, gf) = out[False], out[True]

    def rel(a, b):
        return float((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-30))

    assert rel(lf, lu) < 2e-2
    assert abs(float(sf) - float(su)) < 2e-2 * max(1.0, abs(float(su)))
    for name in gu:
        assert rel(gf[name], gu[name]) < 5e-2, name

    torch.manual_seed(0)
    model = gv.GRKANViT(small_cfg(fused_gemm=True)).to(cuda_device, dtype=torch.bfloat16)
    opt = gv.make_optimizer(model, lr=1e-3, capturable=True)
    step = gv.GraphedTrainStep(model, opt, images, labels, warmup=3)
    losses = [step().item() for _ in range(10)]
    assert all(torch.isfinite(torch.tensor(losses)))
    assert losses[-1] < 0.9 * losses[0]
