"""Generate the golden vectors in this directory by running the REFERENCE implementation.

Imports the reference's own PyTorch path, kat_rational/kat_1dgroup_torch.py of
felippe-alves/rational_kat_cu (KAT_Group_Torch / Rational_CUDA_A_1DGroup), straight from
its source file, runs forward + torch-autograd backward on seeded inputs, and stores
inputs, outputs and gradients as small .npz fixtures plus a JSON manifest:

  golden_small.npz / cases.json   a dozen small cases: channels-last [B,L,C], [B,C], NCHW,
                                  fp32 / bf16 / fp16 inputs, every init.json mode, odd and
                                  12-wide groups, random coefficients
  golden_cfg1.npz                 the KAT_Group fp32 workload x[8,197,768] (seed 0),
                                  grad_out seed 1, G=8, 'gelu': a 4096-element sample of
                                  x / y / dx, checksums, and the full coefficient gradients

Conventions the reference forces (it has no other entry for these cases):
  [B, C] input  -> viewed as [1, B, C];  NCHW -> permute to [B, H*W, C] and back;
  bf16 / fp16   -> values upcast to fp32 before the reference (its bmm rejects mixed
                   dtypes); outputs are stored unrounded in fp32.

Usage (needs the reference checkout; the fixtures are committed):
  python tests/golden/make_golden.py /path/to/rational_kat_cu   (or set KAT_REFERENCE_ROOT)
"""

from __future__ import annotations

import importlib.util
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
def reference_root() -> str:
    """The reference checkout: the first command-line argument, else $KAT_REFERENCE_ROOT."""
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("KAT_REFERENCE_ROOT")
    if not root:
        sys.exit("usage: python tests/golden/make_golden.py /path/to/rational_kat_cu "
                 "(or set KAT_REFERENCE_ROOT)")
    return root


def load_reference(ref_root: str):
    path = os.path.join(ref_root, "kat_rational", "kat_1dgroup_torch.py")
    spec = importlib.util.spec_from_file_location("reference_kat_1dgroup_torch", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def gen(shape, seed, scale=1.0):
    return torch.randn(*shape, generator=torch.Generator().manual_seed(seed)) * scale


def run_reference(ref, x, gy, group, mode, layout, coef=None):
    """Forward + autograd backward through the reference module KAT_Group_Torch."""
    m = ref.KAT_Group_Torch(num_groups=group, mode=mode)
    if coef is not None:
        with torch.no_grad():
            m.weight_numerator.copy_(coef[0])
            m.weight_denominator.copy_(coef[1])
    xin = x.detach().clone().requires_grad_(True)
    if layout == "blc":
        y = m(xin)
    elif layout == "bc":
        y = m(xin.view(1, *xin.shape)).view(xin.shape)
    elif layout == "nchw":
        B, C, H, W = xin.shape
        y3 = m(xin.permute(0, 2, 3, 1).reshape(B, H * W, C))
        y = y3.view(B, H, W, C).permute(0, 3, 1, 2)
    else:
        raise ValueError(layout)
    y.backward(gy)
    return (y.detach().contiguous(), xin.grad.contiguous(), m.weight_numerator.detach().clone(),
            m.weight_denominator.detach().clone(), m.weight_numerator.grad.clone(),
            m.weight_denominator.grad.clone())


def small_cases(init_table):
    cases = [
        dict(name="gelu_blc_f32", shape=(2, 5, 64), layout="blc", G=8, mode="gelu", dtype="f32"),
        dict(name="identity_blc_f32", shape=(3, 7, 32), layout="blc", G=8, mode="identity",
             dtype="f32"),
        dict(name="random_blc_f32", shape=(2, 3, 48), layout="blc", G=4, mode="random",
             dtype="f32", x_scale=2.0),
        dict(name="gelu_bc_f32", shape=(6, 48), layout="bc", G=4, mode="gelu", dtype="f32"),
        dict(name="gelu_nchw_f32", shape=(2, 16, 5, 7), layout="nchw", G=4, mode="gelu",
             dtype="f32"),
        dict(name="identity_nchw_f32", shape=(2, 16, 3, 3), layout="nchw", G=8,
             mode="identity", dtype="f32"),
        dict(name="gelu_pert_blc_bf16", shape=(2, 4, 64), layout="blc", G=8, mode="gelu_pert",
             dtype="bf16"),
        dict(name="gelu_blc_f16", shape=(2, 4, 64), layout="blc", G=8, mode="gelu",
             dtype="f16"),
        dict(name="odd_group_f32", shape=(3, 5, 36), layout="blc", G=12, mode="gelu",
             dtype="f32"),
        dict(name="g64_blc_bf16", shape=(2, 3, 768), layout="blc", G=64, mode="gelu_pert",
             dtype="bf16"),
        dict(name="gelu_nchw_bf16", shape=(2, 8, 7, 7), layout="nchw", G=8, mode="gelu_pert",
             dtype="bf16"),
    ]
    for mode in init_table:
        cases.append(dict(name=f"mode_{mode}", shape=(2, 3, 32), layout="blc", G=4, mode=mode,
                          dtype="f32"))
    return cases


def quantize(t, dtype):
    if dtype == "bf16":
        return t.to(torch.bfloat16).float()
    if dtype == "f16":
        return t.to(torch.float16).float()
    return t


def main(ref_root: str) -> None:
    ref = load_reference(ref_root)
    with open(os.path.join(ref_root, "kat_rational", "init.json")) as fh:
        init_table = json.load(fh)
    arrays, manifest = {}, []
    for case in small_cases(init_table):
        G = case["G"]
        x = quantize(gen(case["shape"], 0, case.get("x_scale", 1.0)), case["dtype"])
        gy = quantize(gen(case["shape"], 1), case["dtype"])
        coef, mode = None, case["mode"]
        if mode == "random":
            mode = "gelu"
            coef = (gen((1, 6), 3, 0.5), gen((G, 4), 4, 0.5))
        elif mode == "gelu_pert":
            mode = "gelu"
            base_n = torch.tensor(init_table["gelu"]["init_w_numerator"]).view(1, 6)
            base_d = torch.tensor(init_table["gelu"]["init_w_denominator"]).repeat(G, 1)
            coef = (base_n + gen((1, 6), 2, 0.01), base_d + gen((G, 4), 5, 0.01))
        y, dx, wn, wd, dwn, dwd = run_reference(ref, x, gy, G, mode, case["layout"], coef)
        key = case["name"]
        for name, t in (("x", x), ("grad_out", gy), ("y", y), ("dx", dx), ("w_num", wn),
                        ("w_den", wd), ("d_num", dwn), ("d_den", dwd)):
            arrays[f"{key}/{name}"] = t.numpy().astype(np.float32)
        manifest.append({k: (list(v) if isinstance(v, tuple) else v) for k, v in case.items()})
    np.savez_compressed(os.path.join(HERE, "golden_small.npz"), **arrays)
    with open(os.path.join(HERE, "cases.json"), "w") as fh:
        json.dump(manifest, fh, indent=1)

    # The 1.2 M-element fp32 workload: sampled elements and checksums.
    shape, G = (8, 197, 768), 8
    x = gen(shape, 0)
    gy = gen(shape, 1)
    y, dx, wn, wd, dwn, dwd = run_reference(ref, x, gy, G, "gelu", "blc")
    idx = np.sort(np.random.default_rng(7).choice(x.numel(), size=4096, replace=False))
    flat = lambda t: t.reshape(-1).numpy()
    np.savez_compressed(
        os.path.join(HERE, "golden_cfg1.npz"),
        shape=np.array(shape), groups=np.array(G), index=idx,
        x_sample=flat(x)[idx], y_sample=flat(y)[idx], dx_sample=flat(dx)[idx],
        x_sum=np.array(x.double().sum().item()), x_sumsq=np.array((x.double() ** 2).sum().item()),
        gy_sum=np.array(gy.double().sum().item()),
        y_sum=np.array(y.double().sum().item()), dx_sum=np.array(dx.double().sum().item()),
        w_num=wn.numpy(), w_den=wd.numpy(), d_num=dwn.numpy(), d_den=dwd.numpy())
    print(f"wrote {len(manifest)} small cases and the [8,197,768] sample to {HERE}")


if __name__ == "__main__":
    main(reference_root())
