"""Benchmark: KAT_Group forward+backward throughput (Gelem/s) on B200, one process per GPU.

Workload (default): KAT_Group bf16 at the ViT-B MLP-hidden shape x[128,197,3072] ~ N(0,1),
num_groups=8, 'gelu' coefficients + N(0, 0.01) perturbation, grad_out ~ N(0,1) — the
configuration the headline metric is quoted on.  A step is one forward and one backward
pass of the module over that batch (y = mod(x); y.backward(gy)); with N GPUs every rank
processes its own batch (weak scaling) and the coefficient gradients are all-gathered over
NCCL and summed in rank order each step.

Printed (rank 0, one JSON line):
  value        whole-job Gelem/s with inputs resident in HBM (device-timed, CUDA events,
               max over ranks); each tensor (155 MB) is larger than the 126 MB L2
  e2e          the same step through the module with host buffers: pinned-host -> device
               copies of x and grad_out, forward+backward, device -> host copies of y, dx
               and the coefficient gradients, all inside the timed region
  roofline     the dominant kernel (the fused backward: read x, grad_out; write dx) against
               the measured HBM copy bandwidth in MEASURED_PEAKS.json
  cpu_baseline the reference's CPU path (the oracle's restatement of kat_1dgroup_torch.py,
               fp32 upcast) on a bounded sample of the same workload, on this host's cores
  clocks       SM clocks sampled with nvidia-smi while the GPU was busy

`--impl reference` times only the reference's CPU implementation (rank 0; other ranks exit).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

import torch  # noqa: E402

METRIC = "KAT_Group fwd+bwd Gelem/s"
UNIT = "Gelem/s"
FALLBACK_HBM_GBS = 6650.0
SPEC_HBM_GBS = 8000.0          # the ~8 TB/s HBM3e figure the fractions are also quoted against
L2_BYTES = 126 * 1024 * 1024


def bwd_kernel_names() -> str:
    """The kernels of one backward call for the streaming design in use."""
    mode = os.environ.get("KAT_RATIONAL_PIPELINE", "async")
    names = {"registers": "kat_bwd_kernel", "bulk": "kat_bwd_tma_kernel"}.get(
        mode, "kat_bwd_async_kernel")
    return names + " + kat_bwd_reduce_kernel (one C-ABI backward call)"


def metric_for(workload) -> str:
    return "rat_cuda fwd+bwd Gelem/s" if workload.formula == 1 else METRIC


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="kat_group_vitb_bf16")
    ap.add_argument("--no-graph", action="store_true", help="eager steps instead of a CUDA graph")
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--e2e-chunks", type=int, default=4,
                    help="row chunks the host-buffer pipeline overlaps")
    ap.add_argument("--kernel-iters", type=int, default=100)
    ap.add_argument("--cpu-seconds", type=float, default=30.0,
                    help="CPU budget of our line's reference-path baseline (median of 5 steps "
                         "after one warm-up, full batch when it fits the budget)")
    ap.add_argument("--ref-seconds", type=float, default=300.0,
                    help="CPU budget of the whole --impl reference run (full batch per step "
                         "when (steps + warmup) full steps fit, else a row sample)")
    ap.add_argument("--skip-cpu-baseline", action="store_true")
    ap.add_argument("--skip-gpu-bar", action="store_true",
                    help="do not time the reference's Triton kernels on this GPU")
    ap.add_argument("--skip-2d", action="store_true",
                    help="do not time the KAT_Group2D workload beside the headline")
    ap.add_argument("--gpu-bar-child", default=None, help=argparse.SUPPRESS)
    ap.add_argument("--sweep", action="store_true",
                    help="print one line per bandwidth-sweep point (kernel timings) instead")
    ap.add_argument("--sweep-logn", default="",
                    help="with --sweep: only the points with these log2(elements), e.g. 20,24")
    ap.add_argument("--vit-batch", type=int, default=128,
                    help="per-GPU batch of the GR-KAN ViT-B/16 training step (--workload "
                         "grkan_vit_b16)")
    ap.add_argument("--kat-exchange", choices=["ddp", "fused"], default="ddp",
                    help="how the ViT step exchanges the KAT coefficient gradients")
    ap.add_argument("--vit-eager", action="store_true",
                    help="eager ViT steps on one GPU instead of the captured CUDA graph")
    ap.add_argument("--vit-fused-gemm", dest="vit_fused_gemm", action="store_true", default=True,
                    help="ViT: KAN blocks run fc1 -> act2 -> fc2 on the tcgen05 GEMMs with act2 "
                         "in their epilogues (default)")
    ap.add_argument("--vit-unfused-gemm", dest="vit_fused_gemm", action="store_false",
                    help="ViT: KAN blocks on torch linear layers + the KAT_Group kernels")
    ap.add_argument("--vit-compare", action="store_true",
                    help="also time the ViT step with the reference's PyTorch KAT formulation "
                         "and with plain GELU MLPs (one GPU)")
    return ap.parse_args()


# ---------------------------------------------------------------------------
# Distributed plumbing
# ---------------------------------------------------------------------------

def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def init_process_group(world, rank, local):
    import datetime

    import torch.distributed as dist

    torch.cuda.set_device(local)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", local))
    return dist


def bind_to_gpu_numa(local: int) -> dict:
    """Restrict this process to the host CPUs next to GPU `local` (its PCI device's NUMA
    node), so that pinned host buffers allocated afterwards land in that node's memory.
    Returns what was found: node, CPU count and PCI address (or the reason it is unknown)."""
    try:
        props = torch.cuda.get_device_properties(local)
        bus = f"{props.pci_domain_id:04x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
        base = f"/sys/bus/pci/devices/{bus}"
        with open(base + "/numa_node") as fh:
            node = int(fh.read().strip())
        cpus = set()
        with open(base + "/local_cpulist") as fh:
            for part in fh.read().strip().split(","):
                if "-" in part:
                    lo, hi = part.split("-")
                    cpus.update(range(int(lo), int(hi) + 1))
                elif part:
                    cpus.add(int(part))
        usable = cpus & os.sched_getaffinity(0)
        if usable:
            os.sched_setaffinity(0, usable)
        return {"numa_node": node, "cpus": len(usable), "pci": bus}
    except Exception as e:  # no sysfs entry (containers, other platforms)
        return {"numa_node": None, "reason": f"{type(e).__name__}: {str(e)[:80]}"}


def host_link_gbs(dev, host: torch.Tensor, stream) -> dict:
    """H2D and D2H rates of one pinned host tensor's size on this rank (CUDA events)."""
    d = torch.empty(host.shape, dtype=host.dtype, device=dev)
    out = {}
    for name, fn in (("h2d_GBps", lambda: d.copy_(host, non_blocking=True)),
                     ("d2h_GBps", lambda: host.copy_(d, non_blocking=True))):
        fn()
        torch.cuda.synchronize(dev)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(3):
            fn()
        b.record(stream)
        torch.cuda.synchronize(dev)
        out[name] = 3 * host.numel() * host.element_size() / (a.elapsed_time(b) * 1e-3) / 1e9
    del d
    return out


# ---------------------------------------------------------------------------
# Clock sampling (nvidia-smi while the GPU works)
# ---------------------------------------------------------------------------

class ClockSampler:
    QUERY = ("uuid,clocks.sm,clocks.max.sm,utilization.gpu,power.draw,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.uuid = None
        try:
            u = str(torch.cuda.get_device_properties(device_index).uuid)
            self.uuid = u if u.startswith("GPU-") else "GPU-" + u
        except Exception:
            pass
        self.samples = []
        self.proc = None
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            if self.uuid and parts[0] != self.uuid:
                continue
            self.samples.append(parts[1:])

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=5)

    def summary(self):
        def num(s):
            try:
                return float(s)
            except ValueError:
                return None

        rows = [[num(s[0]), num(s[1]), num(s[2]), num(s[3])] + s[4:] for s in self.samples]
        busy = [r for r in rows if r[2] is not None and r[2] > 0 and r[0] is not None]
        use = busy if busy else [r for r in rows if r[0] is not None]
        if not use:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"],
                    "samples": 0}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in use for i, v in enumerate(r[4:8])
                          if str(v).strip().lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in use),
                "sm_max_mhz": max((r[1] for r in use if r[1] is not None), default=None),
                "reasons": reasons, "samples": len(use),
                "power_w_max": max((r[3] for r in use if r[3] is not None), default=None)}


# ---------------------------------------------------------------------------
# CPU baseline: the reference's CPU path (oracle restatement) on a bounded sample
# ---------------------------------------------------------------------------

def workload_config(w):
    """The `config` both arms print for workload `w` (identical, so the two lines compare)."""
    eb = {"f32": 4, "bf16": 2, "f16": 2}[w.dtype]
    tensor = w.numel * eb
    return {
        "workload": w.name, "shape": list(w.shape), "num_groups": w.groups, "io_dtype": w.dtype,
        "coefficients": "gelu + N(0,0.01)" if w.perturb else w.mode,
        "formula": "abs-after-sum (rat_cuda)" if w.formula == 1 else "KAT (kat_1dgroup_torch)",
        "layout": w.layout, "elements_per_gpu": w.numel,
        "l2": (f"inputs larger than L2 ({tensor / 1e6:.0f} MB per tensor > {L2_BYTES / 1e6:.0f} MB)"
               if tensor > L2_BYTES else "inputs fit in L2"),
    }


def cpu_reference_rate(workload, budget_s: float, steps: int = 5, warmup: int = 1):
    """Time fwd+bwd of the reference's PyTorch CPU path (restated in oracle/) on `workload`:
    `warmup` untimed steps, then `steps` timed ones; the rate is elements per step over the
    median step time.  Each step covers the full batch when (steps + warmup) full steps fit in
    `budget_s` (estimated from one row), else the largest row sample that does.  Returns
    (Gelem/s, dict describing the sample)."""
    from oracle import kat_torch_oracle

    torch.set_num_threads(os.cpu_count() or 1)
    cores = torch.get_num_threads()
    wn, wd = workload.coefficients()
    shape = list(workload.shape)
    row_elems = workload.numel // shape[0]

    def make(rows):
        s = [rows] + shape[1:]
        g = torch.Generator().manual_seed(0)
        x = torch.randn(*s, generator=g).to(torch.bfloat16 if workload.dtype == "bf16" else
                                            torch.float32 if workload.dtype == "f32" else
                                            torch.float16).float()
        gy = torch.randn(*s, generator=g).to(x.dtype)
        return x, gy

    def one(x, gy):
        if workload.formula == 1:
            from oracle import rat_torch_oracle

            rat_torch_oracle.rat_forward_backward(x.reshape(-1, shape[-1]), wn.reshape(6), wd,
                                                  gy.reshape(-1, shape[-1]))
            return
        kat_torch_oracle.forward_backward(x, wn, wd, workload.groups, gy,
                                          layout="nchw" if workload.layout == "nchw" else "blc")

    # calibrate on one row
    x, gy = make(1)
    one(x, gy)
    t0 = time.perf_counter()
    one(x, gy)
    per_row = max(time.perf_counter() - t0, 1e-4)
    steps = max(1, steps)
    n_calls = steps + warmup
    rows = int(max(1, min(shape[0], budget_s / n_calls / per_row)))
    x, gy = make(rows)
    for _ in range(warmup):
        one(x, gy)
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        one(x, gy)
        times.append(time.perf_counter() - t0)
    dt = statistics.median(times)
    elems = rows * row_elems
    full = rows == shape[0]
    return elems / dt / 1e9, {
        "cores": cores, "rows": rows, "full_batch": full, "elements": elems,
        "seconds_per_step": dt, "steps": steps, "warmup": warmup,
        "sample": (f"x[{rows},{','.join(str(s) for s in shape[1:])}] "
                   + ("(the full batch)" if full else f"(a {rows}-row sample)")
                   + f" of {workload.name} (fp32 upcast), fwd+bwd"
                   + (" (rat_cuda formula, the reference's PyTorch definition)"
                      if workload.formula == 1 else "")
                   + f", median of {steps} timed steps after {warmup} warm-up")}


def run_reference(args):
    world, rank, local = dist_setup()
    if rank != 0:
        return
    from rational_kat_cu_b200 import workloads

    w = workloads.get(args.workload)
    rate, info = cpu_reference_rate(w, budget_s=args.ref_seconds, steps=args.steps,
                                    warmup=args.warmup)
    line = {
        "metric": metric_for(w), "value": rate, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": info["seconds_per_step"] * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic", "impl": "reference",
        "config": workload_config(w),
        "sample_rows": info["rows"], "full_batch": info["full_batch"],
        "cpu_baseline": {"value": rate, "unit": UNIT, "cores": info["cores"], "kind": "port",
                         "sample": info["sample"]},
        "e2e": {"value": rate, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# Our arm
# ---------------------------------------------------------------------------

def measured_peak():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as fh:
            return float(json.load(fh)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


# DRAM bytes per backward launch from the committed ncu capture of the same kernel and workload.
NCU_BWD_TRAFFIC = {"kat_group_vitb_bf16": 309_906_688 + 124_804_864}


def run_ours(args):
    import rational_kat_cu_b200 as kat
    from rational_kat_cu_b200 import distributed as kdist
    from rational_kat_cu_b200 import workloads

    world, rank, local = dist_setup()
    dist = init_process_group(world, rank, local) if world > 1 else None
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    w = workloads.get(args.workload)
    w.x_seed += 1000 * rank
    w.gy_seed += 1000 * rank
    elem_bytes = {"f32": 4, "bf16": 2, "f16": 2}[w.dtype]
    N = w.numel

    wn, wd = w.coefficients()
    formula = w.formula
    if formula == 1:
        mod = kat.RatGroup(num_groups=w.groups).to(dev)
    else:
        cls = kat.KAT_Group2D if w.layout == "nchw" else kat.KAT_Group
        mod = cls(num_groups=w.groups, mode="gelu").to(dev)
    with torch.no_grad():
        mod.weight_numerator.copy_(wn.view_as(mod.weight_numerator))
        mod.weight_denominator.copy_(wd)
    eager_exchange = False
    if dist is not None and formula == 0:
        # Coefficient gradients are exchanged inside the backward's reduction kernel over
        # NVLink peer memory (no NCCL call on the step).
        mod.enable_data_parallel(timeout_ms=20000)
    elif dist is not None:
        eager_exchange = True   # rat_cuda: NCCL all-gather after the backward, eager steps
    x, gy = w.inputs(dev)
    x.requires_grad_(True)
    stream = torch.cuda.current_stream(dev)

    def step_eager():
        y = mod(x)
        y.backward(gy)
        if eager_exchange:
            kdist.allreduce_coefficient_grads(mod)
        return y

    # Warm up (also fills the workspace-size cache before any capture).
    side = torch.cuda.Stream(dev)
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        for _ in range(3):
            mod.zero_grad(set_to_none=True)
            x.grad = None
            step_eager()
    stream.wait_stream(side)
    torch.cuda.synchronize(dev)

    graph = None
    if not args.no_graph and not eager_exchange:
        mod.zero_grad(set_to_none=True)
        x.grad = None
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step_eager()
        torch.cuda.synchronize(dev)

    def step():
        if graph is not None:
            graph.replay()
        else:
            mod.zero_grad(set_to_none=True)
            x.grad = None
            step_eager()

    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()

    for _ in range(args.warmup):
        step()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(args.steps):
        step()
    end.record(stream)
    torch.cuda.synchronize(dev)
    if dist is not None:
        dist.barrier()
    ms_total = start.elapsed_time(end)
    if dist is not None:
        t = torch.tensor([ms_total], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_total = float(t.item())
    ms_per_step = ms_total / args.steps
    value = world * N / (ms_per_step * 1e-3) / 1e9

    # The coefficient gradients of the last step on every rank, compared bit for bit.
    grads = torch.cat([mod.weight_numerator.grad.reshape(-1).float(),
                       mod.weight_denominator.grad.reshape(-1).float()]).contiguous()
    grads_finite = bool(torch.isfinite(grads).all().item())
    if dist is not None:
        gathered = torch.empty(world, grads.numel(), device=dev, dtype=grads.dtype)
        dist.all_gather_into_tensor(gathered, grads)
        bits = gathered.view(torch.int32)
        grads_identical = bool((bits == bits[0:1]).all().item())
        fin = torch.tensor([1 if grads_finite else 0], device=dev)
        dist.all_reduce(fin, op=dist.ReduceOp.MIN)
        grads_finite = bool(fin.item())
    else:
        grads_identical = True

    # Kernel-level timing: back-to-back C-ABI launches on device-resident, preallocated
    # buffers (no Python work inside the loop beyond the call), CUDA events on the launching
    # stream around the whole run, average per launch.
    import ctypes

    from rational_kat_cu_b200 import _native

    lib = _native.lib()
    code = {"f32": _native.KAT_DTYPE_F32, "bf16": _native.KAT_DTYPE_BF16,
            "f16": _native.KAT_DTYPE_F16}[w.dtype]
    dims = w.dims()
    n_rep = wn.repeat(w.groups, 1).to(dev).contiguous()
    d_rep = wd.to(dev).contiguous()
    xs = x.detach()
    y_buf = torch.empty_like(xs)
    dx_buf = torch.empty_like(xs)
    dn_buf = torch.empty(w.groups, 6, device=dev)
    dd_buf = torch.empty(w.groups, 4, device=dev)
    ws_need = ctypes.c_size_t(0)
    _native.check("workspace", lib.kat_rational_bwd_workspace_size(
        dims[0], dims[1], dims[2], w.groups, code, dev.index, ctypes.byref(ws_need)))
    ws_buf = torch.empty(max(ws_need.value, 16), dtype=torch.uint8, device=dev)
    sp = ctypes.c_void_p(stream.cuda_stream)
    fwd_args = (xs.data_ptr(), y_buf.data_ptr(), n_rep.data_ptr(), d_rep.data_ptr(),
                dims[0], dims[1], dims[2], w.groups, code)
    bwd_args = (xs.data_ptr(), gy.data_ptr(), dx_buf.data_ptr(), n_rep.data_ptr(),
                d_rep.data_ptr(), dn_buf.data_ptr(), dd_buf.data_ptr(), ws_buf.data_ptr(),
                ws_buf.numel(), dims[0], dims[1], dims[2], w.groups, code)
    if formula == 0:
        fwd_fn, bwd_fn = lib.kat_rational_fwd, lib.kat_rational_bwd
        fwd_args, bwd_args = fwd_args + (sp,), bwd_args + (sp,)
    else:
        fwd_fn, bwd_fn = lib.kat_rational_fwd_formula, lib.kat_rational_bwd_formula
        fwd_args, bwd_args = fwd_args + (formula, sp), bwd_args + (formula, sp)

    def time_launches(fn, args, iters):
        for _ in range(3):
            _native.check("launch", fn(*args))
        torch.cuda.synchronize(dev)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(iters):
            fn(*args)
        b.record(stream)
        torch.cuda.synchronize(dev)
        return a.elapsed_time(b) / iters

    fwd_ms = time_launches(fwd_fn, fwd_args, args.kernel_iters)
    bwd_ms = time_launches(bwd_fn, bwd_args, args.kernel_iters)
    bwd_kernel_name = bwd_kernel_names()
    launches_per_step = 1 + bwd_kernel_name.count("+") + 1
    fwd_gbs = 2 * N * elem_bytes / (fwd_ms * 1e-3) / 1e9
    bwd_gbs = 3 * N * elem_bytes / (bwd_ms * 1e-3) / 1e9

    # End to end through the public host-buffer API: pinned host x, grad_out in; y, dx and
    # the coefficient gradients back in pinned host memory, copies overlapped with compute.
    from rational_kat_cu_b200.host_io import HostPipeline

    numa = bind_to_gpu_numa(local)
    h_x = torch.empty(w.shape, dtype=x.dtype, pin_memory=True)
    h_gy = torch.empty(w.shape, dtype=x.dtype, pin_memory=True)
    h_x.copy_(xs.cpu())
    h_gy.copy_(gy.cpu())
    h_y = torch.empty_like(h_x, pin_memory=True)
    h_dx = torch.empty_like(h_x, pin_memory=True)
    h_grads = [torch.empty(mod.weight_numerator.shape, pin_memory=True),
               torch.empty(mod.weight_denominator.shape, pin_memory=True)]
    pipe = HostPipeline(mod, chunks=args.e2e_chunks)

    def e2e_step():
        mod.zero_grad(set_to_none=True)
        if eager_exchange:
            pipe.run(h_x, h_gy, h_y, h_dx, wait=False)
            pipe.wait_compute()
            kdist.allreduce_coefficient_grads(mod)
            h_grads[0].copy_(mod.weight_numerator.grad, non_blocking=True)
            h_grads[1].copy_(mod.weight_denominator.grad, non_blocking=True)
        else:
            # data parallel: the pipeline exchanges the gradients through the module's
            # NVLink exchange buffers (no NCCL call)
            pipe.run(h_x, h_gy, h_y, h_dx, grads_host=h_grads, wait=False)

    for _ in range(2):
        e2e_step()
    pipe.wait()
    torch.cuda.synchronize(dev)
    if dist is not None:
        dist.barrier()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record(stream)
    for _ in range(args.e2e_steps):
        e2e_step()
    pipe.wait()
    e_end.record(stream)
    torch.cuda.synchronize(dev)
    e_ms = e_start.elapsed_time(e_end)
    if dist is not None:
        t = torch.tensor([e_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e_ms = float(t.item())
    e2e_ms_step = e_ms / args.e2e_steps
    e2e_value = world * N / (e2e_ms_step * 1e-3) / 1e9
    link = host_link_gbs(dev, h_x, stream)
    if dist is not None:
        rates = [None] * world
        dist.all_gather_object(rates, dict(link, **numa))
    else:
        rates = [dict(link, **numa)]
    h2d = 2 * N * elem_bytes
    d2h = 2 * N * elem_bytes + sum(h.numel() for h in h_grads) * 4

    clocks = None
    if sampler:
        sampler.stop()
        clocks = sampler.summary()

    cpu = None
    if rank == 0 and world == 1 and not args.skip_cpu_baseline:
        rate, info = cpu_reference_rate(w, budget_s=args.cpu_seconds, steps=5, warmup=1)
        cpu = {"value": rate, "unit": UNIT, "cores": info["cores"], "kind": "port",
               "sample": info["sample"]}

    # KAT_Group2D (x[64,256,56,56] fp32 NCHW, identity init) beside the headline, and the
    # reference's own Triton kernels on this GPU as a throughput bar (one GPU only).
    kat2d = None
    if rank == 0 and world == 1 and not args.skip_2d and w.name == "kat_group_vitb_bf16":
        kat2d = _kat2d_numbers(dev, stream, args)
    gpu_bar = None
    if rank == 0 and world == 1 and not args.skip_gpu_bar and w.formula == 0:
        names = ["kat_group_vitb_bf16", "kat_group2d_f32"] if w.name == "kat_group_vitb_bf16" \
            else [w.name]
        gpu_bar = _gpu_bar(local, names)

    if dist is not None:
        dist.barrier()
    if rank == 0:
        peak, peak_kind = measured_peak()
        step_bytes = 5 * N * elem_bytes
        line = {
            "metric": metric_for(w), "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": w.dtype, "data": "synthetic",
            "config": workload_config(w),
            "step": "module forward + backward" + (" in a CUDA graph" if graph else "")
                    + (" with the coefficient-gradient exchange fused into the reduction "
                       "kernel (NVLink peer stores)" if world > 1 and not eager_exchange
                       else "")
                    + (" and an NCCL all-gather of the coefficient gradients"
                       if eager_exchange else ""),
            "nranks": world, "grads_identical": grads_identical, "grads_finite": grads_finite,
            "roofline": {
                "bound": "hbm", "kernel": bwd_kernel_name,
                "achieved": bwd_gbs, "peak": peak, "unit": "GB/s", "frac": bwd_gbs / peak,
                "peak_source": f"{peak_kind} hbm_gbs",
                "frac_of_spec": bwd_gbs / SPEC_HBM_GBS,
                "spec_gbs": SPEC_HBM_GBS,
                "traffic": NCU_BWD_TRAFFIC.get(w.name),
                "traffic_source": ("ncu dram__bytes_read.sum + dram__bytes_write.sum of one "
                                   "kat_bwd_async_kernel launch, profiles/"
                                   "kat_bwd_async_kernel_kat_group_vitb_bf16.md (writes still in "
                                   "L2 at kernel end are not counted)")
                if w.name in NCU_BWD_TRAFFIC else None,
                "algorithmic_bytes_per_launch": 3 * N * elem_bytes,
                "ms_per_launch": bwd_ms,
            },
            "kernels": {
                "fwd_ms": fwd_ms, "fwd_GBps": fwd_gbs, "fwd_frac": fwd_gbs / peak,
                "fwd_frac_spec": fwd_gbs / SPEC_HBM_GBS,
                "bwd_ms": bwd_ms, "bwd_GBps": bwd_gbs, "bwd_frac": bwd_gbs / peak,
                "bwd_frac_spec": bwd_gbs / SPEC_HBM_GBS,
                "step_GBps": step_bytes / (ms_per_step * 1e-3) / 1e9,
                "step_hbm_frac": step_bytes * world / (ms_per_step * 1e-3) / 1e9 / (peak * world),
                "step_hbm_frac_spec": step_bytes / (ms_per_step * 1e-3) / 1e9 / SPEC_HBM_GBS,
                "fractions": f"of measured {peak:.0f} GB/s ({peak_kind}) and of the "
                             f"{SPEC_HBM_GBS:.0f} GB/s spec (_spec)",
            },
            "kat_group2d": kat2d,
            "gpu_bar": gpu_bar,
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d * world,
                    "d2h_bytes_per_step": d2h * world, "ms_per_step": e2e_ms_step,
                    "api": f"rational_kat_cu_b200.host_io.HostPipeline ({args.e2e_chunks} "
                           f"row chunks, H2D / compute / D2H overlapped, consecutive steps "
                           f"overlapped)",
                    "per_rank_host": rates},
            "gpu_launches": launches_per_step * args.steps * world,
            "cpu_baseline": cpu,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    if graph is not None:
        del graph
    if dist is not None:
        if getattr(mod, "exchange", None) is not None:
            mod.disable_data_parallel()       # collective: unmap, barrier, free
        dist.barrier()
        dist.destroy_process_group()


def _kat2d_numbers(dev, stream, args):
    """KAT_Group2D over x[64,256,56,56] fp32 NCHW (identity init, G=8): module forward and
    module forward + backward, each captured in a CUDA graph and timed over replays, and the
    C-ABI forward / backward launches back to back; fractions of the HBM bytes 2s / 3s / 5s
    per element against the measured peak and the spec figure."""
    import ctypes

    import rational_kat_cu_b200 as kat
    from rational_kat_cu_b200 import _native, workloads

    w = workloads.get("kat_group2d_f32")
    N = w.numel
    eb = 4
    mod = kat.KAT_Group2D(num_groups=w.groups, mode=w.mode).to(dev)
    x, gy = w.inputs(dev)
    x.requires_grad_(True)
    peak, _ = measured_peak()
    reps = max(5, min(args.steps, 50))

    def graphed(fn):
        side = torch.cuda.Stream(dev)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            for _ in range(3):
                fn()
        stream.wait_stream(side)
        torch.cuda.synchronize(dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        torch.cuda.synchronize(dev)
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize(dev)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(reps):
            g.replay()
        b.record(stream)
        torch.cuda.synchronize(dev)
        del g
        return a.elapsed_time(b) / reps

    def fwd_only():
        with torch.no_grad():
            mod(x)

    def fwd_bwd():
        mod.zero_grad(set_to_none=False)
        x.grad = None
        mod(x).backward(gy)

    mod_fwd_ms = graphed(fwd_only)
    mod.zero_grad(set_to_none=True)
    mod_step_ms = graphed(fwd_bwd)

    lib = _native.lib()
    dims = w.dims()
    wn, wd = w.coefficients()
    num = wn.repeat(w.groups, 1).to(dev).contiguous()
    den = wd.to(dev).contiguous()
    xs = x.detach()
    y, dx = torch.empty_like(xs), torch.empty_like(xs)
    dn = torch.empty(w.groups, 6, device=dev)
    dd = torch.empty(w.groups, 4, device=dev)
    need = ctypes.c_size_t(0)
    _native.check("ws", lib.kat_rational_bwd_workspace_size(*dims, w.groups, _native.KAT_DTYPE_F32,
                                                            dev.index, ctypes.byref(need)))
    ws = torch.empty(max(need.value, 16), dtype=torch.uint8, device=dev)
    sp = ctypes.c_void_p(stream.cuda_stream)
    fa = (xs.data_ptr(), y.data_ptr(), num.data_ptr(), den.data_ptr(), *dims, w.groups,
          _native.KAT_DTYPE_F32, sp)
    ba = (xs.data_ptr(), gy.data_ptr(), dx.data_ptr(), num.data_ptr(), den.data_ptr(),
          dn.data_ptr(), dd.data_ptr(), ws.data_ptr(), ws.numel(), *dims, w.groups,
          _native.KAT_DTYPE_F32, sp)
    out = []
    for fn, a in ((lib.kat_rational_fwd, fa), (lib.kat_rational_bwd, ba)):
        for _ in range(3):
            _native.check("launch", fn(*a))
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.kernel_iters):
            fn(*a)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        out.append(e0.elapsed_time(e1) / args.kernel_iters)
    k_fwd, k_bwd = out

    def gbs(nbytes, ms):
        return nbytes / (ms * 1e-3) / 1e9

    res = {
        "workload": w.name, "shape": list(w.shape), "num_groups": w.groups, "io_dtype": "f32",
        "coefficients": w.mode, "elements": N,
        "module_fwd_ms": mod_fwd_ms, "module_fwd_bwd_ms": mod_step_ms,
        "fwd_bwd_gelem_s": N / (mod_step_ms * 1e-3) / 1e9,
        "kernel_fwd_ms": k_fwd, "kernel_bwd_ms": k_bwd,
        "fwd_frac": gbs(2 * N * eb, k_fwd) / peak,
        "fwd_frac_spec": gbs(2 * N * eb, k_fwd) / SPEC_HBM_GBS,
        "bwd_frac": gbs(3 * N * eb, k_bwd) / peak,
        "bwd_frac_spec": gbs(3 * N * eb, k_bwd) / SPEC_HBM_GBS,
        "fwd_bwd_frac": gbs(5 * N * eb, mod_step_ms) / peak,
        "fwd_bwd_frac_spec": gbs(5 * N * eb, mod_step_ms) / SPEC_HBM_GBS,
        "timing": f"module steps in a CUDA graph, {reps} replays; C-ABI launches back to back, "
                  f"{args.kernel_iters} per direction; CUDA events",
    }
    del mod, x, gy, y, dx, ws
    torch.cuda.empty_cache()
    return res


def _gpu_bar(local, names):
    """The reference's own Triton kernels (rational_fwd_triton / rational_bwd_triton and the
    2D ones, from the reference installed under baseline/_ref) timed on this GPU at the given
    workloads, in a child process so their package cannot shadow this repository's import
    shims.  A throughput bar only: those kernels compute other denominator formulas."""
    ref = os.path.join(REPO, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "kat_rational")):
        return {"kind": "reference_triton", "unavailable": "reference not installed under "
                "baseline/_ref"}
    env = dict(os.environ, LOCAL_RANK=str(local))
    for k in ("RANK", "WORLD_SIZE", "MASTER_ADDR", "MASTER_PORT"):
        env.pop(k, None)
    try:
        res = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--gpu-bar-child",
                              ",".join(names)], env=env, capture_output=True, text=True,
                             timeout=900, cwd=os.path.dirname(REPO))
    except subprocess.TimeoutExpired:
        return {"kind": "reference_triton", "unavailable": "timed out after 900 s"}
    lines = [l for l in res.stdout.splitlines() if l.startswith("{")]
    if res.returncode != 0 or not lines:
        tail = (res.stderr or res.stdout).strip().splitlines()[-1:] or ["no output"]
        return {"kind": "reference_triton",
                "unavailable": f"child exited {res.returncode}: {tail[0][:300]}"}
    return json.loads(lines[-1])


def run_gpu_bar_child(names):
    """Child of _gpu_bar: imports the installed reference first on sys.path, then times its
    Triton launchers with CUDA events (3 warm-up calls, which include the JIT compile, then
    10 timed calls per direction)."""
    ref = os.path.join(REPO, "baseline", "_ref")
    sys.path[:] = [ref] + [p for p in sys.path
                           if p not in ("", ".") and os.path.abspath(p) != REPO] + [REPO]
    out = {"kind": "reference_triton",
           "source": "kat_rational.rational_triton.rational_fwd_triton / rational_bwd_triton and "
                     "rational_triton2d.rational_fwd_triton_2d / rational_bwd_triton_2d of the "
                     "reference installed under baseline/_ref",
           "formula_note": "throughput bar only: the reference's Triton forward uses "
                           "Q = 1 + |sum b_i x^i| and its backward Q = 1 + sum |b_i||x|^i, not the "
                           "PyTorch formula this repository implements; its backward adds 10 "
                           "float atomics per element"}
    try:
        import kat_rational.rational_triton as rt
        import kat_rational.rational_triton2d as rt2
        import triton
        if not os.path.abspath(rt.__file__).startswith(os.path.abspath(ref)):
            raise ImportError(f"kat_rational resolved to {rt.__file__}")
        out["triton"] = triton.__version__
    except Exception as e:
        out["unavailable"] = f"import failed: {type(e).__name__}: {e}"
        print(json.dumps(out), flush=True)
        return
    from rational_kat_cu_b200 import workloads

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev)
    peak, _ = measured_peak()
    for name in names:
        w = workloads.get(name)
        eb = {"f32": 4, "bf16": 2, "f16": 2}[w.dtype]
        x, gy = w.inputs(dev)
        wn, wd = w.coefficients()
        n = wn.repeat(w.groups, 1).to(dev).contiguous()
        d = wd.to(dev).contiguous()
        if w.layout == "nchw":
            fwd = lambda: rt2.rational_fwd_triton_2d(x, n, d, w.groups)  # noqa: E731
            bwd = lambda: rt2.rational_bwd_triton_2d(gy, x, n, d, w.groups)  # noqa: E731
        else:
            fwd = lambda: rt.rational_fwd_triton(x, n, d, w.groups)  # noqa: E731
            bwd = lambda: rt.rational_bwd_triton(gy, x, n, d, w.groups)  # noqa: E731
        entry = {"shape": list(w.shape), "io_dtype": w.dtype, "num_groups": w.groups}
        for label, fn, nbytes in (("fwd", fwd, 2 * w.numel * eb), ("bwd", bwd, 3 * w.numel * eb)):
            try:
                for _ in range(3):
                    fn()
                torch.cuda.synchronize(dev)
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                for _ in range(10):
                    fn()
                b.record(stream)
                torch.cuda.synchronize(dev)
                ms = a.elapsed_time(b) / 10
                entry[f"{label}_ms"] = ms
                entry[f"{label}_frac"] = nbytes / (ms * 1e-3) / 1e9 / peak
            except Exception as e:
                entry[f"{label}_unavailable"] = f"{type(e).__name__}: {str(e)[:300]}"
        if "fwd_ms" in entry and "bwd_ms" in entry:
            entry["fwd_bwd_gelem_s"] = w.numel / ((entry["fwd_ms"] + entry["bwd_ms"]) * 1e-3) / 1e9
        out[name] = entry
        del x, gy, n, d
        torch.cuda.empty_cache()
    print(json.dumps(out), flush=True)


def run_sweep(args):
    """Bandwidth sweep on one GPU: per point, C-ABI forward and backward launches on
    device-resident inputs, `iters` of each captured in a CUDA graph and timed with CUDA events
    around one replay; one JSON line per point."""
    import ctypes

    from rational_kat_cu_b200 import _native, workloads

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    lib = _native.lib()
    peak, peak_kind = measured_peak()
    stream = torch.cuda.current_stream(dev)
    sp = ctypes.c_void_p(stream.cuda_stream)
    keep = {int(v) for v in args.sweep_logn.split(",") if v.strip()}
    for c, g, n, dt in workloads.sweep_points():
        if keep and n.bit_length() - 1 not in keep:
            continue
        w = workloads.sweep(c, g, n, dt)
        N = w.numel
        eb = {"f32": 4, "bf16": 2, "f16": 2}[dt]
        code = {"f32": 0, "f16": 1, "bf16": 2}[dt]
        x, gy = w.inputs(dev)
        wn, wd = w.coefficients()
        num = wn.repeat(g, 1).to(dev).contiguous()
        den = wd.to(dev).contiguous()
        y = torch.empty_like(x)
        dx = torch.empty_like(x)
        dn = torch.empty(g, 6, device=dev)
        dd = torch.empty(g, 4, device=dev)
        dims = w.dims()
        need = ctypes.c_size_t(0)
        _native.check("ws", lib.kat_rational_bwd_workspace_size(dims[0], dims[1], dims[2], g,
                                                                code, dev.index,
                                                                ctypes.byref(need)))
        ws = torch.empty(max(need.value, 16), dtype=torch.uint8, device=dev)
        fa = (x.data_ptr(), y.data_ptr(), num.data_ptr(), den.data_ptr(), *dims, g, code, sp)
        ba = (x.data_ptr(), gy.data_ptr(), dx.data_ptr(), num.data_ptr(), den.data_ptr(),
              dn.data_ptr(), dd.data_ptr(), ws.data_ptr(), ws.numel(), *dims, g, code, sp)
        iters = max(3, min(200, int(2e10 / (N * eb * 5))))

        def timed(fn, a):
            # `iters` launches captured in a CUDA graph and replayed: device time per launch
            # without the host's per-call cost.
            for _ in range(2):
                _native.check("launch", fn(*a))
            torch.cuda.synchronize(dev)
            cap = torch.cuda.Stream(dev)
            graph = torch.cuda.CUDAGraph()
            ca = a[:-1] + (ctypes.c_void_p(cap.cuda_stream),)
            cap.wait_stream(stream)
            with torch.cuda.stream(cap):
                graph.capture_begin()
                for _ in range(iters):
                    fn(*ca)
                graph.capture_end()
            torch.cuda.synchronize(dev)
            graph.replay()
            torch.cuda.synchronize(dev)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            graph.replay()
            e1.record(stream)
            torch.cuda.synchronize(dev)
            del graph
            return e0.elapsed_time(e1) / iters

        f_ms = timed(lib.kat_rational_fwd, fa)
        b_ms = timed(lib.kat_rational_bwd, ba)
        line = {
            "metric": "KAT_Group sweep", "workload": w.name, "channels": c, "num_groups": g,
            "elements": N, "dtype": dt, "iters": iters,
            "fwd_ms": f_ms, "bwd_ms": b_ms,
            "fwd_gelem_s": N / f_ms / 1e6, "fwd_bwd_gelem_s": N / (f_ms + b_ms) / 1e6,
            "fwd_hbm_frac": 2 * N * eb / f_ms / 1e6 / peak,
            "bwd_hbm_frac": 3 * N * eb / b_ms / 1e6 / peak,
            "fwd_bwd_hbm_frac": 5 * N * eb / (f_ms + b_ms) / 1e6 / peak,
            "peak_gbs": peak, "peak_source": peak_kind,
            "l2": "larger than L2" if N * eb > L2_BYTES else "fits in L2 (inputs reused across launches)",
        }
        print(json.dumps(line), flush=True)
        del x, gy, y, dx, ws
        torch.cuda.empty_cache()


# ---------------------------------------------------------------------------
# GR-KAN ViT-B/16 data-parallel training step (--workload grkan_vit_b16)
# ---------------------------------------------------------------------------

VIT_WORKLOAD = "grkan_vit_b16"
VIT_METRIC = "GR-KAN ViT-B/16 training images/s"
VIT_UNIT = "images/s"


def _time_steps(step, steps, warmup, dev, stream, dist=None):
    """Average device time of one `step` over `steps` timed calls after `warmup` untimed ones
    (CUDA events on `stream`, barrier + synchronize on both sides, max over ranks)."""
    for _ in range(warmup):
        step()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(steps):
        step()
    b.record(stream)
    torch.cuda.synchronize(dev)
    if dist is not None:
        dist.barrier()
    ms = a.elapsed_time(b)
    if dist is not None:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms / steps


def _kat_kernel_ms(dev, stream, shape, mode, groups, iters):
    """C-ABI forward and backward launch times (ms) of one KAT_Group at `shape` (bf16,
    `mode` coefficients), back-to-back on device-resident buffers."""
    import ctypes

    from rational_kat_cu_b200 import _native
    from rational_kat_cu_b200._init_table import load_table

    lib = _native.lib()
    code = _native.KAT_DTYPE_BF16
    C = shape[-1]
    rows = 1
    for d in shape[:-1]:
        rows *= d
    g = torch.Generator(device=dev).manual_seed(11)
    x = torch.randn(shape, generator=g, device=dev).to(torch.bfloat16)
    gy = torch.randn(shape, generator=g, device=dev).to(torch.bfloat16)
    table = load_table()[mode]
    num = torch.tensor(table["init_w_numerator"], device=dev).view(1, 6).repeat(groups, 1)
    den = torch.tensor(table["init_w_denominator"], device=dev).view(1, 4).repeat(groups, 1)
    y, dx = torch.empty_like(x), torch.empty_like(x)
    dn = torch.empty(groups, 6, device=dev)
    dd = torch.empty(groups, 4, device=dev)
    need = ctypes.c_size_t(0)
    _native.check("ws", lib.kat_rational_bwd_workspace_size(rows, C, 1, groups, code, dev.index,
                                                            ctypes.byref(need)))
    ws = torch.empty(max(need.value, 16), dtype=torch.uint8, device=dev)
    sp = ctypes.c_void_p(stream.cuda_stream)
    fa = (x.data_ptr(), y.data_ptr(), num.data_ptr(), den.data_ptr(), rows, C, 1, groups, code, sp)
    ba = (x.data_ptr(), gy.data_ptr(), dx.data_ptr(), num.data_ptr(), den.data_ptr(),
          dn.data_ptr(), dd.data_ptr(), ws.data_ptr(), ws.numel(), rows, C, 1, groups, code, sp)
    out = []
    for fn, a in ((lib.kat_rational_fwd, fa), (lib.kat_rational_bwd, ba)):
        for _ in range(3):
            _native.check("launch", fn(*a))
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(iters):
            fn(*a)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        out.append(e0.elapsed_time(e1) / iters)
    return out[0], out[1], x.numel()


def _vit_cpu_rate(budget_s: float, steps: int = 0, warmup: int = 0):
    """The reference's CPU path for the ViT step: the same GR-KAN ViT-B/16, fp32 on the host
    cores, its KAT activations evaluated by the oracle's restatement of kat_1dgroup_torch.py,
    on a bounded batch.  Returns (images/s, info)."""
    from oracle import kat_torch_oracle
    from rational_kat_cu_b200 import grkan_vit as gv

    torch.set_num_threads(os.cpu_count() or 1)
    cores = torch.get_num_threads()
    cfg = gv.vit_b16()
    torch.manual_seed(0)
    model = gv.GRKANViT(cfg, kat_device="cpu")
    for m in model.kat_modules():
        m.rational = kat_torch_oracle.rational_1dgroup
    opt = gv.make_optimizer(model)

    def run(batch, n):
        images, labels = gv.synthetic_batch(batch, cfg, dtype=torch.float32, seed=0)
        t0 = time.perf_counter()
        for _ in range(n):
            gv.train_step(model, opt, images, labels)
        return (time.perf_counter() - t0) / max(n, 1)

    per_image = run(1, 1)
    n_calls = (steps + warmup) if steps else 2
    batch = int(max(1, min(32, budget_s / max(n_calls, 1) / per_image)))
    run(batch, warmup if steps else 1)
    reps = steps if steps else 1
    dt = run(batch, reps)
    return batch / dt, {
        "cores": cores, "batch": batch, "seconds_per_step": dt, "reps": reps,
        "sample": f"GR-KAN ViT-B/16 training step (AdamW) at batch {batch}, fp32 on the host "
                  f"cores, KAT activations by the oracle's kat_1dgroup_torch restatement, mean "
                  f"of {reps} timed steps"}


def run_vit_reference(args):
    world, rank, local = dist_setup()
    if rank != 0:
        return
    rate, info = _vit_cpu_rate(budget_s=min(150.0, 20.0 + 2.0 * (args.steps + args.warmup)),
                               steps=min(args.steps, 3), warmup=min(args.warmup, 1))
    line = {
        "metric": VIT_METRIC, "value": rate, "unit": VIT_UNIT, "n_gpus": args.gpus,
        "steps": min(args.steps, 3), "warmup": min(args.warmup, 1),
        "ms_per_step": info["seconds_per_step"] * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "impl": "reference",
        "config": {"workload": VIT_WORKLOAD, "model": "GR-KAN ViT-B/16", "image": 224,
                   "sample_batch": info["batch"]},
        "cpu_baseline": {"value": rate, "unit": VIT_UNIT, "cores": info["cores"], "kind": "port",
                         "sample": info["sample"]},
        "e2e": {"value": rate, "unit": VIT_UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_vit(args):
    """One data-parallel training step of GR-KAN ViT-B/16 (bf16 parameters and activations,
    AdamW) per timed iteration, `--vit-batch` synthetic 224x224 images per GPU."""
    import dataclasses

    from rational_kat_cu_b200 import grkan_vit as gv

    world, rank, local = dist_setup()
    dist = init_process_group(world, rank, local) if world > 1 else None
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev)
    cfg = gv.vit_b16()
    B = args.vit_batch

    def build(act="kat", kat_device="cuda", fused_gemm=args.vit_fused_gemm):
        torch.manual_seed(0)
        return gv.GRKANViT(dataclasses.replace(cfg, act=act, fused_gemm=fused_gemm),
                           kat_device=kat_device).to(dev, dtype=torch.bfloat16)

    graphed = dist is None and not args.vit_eager
    model = build()
    net = model
    if dist is not None:
        net = gv.wrap_data_parallel(model, args.kat_exchange, device_ids=[local],
                                    timeout_ms=20000, gradient_as_bucket_view=True)
    opt = gv.make_optimizer(model, capturable=graphed)
    h_img, h_lab = gv.synthetic_batch(B, cfg, dtype=torch.bfloat16, seed=rank, device=dev)
    d_img, d_lab = h_img.to(dev), h_lab.to(dev)

    def make_step(m, o):
        """One training step: the captured graph (one GPU) or an eager step."""
        if graphed:
            g = gv.GraphedTrainStep(m, o, d_img, d_lab)
            return g, (lambda img=None, lab=None: g(img, lab))
        return None, (lambda img=d_img, lab=d_lab: gv.train_step(m, o, img, lab))

    graph_obj, step = make_step(net, opt)
    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
    ms = _time_steps(lambda: step(), args.steps, args.warmup, dev, stream, dist)
    value = world * B / (ms * 1e-3)

    # End to end: every step uploads its images and labels from pinned host memory and
    # reads the loss back into pinned host memory.
    h_loss = torch.empty((), dtype=torch.float32, pin_memory=True)

    def e2e_step():
        img = h_img.to(dev, non_blocking=True)
        lab = h_lab.to(dev, non_blocking=True)
        h_loss.copy_(step(img, lab), non_blocking=True)

    e2e_ms = _time_steps(e2e_step, args.e2e_steps, 2, dev, stream, dist)
    loss_value = float(h_loss.item())
    clocks = None
    if sampler:
        sampler.stop()
        clocks = sampler.summary()

    # KAT kernels at the model's shapes (standalone C-ABI timings): 12 x act1 [B,197,768]
    # 'identity' + 12 x act2 [B,197,3072] 'gelu', forward + backward.
    f1, b1, n1 = _kat_kernel_ms(dev, stream, (B, cfg.num_tokens, cfg.embed_dim), "identity",
                                cfg.num_groups, args.kernel_iters // 4 or 1)
    f2, b2, n2 = _kat_kernel_ms(dev, stream, (B, cfg.num_tokens, 4 * cfg.embed_dim), "gelu",
                                cfg.num_groups, args.kernel_iters // 4 or 1)
    kat_ms = cfg.depth * (f1 + b1 + f2 + b2)
    bwd2_names = bwd_kernel_names()
    launches_per_step = cfg.depth * 2 * (1 + bwd2_names.count("+") + 1)
    peak, peak_kind = measured_peak()
    bwd_gbs = 3 * n2 * 2 / (b2 * 1e-3) / 1e9

    compare = None
    if args.vit_compare and world == 1:
        compare = {}
        del opt, graph_obj, step
        torch.cuda.empty_cache()
        other = ("kat_unfused", dict(fused_gemm=False)) if args.vit_fused_gemm else \
            ("kat_fused_gemm", dict(fused_gemm=True))
        for name, kw in (other, ("kat_torch_formulation", dict(kat_device="cpu", fused_gemm=False)),
                         ("gelu_mlp", dict(act="gelu"))):
            m2 = build(**kw)
            o2 = gv.make_optimizer(m2, capturable=graphed)
            g2, step2 = make_step(m2, o2)
            steps2 = max(5, min(args.steps, 30))
            ms2 = _time_steps(lambda: step2(), steps2, 3, dev, stream)
            compare[name] = {"ms_per_step": ms2, "images_s": B / (ms2 * 1e-3), "steps": steps2}
            del m2, o2, g2, step2
            torch.cuda.empty_cache()
        compare["kat_torch_formulation"]["what"] = (
            "KAT_Group on the reference's PyTorch formulation (power stack + bmm, "
            "kat_1dgroup_torch.py) on the GPU, everything else identical")
        compare["gelu_mlp"]["what"] = "plain ViT-B/16 MLP (fc1 -> GELU -> fc2), no KAT"
        compare[other[0]]["what"] = (
            "KAN blocks on torch linears + KAT_Group kernels" if args.vit_fused_gemm else
            "KAN blocks' fc1 -> act2 -> fc2 on the tcgen05 GEMMs with act2 in their epilogues")

    cpu = None
    if rank == 0 and world == 1 and not args.skip_cpu_baseline:
        rate, info = _vit_cpu_rate(budget_s=args.cpu_seconds)
        cpu = {"value": rate, "unit": VIT_UNIT, "cores": info["cores"], "kind": "port",
               "sample": info["sample"]}

    if dist is not None:
        dist.barrier()
    if rank == 0:
        line = {
            "metric": VIT_METRIC, "value": value, "unit": VIT_UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic",
            "config": {
                "workload": VIT_WORKLOAD,
                "model": "GR-KAN ViT-B/16 (12 layers, d=768, MLP 3072, 12 heads, KAT_Group "
                         "act1 'identity' / act2 'gelu', 8 groups)",
                "global_batch": B * world, "per_gpu_batch": B, "image": [3, 224, 224],
                "seq_len": cfg.num_tokens, "parallelism": f"dp{world}",
                "kat_exchange": args.kat_exchange if world > 1 else None,
                "fused_gemm": bool(args.vit_fused_gemm),
                "optimizer": "AdamW (fused)", "params": "bf16",
                "step": ("forward + loss + backward + optimizer captured in one CUDA graph"
                         if graphed else "eager" + (" with DistributedDataParallel over NCCL"
                                                    if dist is not None else "")),
                "l2": "activations of one step are far larger than L2 (no flush needed)",
                "loss_last_step": loss_value,
            },
            "roofline": {
                "bound": "hbm", "kernel": "KAT act2 backward call [B,197,3072] bf16: "
                                          + bwd2_names,
                "achieved": bwd_gbs, "peak": peak, "unit": "GB/s", "frac": bwd_gbs / peak,
                "peak_source": f"{peak_kind} hbm_gbs", "traffic": None,
                "algorithmic_bytes_per_launch": 3 * n2 * 2, "ms_per_launch": b2,
            },
            "kat": {
                "act1_fwd_ms": f1, "act1_bwd_ms": b1, "act2_fwd_ms": f2, "act2_bwd_ms": b2,
                "kat_ms_per_step": kat_ms, "kat_share_of_step": kat_ms / ms,
                "note": "standalone C-ABI timings at the model's shapes, times 12 blocks",
            },
            "compare": compare,
            "e2e": {"value": world * B / (e2e_ms * 1e-3), "unit": VIT_UNIT,
                    "h2d_bytes_per_step": world * (h_img.numel() * 2 + h_lab.numel() * 8),
                    "d2h_bytes_per_step": world * 4, "ms_per_step": e2e_ms,
                    "api": "grkan_vit.train_step on pinned host images/labels (H2D per step), "
                           "loss read back to pinned host"},
            "gpu_launches": launches_per_step * args.steps * world,
            "cpu_baseline": cpu,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        for m in model.kat_modules():
            if getattr(m, "exchange", None) is not None:
                m.exchange.close()
        dist.barrier()
        dist.destroy_process_group()


# ---------------------------------------------------------------------------
# B-spline basis (--workload bspline_kan): the fused Cox-de Boor basis of a KAN layer
# ---------------------------------------------------------------------------

BSPLINE_WORKLOAD = "bspline_kan"
BSPLINE_METRIC = "B-spline basis fwd+bwd Gelem/s"
BSPLINE_SHAPE = (16384, 1024, 8, 3)   # batch, in_features, grid_size, spline_order


def _bspline_inputs(B, D, gs, order, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, D, generator=g) * 0.6
    gb = torch.randn(B, D, gs + order, generator=g)
    return x, gb


def _bspline_grid(D, gs, order):
    from rational_kat_cu_b200.bspline import FusedKANLinear

    return FusedKANLinear(D, 1, grid_size=gs, spline_order=order).grid


def _bspline_cpu_rate(budget_s: float, steps: int = 0, warmup: int = 0):
    from oracle import bspline_oracle as bs

    torch.set_num_threads(os.cpu_count() or 1)
    B, D, gs, order = BSPLINE_SHAPE
    grid = _bspline_grid(D, gs, order)

    def run(rows, n):
        x, gb = _bspline_inputs(rows, D, gs, order)
        t0 = time.perf_counter()
        for _ in range(n):
            bs.b_splines_fwd_bwd(x, grid, order, gb)
        return (time.perf_counter() - t0) / max(n, 1)

    per_row = run(8, 1) / 8
    n_calls = (steps + warmup) if steps else 3
    rows = int(max(1, min(B, budget_s / max(n_calls, 1) / per_row)))
    run(rows, warmup if steps else 1)
    reps = steps if steps else 2
    dt = run(rows, reps)
    return rows * D / dt / 1e9, {
        "cores": torch.get_num_threads(), "rows": rows, "seconds_per_step": dt, "reps": reps,
        "sample": f"x[{rows},{D}], grid_size {gs}, order {order}: the reference's PyTorch "
                  f"Cox-de Boor (oracle restatement) forward + autograd backward, fp32, mean of "
                  f"{reps} timed steps"}


def run_bspline_reference(args):
    world, rank, local = dist_setup()
    if rank != 0:
        return
    steps, warmup = min(args.steps, 5), min(args.warmup, 1)
    rate, info = _bspline_cpu_rate(budget_s=min(150.0, 20.0 + 2.0 * (steps + warmup)),
                                   steps=steps, warmup=warmup)
    print(json.dumps({
        "metric": BSPLINE_METRIC, "value": rate, "unit": UNIT, "n_gpus": args.gpus,
        "steps": steps, "warmup": warmup, "ms_per_step": info["seconds_per_step"] * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "impl": "reference",
        "config": {"workload": BSPLINE_WORKLOAD, "shape": list(BSPLINE_SHAPE[:2]),
                   "grid_size": BSPLINE_SHAPE[2], "spline_order": BSPLINE_SHAPE[3],
                   "sample_rows": info["rows"]},
        "cpu_baseline": {"value": rate, "unit": UNIT, "cores": info["cores"], "kind": "port",
                         "sample": info["sample"]},
        "e2e": {"value": rate, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def run_bspline(args):
    """Step = basis forward + backward C-ABI launches on x [16384, 1024] fp32 (grid_size 8,
    order 3: 11 basis values per element), inputs resident; e2e adds the host copies."""
    import ctypes

    from rational_kat_cu_b200 import _native

    world, rank, local = dist_setup()
    dist = init_process_group(world, rank, local) if world > 1 else None
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev)
    B, D, gs, order = BSPLINE_SHAPE
    nb = gs + order
    nk = gs + 2 * order + 1
    x_h, gb_h = _bspline_inputs(B, D, gs, order, seed=rank)
    grid = _bspline_grid(D, gs, order).to(dev)
    x, gb = x_h.to(dev), gb_h.to(dev)
    bases = torch.empty(B, D, nb, device=dev)
    dx = torch.empty(B, D, device=dev)
    lib = _native.lib()
    sp = ctypes.c_void_p(stream.cuda_stream)
    fa = (x.data_ptr(), grid.data_ptr(), bases.data_ptr(), B, D, nk, order, sp)
    ba = (x.data_ptr(), grid.data_ptr(), gb.data_ptr(), dx.data_ptr(), B, D, nk, order, sp)

    def step():
        _native.check("fwd", lib.kat_bspline_basis_fwd(*fa))
        _native.check("bwd", lib.kat_bspline_basis_bwd(*ba))

    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
    ms = _time_steps(step, args.steps, args.warmup, dev, stream, dist)
    iters = args.kernel_iters

    def per_launch(fn, a):
        for _ in range(3):
            fn(*a)
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(iters):
            fn(*a)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) / iters

    f_ms = per_launch(lib.kat_bspline_basis_fwd, fa)
    b_ms = per_launch(lib.kat_bspline_basis_bwd, ba)
    # e2e: pinned host x and grad_bases in, bases and dx back, every step
    hx, hgb = x_h.pin_memory(), gb_h.pin_memory()
    hb = torch.empty(B, D, nb, pin_memory=True)
    hdx = torch.empty(B, D, pin_memory=True)

    def e2e_step():
        x.copy_(hx, non_blocking=True)
        gb.copy_(hgb, non_blocking=True)
        step()
        hb.copy_(bases, non_blocking=True)
        hdx.copy_(dx, non_blocking=True)

    e_ms = _time_steps(e2e_step, max(2, args.e2e_steps // 2), 1, dev, stream, dist)
    clocks = None
    if sampler:
        sampler.stop()
        clocks = sampler.summary()
    cpu = None
    if rank == 0 and world == 1 and not args.skip_cpu_baseline:
        rate, info = _bspline_cpu_rate(budget_s=args.cpu_seconds)
        cpu = {"value": rate, "unit": UNIT, "cores": info["cores"], "kind": "port",
               "sample": info["sample"]}
    if dist is not None:
        dist.barrier()
    if rank == 0:
        N = B * D
        peak, peak_kind = measured_peak()
        fwd_bytes, bwd_bytes = N * 4 * (1 + nb), N * 4 * (2 + nb)
        print(json.dumps({
            "metric": BSPLINE_METRIC, "value": world * N / (ms * 1e-3) / 1e9, "unit": UNIT,
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": BSPLINE_WORKLOAD, "shape": [B, D], "grid_size": gs,
                       "spline_order": order, "n_basis": nb,
                       "l2": f"bases {N * nb * 4 / 1e6:.0f} MB per step, larger than L2"},
            "roofline": {"bound": "hbm", "kernel": "kat_bspline_fwd_kernel<3>",
                         "achieved": fwd_bytes / (f_ms * 1e-3) / 1e9, "peak": peak,
                         "unit": "GB/s", "frac": fwd_bytes / (f_ms * 1e-3) / 1e9 / peak,
                         "peak_source": f"{peak_kind} hbm_gbs", "traffic": None,
                         "algorithmic_bytes_per_launch": fwd_bytes, "ms_per_launch": f_ms},
            "kernels": {"fwd_ms": f_ms, "bwd_ms": b_ms,
                        "fwd_frac": fwd_bytes / (f_ms * 1e-3) / 1e9 / peak,
                        "bwd_frac": bwd_bytes / (b_ms * 1e-3) / 1e9 / peak,
                        "step_hbm_frac": (fwd_bytes + bwd_bytes) / (ms * 1e-3) / 1e9 / peak},
            "e2e": {"value": world * N / (e_ms * 1e-3) / 1e9, "unit": UNIT,
                    "h2d_bytes_per_step": world * N * 4 * (1 + nb),
                    "d2h_bytes_per_step": world * N * 4 * (1 + nb), "ms_per_step": e_ms,
                    "api": "C ABI kat_bspline_basis_fwd/_bwd with pinned host copies"},
            "gpu_launches": 2 * args.steps * world,
            "cpu_baseline": cpu, "clocks": clocks,
        }), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


KAN_WORKLOAD = "kan_mlp_b16"
KAN_METRIC = "GR-KAN MLP block (fc1 -> act2 -> fc2) fwd+bwd tokens/s"
KAN_UNIT = "Mtokens/s"


def _kan_block(C, H, G, dev, seed=0):
    from rational_kat_cu_b200 import KAT_Group

    torch.manual_seed(seed)
    fc1 = torch.nn.Linear(C, H).to(dev, torch.bfloat16)
    act2 = KAT_Group(num_groups=G, mode="gelu").to(dev)
    fc2 = torch.nn.Linear(H, C).to(dev, torch.bfloat16)
    return fc1, act2, fc2


def _kan_cpu_rate(budget_s: float, steps: int = 0, warmup: int = 0):
    """The reference's CPU path for the block: fp32 torch linears on the host cores with act2
    evaluated by the oracle's restatement of kat_1dgroup_torch.py, forward + backward, on a
    bounded number of tokens.  Returns (Mtokens/s, info)."""
    from oracle import kat_torch_oracle

    torch.set_num_threads(os.cpu_count() or 1)
    cores = torch.get_num_threads()
    C, H, G = 768, 3072, 8
    torch.manual_seed(0)
    fc1 = torch.nn.Linear(C, H)
    fc2 = torch.nn.Linear(H, C)
    from rational_kat_cu_b200 import KAT_Group
    act = KAT_Group(num_groups=G, mode="gelu", device="cpu")
    wn = act.weight_numerator.detach().clone().requires_grad_(True)
    wd = act.weight_denominator.detach().clone().requires_grad_(True)

    def run(tokens, n):
        x = torch.randn(1, tokens, C, requires_grad=True)
        gy = torch.randn(1, tokens, C)
        t0 = time.perf_counter()
        for _ in range(n):
            h = fc1(x)
            y = kat_torch_oracle.rational_1dgroup(h, wn.repeat(G, 1), wd, G)
            fc2(y).backward(gy)
        return (time.perf_counter() - t0) / max(n, 1)

    per_token = run(197, 1) / 197
    n_calls = (steps + warmup) if steps else 2
    tokens = int(max(197, min(197 * 32, budget_s / max(n_calls, 1) / per_token)))
    run(tokens, warmup if steps else 1)
    reps = steps if steps else 1
    dt = run(tokens, reps)
    return tokens / dt / 1e6, {
        "cores": cores, "tokens": tokens, "seconds_per_step": dt, "reps": reps,
        "sample": f"fc1 -> act2 -> fc2 forward + backward on {tokens} tokens (768 -> 3072 -> "
                  f"768), fp32 on the host cores, act2 by the oracle's kat_1dgroup_torch "
                  f"restatement, mean of {reps} timed steps"}


def run_kan_mlp_reference(args):
    world, rank, _ = dist_setup()
    if rank != 0:
        return
    steps = max(1, min(args.steps, 3))
    warm = max(0, min(args.warmup, 1))
    rate, info = _kan_cpu_rate(args.cpu_seconds, steps=steps, warmup=warm)
    print(json.dumps({
        "impl": "reference", "metric": KAN_METRIC, "value": rate, "unit": KAN_UNIT,
        "n_gpus": args.gpus, "steps": steps, "warmup": warm, "ms_per_step": info["seconds_per_step"] * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": {"workload": KAN_WORKLOAD, "tokens": info["tokens"]},
        "cpu_baseline": {"value": rate, "unit": KAN_UNIT, "cores": info["cores"], "kind": "port",
                         "sample": info["sample"]},
        "e2e": {"value": rate, "unit": KAN_UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def run_kan_mlp(args):
    """Step = the GR-KAN ViT-B/16 MLP block fc1 (768 -> 3072) -> act2 (KAT 'gelu', 8 groups)
    -> fc2 (3072 -> 768), forward + backward, on --vit-batch x 197 tokens of bf16, through
    fused_gemm.kan_mlp_fused (act2 in the tcgen05 GEMM epilogues), captured in a CUDA graph.
    The same block on cuBLAS linears + the activation kernels is timed beside it."""
    import ctypes

    from rational_kat_cu_b200 import fused_gemm

    world, rank, local = dist_setup()
    dist = init_process_group(world, rank, local) if world > 1 else None
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev)
    C, H, G = 768, 3072, 8
    M = args.vit_batch * 197
    fc1, act2, fc2 = _kan_block(C, H, G, dev)
    g = torch.Generator().manual_seed(rank)
    x_h = torch.randn(M, C, generator=g).to(torch.bfloat16)
    gy_h = (torch.randn(M, C, generator=g) * 0.05).to(torch.bfloat16)
    x = x_h.to(dev).requires_grad_(True)
    gy = gy_h.to(dev)
    params = [*fc1.parameters(), *act2.parameters(), *fc2.parameters()]

    def fused_step():
        fused_gemm.kan_mlp_fused(x, fc1, act2, fc2).backward(gy)

    def unfused_step():
        fc2(act2(fc1(x))).backward(gy)

    def graphed(fn):
        for p in params + [x]:
            p.grad = None
        side = torch.cuda.Stream(dev)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            for _ in range(2):
                fn()
        stream.wait_stream(side)
        for p in params + [x]:
            p.grad = None
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            fn()
        return gr

    g_fused = graphed(fused_step)
    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
    ms = _time_steps(g_fused.replay, args.steps, args.warmup, dev, stream, dist)
    g_unfused = graphed(unfused_step)
    ms_unfused = _time_steps(g_unfused.replay, args.steps, args.warmup, dev, stream, dist)
    del g_unfused

    # the two fused kernels alone (C ABI through fused_gemm), graph-captured
    num = act2.weight_numerator.detach().repeat(G, 1).contiguous()
    den = act2.weight_denominator.detach().contiguous()
    xd = x.detach()
    w2t = fc2.weight.detach().t().contiguous()
    h, _ = fused_gemm.gemm_rational_fwd(xd, fc1.weight, fc1.bias, num, den, G)

    def kernel_ms(fn):
        gr = torch.cuda.CUDAGraph()
        fn()
        with torch.cuda.graph(gr):
            fn()
        return _time_steps(gr.replay, max(5, args.kernel_iters // 4), 3, dev, stream)

    f_ms = kernel_ms(lambda: fused_gemm.gemm_rational_fwd(xd, fc1.weight, fc1.bias, num, den, G))
    b_ms = kernel_ms(lambda: fused_gemm.gemm_rational_bwd(gy, w2t, h, num, den, G))
    p_ms = kernel_ms(lambda: fused_gemm.gemm_bf16(xd, fc1.weight, fc1.bias))
    c_ms = kernel_ms(lambda: torch.nn.functional.linear(xd, fc1.weight, fc1.bias))

    # e2e through the module API: x and the output gradient uploaded from pinned host memory,
    # dx read back into pinned host memory, every step (eager)
    hx, hgy = x_h.pin_memory(), gy_h.pin_memory()
    hdx = torch.empty(M, C, dtype=torch.bfloat16, pin_memory=True)

    def e2e_step():
        xi = hx.to(dev, non_blocking=True).requires_grad_(True)
        fused_gemm.kan_mlp_fused(xi, fc1, act2, fc2).backward(hgy.to(dev, non_blocking=True))
        hdx.copy_(xi.grad, non_blocking=True)

    e_ms = _time_steps(e2e_step, max(3, args.e2e_steps), 2, dev, stream, dist)
    status = fused_gemm.device_status(local)
    clocks = None
    if sampler:
        sampler.stop()
        clocks = sampler.summary()
    cpu = None
    if rank == 0 and world == 1 and not args.skip_cpu_baseline:
        rate, info = _kan_cpu_rate(budget_s=args.cpu_seconds)
        cpu = {"value": rate, "unit": KAN_UNIT, "cores": info["cores"], "kind": "port",
               "sample": info["sample"]}
    if dist is not None:
        dist.barrier()
    if rank == 0:
        flops_gemm = 2.0 * M * H * C
        peak_tf = _bf16_peak()
        print(json.dumps({
            "metric": KAN_METRIC, "value": world * M / (ms * 1e-3) / 1e6, "unit": KAN_UNIT,
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": KAN_WORKLOAD, "tokens_per_gpu": M, "in_features": C,
                       "hidden": H, "groups": G, "step": "forward + backward in one CUDA graph",
                       "l2": "activations of one step (155 MB per [tokens, 3072] tensor) exceed L2"},
            "roofline": {"bound": "tensor", "kernel": "kat_gemm_kernel<1, 0> (fc1 + act2 forward)",
                         "achieved": flops_gemm / (f_ms * 1e-3) / 1e12, "peak": peak_tf[0],
                         "unit": "TFLOP/s", "frac": flops_gemm / (f_ms * 1e-3) / 1e12 / peak_tf[0],
                         "peak_source": peak_tf[1],
                         "traffic": 120_227_584 + 259_228_672,
                         "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of "
                                           "one kat_gemm_kernel<1, 0, 1> launch at this shape, "
                                           "profiles/kat_gemm_kernel_kan_mlp_b16.md",
                         "algorithmic_flops_per_launch": flops_gemm, "ms_per_launch": f_ms},
            "kernels": {"fused_fwd_ms": f_ms, "fused_bwd_ms": b_ms, "plain_gemm_ms": p_ms,
                        "cublas_fc1_ms": c_ms,
                        "plain_gemm_tflops": flops_gemm / (p_ms * 1e-3) / 1e12,
                        "cublas_fc1_tflops": flops_gemm / (c_ms * 1e-3) / 1e12},
            "compare": {"unfused_ms_per_step": ms_unfused,
                        "unfused_value": world * M / (ms_unfused * 1e-3) / 1e6,
                        "what": "same block on torch linears (cuBLAS) + KAT_Group kernels"},
            "e2e": {"value": world * M / (e_ms * 1e-3) / 1e6, "unit": KAN_UNIT,
                    "h2d_bytes_per_step": world * M * C * 2 * 2,
                    "d2h_bytes_per_step": world * M * C * 2, "ms_per_step": e_ms,
                    "api": "fused_gemm.kan_mlp_fused forward + backward, pinned host x / grad in, "
                           "dx out"},
            "gpu_launches": 4 * args.steps * world,
            "device_status": status,
            "cpu_baseline": cpu, "clocks": clocks,
        }), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def _bf16_peak():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as fh:
            return float(json.load(fh)["bf16_tflops"]), "measured bf16_tflops (burst)"
    except Exception:
        return 1590.0, "fallback bf16 TFLOP/s (burst)"


def main():
    args = parse_args()
    if args.gpu_bar_child:
        run_gpu_bar_child(args.gpu_bar_child.split(","))
        return
    if args.workload == BSPLINE_WORKLOAD:
        if args.impl == "reference":
            run_bspline_reference(args)
        else:
            run_bspline(args)
    elif args.workload == VIT_WORKLOAD:
        if args.impl == "reference":
            run_vit_reference(args)
        else:
            run_vit(args)
    elif args.workload == KAN_WORKLOAD:
        if args.impl == "reference":
            run_kan_mlp_reference(args)
        else:
            run_kan_mlp(args)
    elif args.impl == "reference":
        run_reference(args)
    elif args.sweep:
        run_sweep(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
