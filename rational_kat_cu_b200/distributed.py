"""Data-parallel support: the one cross-rank exchange of the group-rational path.

The forward and the input gradient are elementwise, so a batch-sharded run needs no
communication for them.  The coefficient gradients (weight_numerator [1, 6] and
weight_denominator [G, 4] of every KAT module, 10 G floats each) are sums over the batch,
so ranks exchange them once per step.  The reference has no distributed layer; this is
the B200 data-parallel design: one process per GPU, torch.distributed over NCCL.

`allreduce_coefficient_grads` all-gathers every rank's flattened coefficient gradients
and adds them in rank order in float64 on every rank, so all ranks end with bit-identical
gradients that do not depend on the collective's internal reduction order.
"""

from __future__ import annotations

from typing import Iterable, List

import torch
import torch.distributed as dist


def coefficient_parameters(module: torch.nn.Module) -> List[torch.nn.Parameter]:
    """weight_numerator / weight_denominator of every KAT module inside `module`, in
    module order."""
    params = []
    for m in module.modules():
        num = getattr(m, "weight_numerator", None)
        den = getattr(m, "weight_denominator", None)
        if isinstance(num, torch.nn.Parameter) and isinstance(den, torch.nn.Parameter):
            params.extend([num, den])
    return params


def allreduce_coefficient_grads(params_or_module, group=None, average: bool = True,
                                async_op: bool = False):
    """Sum (or average) the .grad of the given coefficient parameters across ranks.

    Every rank contributes its local gradient; parameters without a gradient contribute
    zeros.  With async_op=True the gather is issued and a callable is returned that
    finishes the reduction (call it before reading the gradients).
    """
    if isinstance(params_or_module, torch.nn.Module):
        params = coefficient_parameters(params_or_module)
    else:
        params = list(params_or_module)
    if not params:
        return (lambda: None) if async_op else None
    device = params[0].device
    flat = torch.cat([
        (p.grad if p.grad is not None else torch.zeros_like(p)).detach().reshape(-1).float()
        for p in params
    ])
    world = dist.get_world_size(group)
    if world == 1:
        return (lambda: None) if async_op else None
    if dist.get_backend(group) == "nccl":
        gathered = torch.empty(world, flat.numel(), device=device, dtype=flat.dtype)
        work = dist.all_gather_into_tensor(gathered, flat, group=group, async_op=True)
        parts = None
    else:
        parts = [torch.empty_like(flat) for _ in range(world)]
        work = dist.all_gather(parts, flat, group=group, async_op=True)
        gathered = None

    def finish():
        work.wait()
        stacked = gathered if gathered is not None else torch.stack(parts)
        total = stacked.double()[0].clone()
        for r in range(1, world):
            total += stacked[r].double()
        if average:
            total /= world
        offset = 0
        for p in params:
            n = p.numel()
            g = total[offset:offset + n].view_as(p).to(p.dtype)
            if p.grad is None:
                p.grad = g
            else:
                p.grad.copy_(g)
            offset += n

    if async_op:
        return finish
    finish()
    return None


def shard_rows(total_rows: int, rank: int, world: int) -> slice:
    """Even contiguous split of `total_rows` batch rows: the rows rank `rank` processes."""
    lo = total_rows * rank // world
    hi = total_rows * (rank + 1) // world
    return slice(lo, hi)


def barrier_all(groups: Iterable = (None,)) -> None:
    for g in groups:
        dist.barrier(group=g)
