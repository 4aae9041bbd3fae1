"""Data-parallel support: the one cross-rank exchange of the group-rational path.

The forward and the input gradient are elementwise, so a batch-sharded run needs no
communication for them.  The coefficient gradients (weight_numerator [1, 6] and
weight_denominator [G, 4] of every KAT module, 10 G floats each) are sums over the batch,
so ranks exchange them once per step.  The reference has no distributed layer; this is
the B200 data-parallel design: one process per GPU, torch.distributed over NCCL.

Two ways to do it:
  * `PeerExchange` + `KAT_Group.enable_data_parallel()`: the exchange is fused into the
    backward's gradient-reduction kernel (kat_rational_bwd_allreduce): each rank stores its
    fp64 group sums straight into every peer's exchange buffer over NVLink, raises a flag,
    waits (bounded) for the others and adds the ranks in rank order — one kernel, no NCCL
    call on the step.  One node, up to 8 ranks, buffers shared through CUDA IPC.
  * `allreduce_coefficient_grads`: after a plain backward, all-gather every rank's
    flattened coefficient gradients (NCCL or gloo) and add them in rank order in float64.
Both leave bit-identical gradients on every rank, independent of any library's internal
reduction order.
"""

from __future__ import annotations

import ctypes
from typing import Iterable, List, Optional

import torch
import torch.distributed as dist

from . import _native


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


class PeerExchange:
    """Exchange buffers of one KAT module across the ranks of a single node.

    Each rank creates a zeroed buffer of kat_rational_exchange_buffer_bytes(G) bytes on its
    GPU (kat_rational_exchange_create) and publishes its 64-byte CUDA IPC handle
    (all_gather_object); every rank maps the others' buffers on its own device with lazy
    peer access and checks each mapping with a small copy before any kernel uses it
    (kat_rational_exchange_open).  `peers` is the kat_rational_peers descriptor the
    data-parallel backward takes.  Construction and close() are collective.  A failed
    exchange (KAT_DEVICE_EXCHANGE_TIMEOUT) leaves the buffers broken: every later backward
    through them writes NaN gradients until a new PeerExchange replaces this one.
    """

    def __init__(self, num_groups: int, group=None, average: bool = True,
                 timeout_ms: int = 5000, device: Optional[torch.device] = None):
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        if world > _native.KAT_MAX_PEERS:
            raise ValueError(f"PeerExchange supports up to {_native.KAT_MAX_PEERS} ranks on one "
                             f"node, got {world}")
        device = device or torch.device("cuda", torch.cuda.current_device())
        lib = _native.lib()
        self._lib = lib
        self._opened: List[int] = []
        self._local = None
        self.group = group
        self.device = device
        self.peers_groups = int(num_groups)
        with torch.cuda.device(device):
            local = ctypes.c_void_p()
            handle = (ctypes.c_char * 64)()
            _native.check("kat_rational_exchange_create",
                          lib.kat_rational_exchange_create(num_groups, ctypes.byref(local),
                                                           handle))
            self._local = local.value
            handles: list = [None] * world
            dist.all_gather_object(handles, bytes(handle), group=group)
            probe = torch.empty(16, dtype=torch.uint8, device=device)
            ptrs = []
            for r in range(world):
                if r == rank:
                    ptrs.append(self._local)
                    continue
                peer = ctypes.c_void_p()
                h = (ctypes.c_char * 64).from_buffer_copy(handles[r])
                _native.check("kat_rational_exchange_open",
                              lib.kat_rational_exchange_open(h, ctypes.c_void_p(probe.data_ptr()),
                                                             ctypes.byref(peer)))
                self._opened.append(peer.value)
                ptrs.append(peer.value)
        self.peers = _native.KatPeers()
        self.peers.world_size = world
        self.peers.rank = rank
        self.peers.average = 1 if average else 0
        self.peers.timeout_ms = int(timeout_ms)
        for r, ptr in enumerate(ptrs):
            self.peers.buffers[r] = ctypes.c_void_p(ptr)
        dist.barrier(group=group)

    def exchange_grads(self, grad_numerator: torch.Tensor, grad_denominator: torch.Tensor,
                       stream: Optional[torch.cuda.Stream] = None) -> None:
        """In place: this rank's fp32 coefficient gradients [G, 6] and [G, 4] become the
        rank-order sum (or average) over all ranks, through the same buffers and epoch as the
        fused backward (kat_rational_exchange_grads).  Enqueued on `stream` (default: current);
        every rank must make the same sequence of exchanges."""
        for t, cols in ((grad_numerator, 6), (grad_denominator, 4)):
            if (t.dtype != torch.float32 or not t.is_contiguous() or t.device != self.device or
                    t.shape != (self.peers_groups, cols)):
                raise ValueError(f"exchange_grads expects contiguous fp32 [{self.peers_groups}, "
                                 f"{cols}] tensors on {self.device}")
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        _native.check("kat_rational_exchange_grads", self._lib.kat_rational_exchange_grads(
            grad_numerator.data_ptr(), grad_denominator.data_ptr(), self.peers_groups,
            ctypes.byref(self.peers), ctypes.c_void_p(s.cuda_stream)))

    def close(self) -> None:
        """Collective teardown: every rank of the group must call it, after its last use.

        Each rank waits for its own work on the device, unmaps the peers' buffers, then all
        ranks meet at a barrier, and only then does each rank free its own buffer: a buffer is
        never freed while another rank still maps it (freeing an exported allocation before
        its importers close it is undefined).  If the barrier fails (a rank is gone), the
        local buffer is left allocated and the error propagates."""
        if self._lib is None:
            return
        lib = self._lib
        self._close_peers()
        self._lib = None
        dist.barrier(group=self.group)
        if self._local is not None:
            lib.kat_rational_exchange_destroy(ctypes.c_void_p(self._local))
            self._local = None

    def _close_peers(self) -> None:
        if self.device is not None and self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
        for ptr in self._opened:
            self._lib.kat_rational_exchange_close(ctypes.c_void_p(ptr))
        self._opened = []

    def __del__(self):
        # Garbage collection cannot run the collective part of close(): unmap the peers'
        # buffers, but leave the local buffer allocated (it goes with the process) rather than
        # free it under a peer that may still map it.
        try:
            if self._lib is not None:
                self._close_peers()
                self._lib = None
        except Exception:
            pass
