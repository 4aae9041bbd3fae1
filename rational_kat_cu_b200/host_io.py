"""Forward + backward of a KAT module over host-resident batches, with the transfers
overlapped.

A caller that holds its activations in (pinned) host memory pays for moving x and grad_out
to the GPU and y and dx back.  Done one after the other these copies dominate; here the
batch is cut into row chunks and three CUDA streams run them as a pipeline:

    host->device copy of chunk i+1  |  forward+backward of chunk i  |  device->host copy of chunk i-1

H2D and D2H use the two directions of the link at the same time, so a step costs about the
larger of the two transfers instead of their sum.  The kernels are driven through the C ABI
with preallocated per-slot device buffers (no autograd work per chunk); each chunk's
coefficient gradients land in their own row of a [chunks, G, 10] buffer, summed once per
step in chunk order (exchanged with the other ranks when the module is data parallel, see
KAT_Group.enable_data_parallel) and added to the module's .grad — deterministic for a fixed
chunk count.  The reference has no host-buffer API; this is the B200 design's way to feed the
kernels from host memory.
"""

from __future__ import annotations

import ctypes
from typing import List, Optional, Tuple

import torch

from . import _native
from .kat_2dgroup import KAT_Group2D
from .rational_cuda import _DTYPE_CODES


def _chunks(rows: int, n: int) -> List[Tuple[int, int]]:
    n = max(1, min(n, rows)) if rows else 1
    return [(rows * i // n, rows * (i + 1) // n) for i in range(n)]


class HostPipeline:
    """Forward+backward of a KAT_Group / KAT_Group2D (or a RatGroup, the abs-after-sum
    formula) over pinned host tensors with overlapped copies.  Device buffers are kept for
    reuse while the input shape stays."""

    def __init__(self, module: torch.nn.Module, chunks: int = 4, slots: int = 3,
                 device: Optional[torch.device] = None):
        self.module = module
        self.chunks = chunks
        self.slots = max(2, slots)
        self.device = device or module.weight_numerator.device
        self.h2d = torch.cuda.Stream(self.device)
        self.comp = torch.cuda.Stream(self.device)
        self.d2h = torch.cuda.Stream(self.device)
        self._state = None
        self._key = None

    def _dims(self, shape) -> Tuple[int, int, int]:
        if isinstance(self.module, KAT_Group2D):
            return shape[0], shape[1], shape[2] * shape[3]
        c = shape[-1]
        rows = 1
        for s in shape[:-1]:
            rows *= s
        return rows, c, 1

    def _prepare(self, x_host: torch.Tensor, bounds):
        G = self.module.num_groups
        max_rows = max(r1 - r0 for r0, r1 in bounds)
        key = (tuple(x_host.shape), x_host.dtype, tuple(bounds))
        if self._key == key:
            return self._state
        shape = (max_rows,) + tuple(x_host.shape[1:])
        dev, dt = self.device, x_host.dtype
        slots = [dict(x=torch.empty(shape, dtype=dt, device=dev),
                      g=torch.empty(shape, dtype=dt, device=dev),
                      y=torch.empty(shape, dtype=dt, device=dev),
                      dx=torch.empty(shape, dtype=dt, device=dev)) for _ in range(self.slots)]
        dims = self._dims(shape)
        code = _DTYPE_CODES[dt]
        need = ctypes.c_size_t(0)
        _native.check("kat_rational_bwd_workspace_size",
                      _native.lib().kat_rational_bwd_workspace_size(
                          dims[0], dims[1], dims[2], G, code, dev.index, ctypes.byref(need)))
        if self._state is not None:
            self.wait()   # the old buffers may still be in use
        state = dict(slots=slots, code=code, G=G,
                     ws=torch.empty(max(need.value, 16), dtype=torch.uint8, device=dev),
                     dn=torch.empty(len(bounds), G, 6, device=dev),
                     dd=torch.empty(len(bounds), G, 4, device=dev),
                     ev_in=[torch.cuda.Event() for _ in range(self.slots)],
                     ev_comp=[torch.cuda.Event() for _ in range(self.slots)],
                     ev_out=[torch.cuda.Event() for _ in range(self.slots)],
                     used=[False] * self.slots)
        self._state, self._key = state, key
        return state

    def wait(self) -> None:
        """Make the current stream wait for every copy and kernel this pipeline enqueued."""
        cur = torch.cuda.current_stream(self.device)
        cur.wait_stream(self.comp)
        cur.wait_stream(self.d2h)

    def wait_compute(self) -> None:
        """Make the current stream wait for the kernels only (the coefficient gradients are
        final); the downloads of y and dx may still be running."""
        torch.cuda.current_stream(self.device).wait_stream(self.comp)

    def run(self, x_host: torch.Tensor, grad_host: torch.Tensor, y_host: torch.Tensor,
            dx_host: torch.Tensor, grads_host: Optional[List[torch.Tensor]] = None,
            wait: bool = True) -> None:
        """y_host <- module(x_host); dx_host <- d(y . grad_host)/dx; the coefficient
        gradients are added to the module's .grad (as a backward call would).  If
        `grads_host` = [numerator [1,6], denominator [G,4]] host tensors is given, the
        resulting .grad values are copied there.  Host tensors should be pinned.  Returns
        with the work enqueued.  With wait=True the current stream waits for all of it; with
        wait=False consecutive calls overlap (the next call's uploads start while this
        call's downloads run) and the caller calls wait() before using the results."""
        if not (x_host.shape == grad_host.shape == y_host.shape == dx_host.shape):
            raise ValueError("x, grad_out, y and dx host tensors must have the same shape")
        if x_host.dtype not in _DTYPE_CODES or grad_host.dtype != x_host.dtype:
            raise TypeError("host tensors must share a float32 / float16 / bfloat16 dtype")
        mod = self.module
        lib = _native.lib()
        cur = torch.cuda.current_stream(self.device)
        bounds = _chunks(x_host.shape[0], self.chunks)
        st = self._prepare(x_host, bounds)
        G, code = st["G"], st["code"]
        for s in (self.h2d, self.comp, self.d2h):
            s.wait_stream(cur)
        with torch.cuda.stream(self.comp):
            num = mod.weight_numerator.detach().float().expand(G, 6).contiguous()
            den = mod.weight_denominator.detach().float().contiguous()
        comp_ptr = ctypes.c_void_p(self.comp.cuda_stream)
        formula = getattr(mod, "formula", _native.KAT_FORMULA_KAT)
        if formula == _native.KAT_FORMULA_KAT:
            fwd = lambda *a: lib.kat_rational_fwd(*a, comp_ptr)
            bwd = lambda *a: lib.kat_rational_bwd(*a, comp_ptr)
        else:
            fwd = lambda *a: lib.kat_rational_fwd_formula(*a, formula, comp_ptr)
            bwd = lambda *a: lib.kat_rational_bwd_formula(*a, formula, comp_ptr)
        ev_in, ev_comp, ev_out, used = st["ev_in"], st["ev_comp"], st["ev_out"], st["used"]
        for i, (r0, r1) in enumerate(bounds):
            k = i % self.slots
            b = st["slots"][k]
            n = r1 - r0
            dims = self._dims((n,) + tuple(x_host.shape[1:]))
            with torch.cuda.stream(self.h2d):
                if used[k]:
                    self.h2d.wait_event(ev_comp[k])   # compute of the slot's last chunk done
                b["x"][:n].copy_(x_host[r0:r1], non_blocking=True)
                b["g"][:n].copy_(grad_host[r0:r1], non_blocking=True)
                ev_in[k].record(self.h2d)
            self.comp.wait_event(ev_in[k])
            if used[k]:
                self.comp.wait_event(ev_out[k])       # y / dx of the slot copied out
            _native.check("kat_rational_fwd", fwd(
                b["x"].data_ptr(), b["y"].data_ptr(), num.data_ptr(), den.data_ptr(),
                dims[0], dims[1], dims[2], G, code))
            _native.check("kat_rational_bwd", bwd(
                b["x"].data_ptr(), b["g"].data_ptr(), b["dx"].data_ptr(), num.data_ptr(),
                den.data_ptr(), st["dn"][i].data_ptr(), st["dd"][i].data_ptr(),
                st["ws"].data_ptr(), st["ws"].numel(), dims[0], dims[1], dims[2], G, code))
            ev_comp[k].record(self.comp)
            with torch.cuda.stream(self.d2h):
                self.d2h.wait_event(ev_comp[k])
                y_host[r0:r1].copy_(b["y"][:n], non_blocking=True)
                dx_host[r0:r1].copy_(b["dx"][:n], non_blocking=True)
                ev_out[k].record(self.d2h)
            used[k] = True
        with torch.cuda.stream(self.comp):
            dn_g = st["dn"][:len(bounds)].sum(dim=0)     # [G, 6], chunks in order
            d_den = st["dd"][:len(bounds)].sum(dim=0)    # [G, 4]
            exchange = getattr(mod, "exchange", None)
            if exchange is not None:
                # data parallel (KAT_Group.enable_data_parallel): the rank-order sum over the
                # ranks, through the module's NVLink exchange buffers
                exchange.exchange_grads(dn_g, d_den, self.comp)
            d_num = dn_g.sum(dim=0).view(1, 6)
            for p, g in ((mod.weight_numerator, d_num), (mod.weight_denominator, d_den)):
                g = g.reshape(p.shape).to(p.dtype)
                if p.grad is None:
                    p.grad = g
                else:
                    p.grad.add_(g)
        if grads_host is not None:
            with torch.cuda.stream(self.d2h):
                self.d2h.wait_stream(self.comp)
                grads_host[0].copy_(mod.weight_numerator.grad, non_blocking=True)
                grads_host[1].copy_(mod.weight_denominator.grad, non_blocking=True)
        if wait:
            self.wait()
