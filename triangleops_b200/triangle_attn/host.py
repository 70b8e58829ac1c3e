"""Triangle attention on host (pinned) tensors with the copies overlapped.

A caller whose pair tensor lives in host memory pays one host->device copy of X
and one device->host copy of the result per call (2 x 1 GiB at N = 2048, C = 128,
about 20 ms each over PCIe). ``HostPipeline`` hides most of it:

* within a call, X arrives in row slabs on a copy stream and each slab is
  projected (LN + Q/K/V/bias, ``tops_triangle_attn_project``) as soon as it lands;
  after the last slab the bias slabs are assembled (every row's attention needs the
  whole shared bias), then attention + gate run slab by slab and each finished slab
  leaves on a second copy stream while the next one computes;
* across calls nothing synchronises, so the host->device copy of call t+1 runs
  while call t computes and copies its result back (PCIe is full duplex).

Device buffers are allocated once per (N, C, H, D, dtype) and reused; events keep
each buffer from being overwritten before its previous reader has finished. The
work of a call is complete when ``wait(stream)`` returns on a stream (it makes that
stream wait) or after ``torch.cuda.synchronize()``.

With torch.distributed initialised (one process per GPU), each rank passes its own
pair rows (rows [r*N/P, (r+1)*N/P) of X and the mask, and its rows of the output):
the ranks' bias rows are all-gathered on the compute stream between the two stages.

No counterpart in the reference (it takes device tensors only); the per-slab work is
the same kernels as ``module.forward``.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from .. import _lib
from .kernel import _mask_u8, gate_forward


class HostPipeline:
    def __init__(self, pre, *, W_proj_g, W_proj_o, scale=1.0, eps=1e-5, slabs=8, group=None):
        self.pre = pre
        self.Wg, self.Wo = W_proj_g, W_proj_o
        self.scale, self.eps, self.slabs = float(scale), float(eps), int(slabs)
        self.group = group
        self._key = None

    def _setup(self, n, N, C, dtype, dev):
        H, D = self.pre["H"], self.pre["D"]
        key = (n, N, C, H, D, dtype, dev)
        if key == self._key:
            return
        assert n % self.slabs == 0, f"{n} rows must be divisible by slabs={self.slabs}"
        nkp = (N + 7) // 8 * 8
        R = n // self.slabs
        f16 = torch.float16
        self.n, self.N, self.C, self.R, self.nkp, self.H, self.D = n, N, C, R, nkp, H, D
        self.x = torch.empty(n, N, C, dtype=dtype, device=dev)
        self.m = torch.empty(n, N, dtype=torch.uint8, device=dev)
        self.xln = torch.empty(n, N, C, dtype=dtype, device=dev)
        self.q = torch.empty(n, H, N, D, dtype=f16, device=dev)
        self.k = torch.empty(n, H, N, D, dtype=f16, device=dev)
        self.vt = torch.empty(n, H, D, nkp, dtype=f16, device=dev)
        self.pen = torch.empty(n, nkp, dtype=f16, device=dev)  # key penalty rows (masked calls)
        self.bias_slab = torch.empty(self.slabs, H, R, nkp, dtype=f16, device=dev)
        self.bias_local = torch.empty(H, n, nkp, dtype=f16, device=dev)
        self.bias = torch.empty(H, N, nkp, dtype=f16, device=dev)
        self.o = torch.empty(n, N, H * D, dtype=dtype, device=dev)
        self.out = torch.empty(n, N, C, dtype=dtype, device=dev)
        self.w = self.pre["W_qkvz"] if self.pre["W_qkvz"].dtype == dtype else self.pre["W_qkvz"].to(dtype)
        self.h2d = torch.cuda.Stream(dev)
        self.d2h = torch.cuda.Stream(dev)
        ev = lambda: [torch.cuda.Event() for _ in range(self.slabs)]  # noqa: E731
        self.ev_in, self.ev_proj, self.ev_gate, self.ev_out = ev(), ev(), ev(), ev()
        self.started = False
        self._key = key

    def __call__(self, X_host, mask_host=None, out_host=None):
        """Enqueue one forward of X_host (n, N, C) pinned — the whole (N, N, C) pair tensor,
        or this rank's n = N/P pair rows when torch.distributed is initialised; the result
        lands in out_host (allocated pinned if None, returned). mask_host: the same rows of
        the (N, N) bool/int mask, pinned, or None."""
        n, N, C = X_host.shape
        world = dist.get_world_size(self.group) if dist.is_available() and dist.is_initialized() else 1
        assert n * world == N, f"X_host holds {n} rows of {N}: expected N / world = {N // world}"
        dev = torch.device("cuda", torch.cuda.current_device())
        _lib.require_cuda(torch.empty(0, device=dev))
        self._setup(n, N, C, X_host.dtype, dev)
        if out_host is None:
            out_host = torch.empty(n, N, C, dtype=X_host.dtype).pin_memory()
        if mask_host is not None:
            mask_host = mask_host.reshape(n, N)
            if mask_host.dtype == torch.bool:
                mask_host = mask_host.view(torch.uint8)  # same bytes, still pinned
            elif mask_host.dtype != torch.uint8:
                mask_host = _mask_u8(mask_host, (n, N))
        compute = torch.cuda.current_stream(dev)
        dt = _lib.dtype_code(X_host.dtype)
        R, H, D, nkp = self.R, self.H, self.D, self.nkp
        st = compute.cuda_stream
        pre = self.pre
        # --- stage A: slabs in, projected as they land
        for i in range(self.slabs):
            r0, r1 = i * R, (i + 1) * R
            with torch.cuda.stream(self.h2d):
                if self.started:
                    self.h2d.wait_event(self.ev_proj[i])  # the previous call's projection read this slab
                self.x[r0:r1].copy_(X_host[r0:r1], non_blocking=True)
                if mask_host is not None:
                    self.m[r0:r1].copy_(mask_host[r0:r1], non_blocking=True)
                self.ev_in[i].record(self.h2d)
            compute.wait_event(self.ev_in[i])
            _lib.call("tops_triangle_attn_project", dt, R, N, C, H, D, self.x[r0].data_ptr(), 1,
                      pre["ln_w32"].data_ptr(), pre["ln_b32"].data_ptr(), self.w.data_ptr(), pre["BZ"].data_ptr(),
                      None if mask_host is None else self.m[r0].data_ptr(), self.scale, self.eps,
                      self.xln[r0].data_ptr(), self.q[r0].data_ptr(), self.k[r0].data_ptr(), self.vt[r0].data_ptr(),
                      None if mask_host is None else self.pen[r0].data_ptr(), self.bias_slab[i].data_ptr(), st)
            self.ev_proj[i].record(compute)
        # the shared bias, [H][N][Np], from the slabs' [H][R][Np] blocks (and the other ranks' rows)
        if world == 1:
            self.bias.view(H, self.slabs, R, nkp).copy_(self.bias_slab.permute(1, 0, 2, 3))
        else:
            self.bias_local.view(H, self.slabs, R, nkp).copy_(self.bias_slab.permute(1, 0, 2, 3))
            gathered = torch.empty(world, H, n, nkp, dtype=self.bias.dtype, device=dev)
            dist.all_gather_into_tensor(gathered.view(-1), self.bias_local.view(-1), group=self.group)
            self.bias.view(H, world, n, nkp).copy_(gathered.permute(1, 0, 2, 3))
        # --- stage B: attention + gate per slab, each slab out while the next computes
        for i in range(self.slabs):
            r0, r1 = i * R, (i + 1) * R
            _lib.call("tops_triangle_attn_attend", dt, R, N, H, D, self.q[r0].data_ptr(), self.k[r0].data_ptr(),
                      self.vt[r0].data_ptr(), None if mask_host is None else self.pen[r0].data_ptr(),
                      self.bias.data_ptr(), self.o[r0].data_ptr(),
                      st)
            if self.started:
                compute.wait_event(self.ev_out[i])  # the previous call's copy-out of this slab
            gate_forward(self.o[r0:r1].view(R * N, H * D), self.xln[r0:r1].view(R * N, C), self.Wg, self.Wo,
                         out=self.out[r0:r1].view(R * N, C))
            self.ev_gate[i].record(compute)
            with torch.cuda.stream(self.d2h):
                self.d2h.wait_event(self.ev_gate[i])
                out_host[r0:r1].copy_(self.out[r0:r1], non_blocking=True)
                self.ev_out[i].record(self.d2h)
        self.started = True
        return out_host

    def wait(self, stream=None):
        """Make ``stream`` (default: the current one) wait for every enqueued copy-out."""
        stream = torch.cuda.current_stream() if stream is None else stream
        if self.started:
            for e in self.ev_out:
                stream.wait_event(e)
