"""TensorProduct forward + VJP over rows held in host memory.

A caller whose rows live on the host (a data loader, a host runtime calling the C ABI)
pays for moving x, y and the cotangent to the GPU and out, dx and dy back.  The runner
streams the rows through the GPU in chunks on three CUDA streams: the host-to-device
copies of chunk c + 1, the kernels of chunk c and the device-to-host copies of chunk
c - 1 run at the same time, and the two copy directions use separate copy engines, so
a step costs about one direction's transfer instead of both.  The weight gradient is
summed over the chunks in chunk order on the compute stream (deterministic).

Host tensors should be pinned (``torch.empty(..., pin_memory=True)``) for the copies to
be asynchronous.  The kernels are those of ``TensorProduct`` (the same C ABI calls).
"""

from __future__ import annotations

import torch

from . import _lib
from .ops import require_cuda_float32


class TensorProductHostRunner:
    """Chunked, overlapped forward + VJP of ``tp`` for host-resident rows.

    ``run(x, y, g, out, dx, dy)`` reads x, y, g (host, ``[N, W]`` float32), writes the
    forward output and the input gradients into out, dx, dy (host, ``[N, W]``) and
    returns the weight gradient (device tensor shaped like ``tp.weight``).  The work
    is ordered before later work on the caller's current stream; synchronize that
    stream before reading the host outputs.
    """

    def __init__(self, tp, chunk_rows: int = 4096):
        from .tensor_product import TensorProduct
        if type(tp) is not TensorProduct:
            raise TypeError("TensorProductHostRunner takes a TensorProduct (channel-major rows)")
        if chunk_rows < 1:
            raise ValueError("chunk_rows must be >= 1")
        self.tp = tp
        self.chunk = int(chunk_rows)
        weight = tp.weight
        require_cuda_float32("TensorProductHostRunner", weight)
        self.device = weight.device
        W = tp.representation_dimension
        self.streams = [torch.cuda.Stream(self.device) for _ in range(3)]
        self.buffers = [{name: torch.empty(self.chunk, W, device=self.device)
                         for name in ("x", "y", "g", "out", "dx", "dy")} for _ in range(2)]
        self.dw_chunk = torch.empty_like(weight)
        size = _lib.tp_backward_workspace(self.chunk, tp.channels, tp.max_frequency, tp.parity,
                                          self.device)
        self.workspace = torch.empty(max(size, 16), dtype=torch.uint8, device=self.device)
        self.loaded = [torch.cuda.Event() for _ in range(2)]
        self.computed = [torch.cuda.Event() for _ in range(2)]
        self.stored = [torch.cuda.Event() for _ in range(2)]

    def _workspace_for(self, rows: int) -> torch.Tensor:
        tp = self.tp
        size = _lib.tp_backward_workspace(rows, tp.channels, tp.max_frequency, tp.parity,
                                          self.device)
        if size > self.workspace.numel():
            # earlier runs may still use the old buffer on the compute stream
            self.workspace.record_stream(self.streams[1])
            self.workspace = torch.empty(size, dtype=torch.uint8, device=self.device)
        return self.workspace

    def run(self, x: torch.Tensor, y: torch.Tensor, g: torch.Tensor, out: torch.Tensor,
            dx: torch.Tensor, dy: torch.Tensor) -> torch.Tensor:
        tp = self.tp
        W = tp.representation_dimension
        for name, t in (("x", x), ("y", y), ("g", g), ("out", out), ("dx", dx), ("dy", dy)):
            if t.device.type != "cpu" or t.dtype != torch.float32 or t.dim() != 2 \
                    or t.shape[1] != W or not t.is_contiguous():
                raise ValueError(f"{name} must be a contiguous host float32 [N, {W}] tensor")
        n = x.shape[0]
        if any(t.shape[0] != n for t in (y, g, out, dx, dy)):
            raise ValueError("all host tensors must have the same number of rows")
        cfg = (tp.channels, tp.max_frequency, tp.parity, tp.normalization)
        weight = tp.weight.detach()
        h2d, comp, d2h = self.streams
        current = torch.cuda.current_stream(self.device)
        for s in self.streams:
            s.wait_stream(current)
        with torch.cuda.stream(comp):
            dw = torch.zeros_like(weight)
        chunks = (n + self.chunk - 1) // self.chunk
        self._workspace_for(min(n, self.chunk))
        workspace = self._workspace_for(n - (chunks - 1) * self.chunk if chunks else 1)
        for c in range(chunks):
            b, buf = c % 2, self.buffers[c % 2]
            r0, r1 = c * self.chunk, min(n, (c + 1) * self.chunk)
            m = r1 - r0
            with torch.cuda.stream(h2d):
                if c >= 2:
                    h2d.wait_event(self.stored[b])  # chunk c - 2 has left this buffer
                for name, src in (("x", x), ("y", y), ("g", g)):
                    buf[name][:m].copy_(src[r0:r1], non_blocking=True)
                self.loaded[b].record(h2d)
            with torch.cuda.stream(comp):
                comp.wait_event(self.loaded[b])
                bx, by, bg = buf["x"][:m], buf["y"][:m], buf["g"][:m]
                _lib.tp_forward(bx, by, weight, buf["out"][:m], *cfg)
                _lib.tp_backward(bx, by, weight, bg, buf["dx"][:m], buf["dy"][:m],
                                 self.dw_chunk, workspace, *cfg)
                dw.add_(self.dw_chunk)
                self.computed[b].record(comp)
            with torch.cuda.stream(d2h):
                d2h.wait_event(self.computed[b])
                for name, dst in (("out", out), ("dx", dx), ("dy", dy)):
                    dst[r0:r1].copy_(buf[name][:m], non_blocking=True)
                self.stored[b].record(d2h)
        current.wait_stream(comp)
        current.wait_stream(d2h)
        dw.record_stream(current)
        return dw
