"""Layer forwards over token batches that live in host memory.

The reference takes host slices and returns host slices (model/mod.rs:1245-1633
runs on the CPU). A caller that keeps its activations on the host hands this
class pinned host batches; each batch is copied to the device, run through the
layer and copied back, with the copies of neighbouring batches overlapping the
compute: a host->device stream and a device->host stream around the compute
stream, and `depth` device staging buffers in each direction.
"""
from __future__ import annotations


def _torch():
    import torch

    return torch


class HostPipeline:
    """Runs ``layer.forward(x_dev, out=y_dev, **fwd_kw)`` over host batches.

    layer: any object with that forward (``MoeLayer``, ``EPMoeLayer``).
    T, d:  rows and columns of every batch (f32).
    """

    def __init__(self, layer, T: int, d: int, depth: int = 2, device=None, **fwd_kw):
        torch = _torch()
        self.layer, self.T, self.d, self.depth, self.kw = layer, T, d, depth, fwd_kw
        dev = torch.device("cuda", torch.cuda.current_device() if device is None else device)
        self.xin = [torch.empty((T, d), dtype=torch.float32, device=dev) for _ in range(depth)]
        self.yout = [torch.empty((T, d), dtype=torch.float32, device=dev) for _ in range(depth)]
        self.h2d, self.d2h = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
        ev = lambda: [torch.cuda.Event() for _ in range(depth)]
        self.in_ready, self.done, self.copied = ev(), ev(), ev()
        self.n = 0  # batches issued so far (buffer reuse is ordered across run() calls)

    def run(self, xs_host, outs_host, layers=None):
        """Issues every batch (batch i through ``layers[i]`` when given, else the
        pipeline's layer); returns when all are queued. ``outs_host`` are valid
        after ``finish()`` and a synchronisation of the compute stream."""
        torch = _torch()
        comp = torch.cuda.current_stream()
        for k, (xh, oh) in enumerate(zip(xs_host, outs_host)):
            if layers is not None:
                self.layer = layers[k]
            i, s = self.n, self.n % self.depth
            with torch.cuda.stream(self.h2d):
                if i >= self.depth:
                    self.h2d.wait_event(self.done[s])  # the compute of batch i - depth has read xin[s]
                self.xin[s].copy_(xh, non_blocking=True)
                self.in_ready[s].record(self.h2d)
            comp.wait_event(self.in_ready[s])
            if i >= self.depth:
                comp.wait_event(self.copied[s])  # yout[s] of batch i - depth is back on the host
            self.layer.forward(self.xin[s], out=self.yout[s], **self.kw)
            self.done[s].record(comp)
            with torch.cuda.stream(self.d2h):
                self.d2h.wait_event(self.done[s])
                oh.copy_(self.yout[s], non_blocking=True)
                self.copied[s].record(self.d2h)
            self.n += 1
        return outs_host

    def finish(self):
        """Makes the compute stream wait for every device->host copy issued so far."""
        _torch().cuda.current_stream().wait_stream(self.d2h)
