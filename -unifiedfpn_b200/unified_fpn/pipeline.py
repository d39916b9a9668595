"""Host-to-host streaming through the neck.

The reference's forward copies nothing itself (python/fpn_pytorch.cpp:84-137 takes CUDA
tensors); a caller whose backbone features live in host memory pays one host->device copy
of C2..C5 and one device->host copy of P2..P6 per batch.  ``HostPipeline`` hides most of
that cost: batch i's neck runs while batch i+1 is copied in and batch i-1 is copied out,
on three CUDA streams (copy-in, compute, copy-out) over ``depth`` device buffer sets, with
events ordering every reuse of a buffer.  Every batch still makes both copies.
"""
from __future__ import annotations

from typing import Sequence

import torch

from .ops import E4M3


class HostPipeline:
    """Overlapped host -> neck -> host streaming for one ``UnifiedFPN``.

    ``like``: C2..C5 tensors (any device) giving the batch's shapes, dtype and memory
    format.  ``submit`` enqueues one batch: ``host_in`` (pinned C2..C5), ``host_out``
    (pinned P2..P5 [, P6]) and, for float8_e4m3fn inputs, ``host_scales`` (pinned fp32 [4]).
    Nothing blocks the host; ``synchronize`` waits for every submitted batch.  The caller
    must not reuse a ``host_out`` set before the batch that fills it has completed.
    """

    def __init__(self, fpn, like: Sequence[torch.Tensor], return_p6: bool = True, depth: int = 2):
        if depth < 1:
            raise ValueError("depth must be >= 1")
        self.fpn = fpn
        self.dev = fpn.device
        self.return_p6 = return_p6
        self.depth = depth
        self.fp8 = like[0].dtype == E4M3
        mf = torch.channels_last if all(
            t.is_contiguous(memory_format=torch.channels_last) for t in like) else torch.contiguous_format
        self.mf = mf
        self.dev_in = [[torch.empty(t.shape, dtype=t.dtype, device=self.dev, memory_format=mf) for t in like]
                       for _ in range(depth)]
        self.dev_scales = [torch.empty(4, dtype=torch.float32, device=self.dev) if self.fp8 else None
                           for _ in range(depth)]
        N = like[0].shape[0]
        odt = torch.bfloat16 if self.fp8 else like[0].dtype
        shapes = [(N, 256, t.shape[2], t.shape[3]) for t in like]
        if return_p6:
            H5, W5 = like[3].shape[2], like[3].shape[3]
            shapes.append((N, 256, (H5 - 1) // 2 + 1, (W5 - 1) // 2 + 1))
        self.out_shapes = shapes
        self.out_dtype = odt
        self.dev_out = [[torch.empty(s, dtype=odt, device=self.dev, memory_format=mf) for s in shapes]
                        for _ in range(depth)]
        self.s_in = torch.cuda.Stream(self.dev)
        self.s_compute = torch.cuda.Stream(self.dev)
        self.s_out = torch.cuda.Stream(self.dev)
        self.ev_in = [torch.cuda.Event() for _ in range(depth)]
        self.ev_done = [torch.cuda.Event() for _ in range(depth)]
        self.ev_out = [torch.cuda.Event() for _ in range(depth)]
        self.used = [False] * depth
        self.k = 0

    def host_buffers(self, pinned: bool = True):
        """A fresh set of host output tensors of the right shapes (pinned by default)."""
        return [torch.empty(s, dtype=self.out_dtype, memory_format=self.mf, pin_memory=pinned)
                for s in self.out_shapes]

    def submit(self, host_in: Sequence[torch.Tensor], host_out: Sequence[torch.Tensor],
               host_scales: torch.Tensor | None = None) -> None:
        j = self.k % self.depth
        self.k += 1
        d_in, d_out = self.dev_in[j], self.dev_out[j]
        with torch.cuda.stream(self.s_in):
            if self.used[j]:
                self.s_in.wait_event(self.ev_done[j])  # the neck that read d_in[j] is done
            for d, h in zip(d_in, host_in):
                d.copy_(h, non_blocking=True)
            if self.fp8:
                if host_scales is None:
                    raise ValueError("float8_e4m3fn inputs need host_scales")
                self.dev_scales[j].copy_(host_scales, non_blocking=True)
            self.ev_in[j].record(self.s_in)
        with torch.cuda.stream(self.s_compute):
            self.s_compute.wait_event(self.ev_in[j])
            if self.used[j]:
                self.s_compute.wait_event(self.ev_out[j])  # d_out[j] has been copied out
            self.fpn(d_in, return_p6=self.return_p6, out=d_out,
                     input_scales=self.dev_scales[j] if self.fp8 else None)
            self.ev_done[j].record(self.s_compute)
        with torch.cuda.stream(self.s_out):
            self.s_out.wait_event(self.ev_done[j])
            for h, d in zip(host_out, d_out):
                h.copy_(d, non_blocking=True)
            self.ev_out[j].record(self.s_out)
        self.used[j] = True

    def join(self, stream: torch.cuda.Stream) -> None:
        """Make ``stream`` wait for everything submitted so far (no host block)."""
        for s in (self.s_in, self.s_compute, self.s_out):
            ev = torch.cuda.Event()
            ev.record(s)
            stream.wait_event(ev)

    def fork(self, stream: torch.cuda.Stream) -> None:
        """Make the pipeline's streams wait for work already enqueued on ``stream``."""
        ev = torch.cuda.Event()
        ev.record(stream)
        for s in (self.s_in, self.s_compute, self.s_out):
            s.wait_event(ev)

    def synchronize(self) -> None:
        for s in (self.s_in, self.s_compute, self.s_out):
            s.synchronize()
