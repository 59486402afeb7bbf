"""Several DCNv2 layers of one network step (the FPN levels of a detector head) as one CUDA graph.

A detector with DCN in its FPN head runs one DCNv2 layer per level (P3..P7 at 512x512 input:
64x64 down to 4x4 outputs). Each small level is a single wave of a few dozen tiles whose
duration is one tile's full K loop, so run one after another the small levels leave most SMs
idle. LevelsRunner issues every level through dcnv2_forward on a stream of its own (forked from
and joined back into the caller's stream with events), so the levels' fused kernels run side by
side on different SMs, and captures that fork-join once into a CUDA graph that each step
replays. Every level keeps its own workspace and output; dcnv2_forward never allocates or
synchronises, which is what makes the capture valid.

This is host-side plumbing over the C ABI (torch for streams, events and the graph); every
layer's arithmetic is the fused kernel's.
"""
from __future__ import annotations

from typing import List, Sequence

from . import capi
from .capi import DCNv2Error, DType, Status


class LevelsRunner:
    """levels: per level a dict with CUDA tensors x, offset, mask, weight, bias (bias may be None)
    and optional stride / padding / dilation / deformable_groups / x_scale / w_scale / math.
    Outputs are allocated once (`outputs`) and rewritten by every run()."""

    def __init__(self, levels: Sequence[dict], use_graph: bool = True):
        import torch
        self.torch = torch
        if not levels:
            raise ValueError("LevelsRunner needs at least one level")
        self.device = levels[0]["x"].device
        self.calls = []
        self.outputs: List = []
        for lv in levels:
            x, w = lv["x"], lv["weight"]
            dt = {torch.float32: DType.FLOAT, torch.float16: DType.HALF,
                  torch.int8: DType.INT8}[x.dtype]
            n, c, h, wd = (int(v) for v in x.shape)
            desc = capi.make_desc(n, c, h, wd, int(w.shape[0]), int(w.shape[2]),
                                  lv.get("stride", 1), lv.get("padding", 1),
                                  lv.get("dilation", 1), lv.get("deformable_groups", 1), dt,
                                  lv.get("math", capi.Math.DEFAULT))
            shape = capi.output_shape(desc)
            ydt = torch.float16 if dt == DType.HALF else torch.float32
            y = torch.empty(shape, dtype=ydt, device=self.device)
            ws = torch.empty(capi.workspace_size(desc), dtype=torch.uint8, device=self.device)
            b = lv.get("bias")
            self.calls.append((desc, x, lv["offset"], lv["mask"], w, b, y, ws,
                               float(lv.get("x_scale", 1.0)), float(lv.get("w_scale", 1.0))))
            self.outputs.append(y)
        self.streams = [torch.cuda.Stream(self.device) for _ in self.calls]
        self.graph = None
        if use_graph:
            # Warm up eagerly on a side stream (first calls set per-device launch attributes),
            # then capture the fork-join.
            side = torch.cuda.Stream(self.device)
            side.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(side):
                for _ in range(2):
                    self._issue(side)
            torch.cuda.current_stream(self.device).wait_stream(side)
            torch.cuda.synchronize(self.device)
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph):
                self._issue(torch.cuda.current_stream(self.device))

    def _issue(self, main):
        torch = self.torch
        fork = torch.cuda.Event()
        fork.record(main)
        joins = []
        for st, (desc, x, off, m, w, b, y, ws, xs, wsc) in zip(self.streams, self.calls):
            st.wait_event(fork)
            rc = capi.forward_raw(desc, x.data_ptr(), off.data_ptr(), m.data_ptr(), w.data_ptr(),
                                  b.data_ptr() if b is not None else None, y.data_ptr(),
                                  ws.data_ptr(), ws.numel(), xs, wsc, st.cuda_stream)
            if rc != Status.OK:
                raise DCNv2Error(rc, "dcnv2_forward")
            ev = torch.cuda.Event()
            ev.record(st)
            joins.append(ev)
        for ev in joins:
            main.wait_event(ev)

    def run(self, stream=None):
        """All levels once, on `stream` (the current stream by default); asynchronous."""
        torch = self.torch
        main = stream if stream is not None else torch.cuda.current_stream(self.device)
        if self.graph is not None:
            with torch.cuda.stream(main):
                self.graph.replay()
        else:
            self._issue(main)
        return self.outputs
