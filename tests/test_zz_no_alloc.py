"""GPU test of dcnv2_forward_static_scratch, the forward for callers that cannot allocate device
memory while they run (a fixed memory plan, a latency-critical loop where cudaMalloc would
synchronise the device, a hard memory budget). Such a caller passes only inputs and outputs;
the scratch comes from the library's own 32 MiB static device buffer.

Two calls in a row go through the C ABI on one stream — a fp16 layer, then an int8 layer of a
different shape that reuses the same buffer — and each output is checked against
dcnv2_forward (own workspace) on the same inputs, with the tolerances of the parity tests
(fp16: mean relative error <= 1e-3; int8: |dy| <= 1e-6 * (|acc*s| + |b|), here exact equality
since the same kernels run), and against the oracle with the same tolerances. The error word of
the static buffer reads clear afterwards. A problem larger than the buffer is refused before any
launch. This file is named to be collected last and runs alone in a fresh process as well.
"""
import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

from dcnv2_b200 import capi  # noqa: E402
from dcnv2_b200.capi import DType, Status  # noqa: E402
from dcnv2_b200.workloads import quantize_sym  # noqa: E402

DEV = "cuda:0"


def _inputs(n, c, h, w, o, k, s, p, d, dg, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    ho = (h + 2 * p - d * (k - 1) - 1) // s + 1
    wo = (w + 2 * p - d * (k - 1) - 1) // s + 1
    x = torch.randn(n, c, h, w, generator=g)
    off = torch.randn(n, 2 * dg * k * k, ho, wo, generator=g) * 0.8
    msk = torch.sigmoid(torch.randn(n, dg * k * k, ho, wo, generator=g))
    wt = (torch.rand(o, c, k, k, generator=g) * 2 - 1) / (c * k * k) ** 0.5
    b = (torch.rand(o, generator=g) * 2 - 1) * 0.05
    xs = ws = 1.0
    if dtype == DType.HALF:
        t = [v.half() for v in (x, off, msk, wt, b)]
        ydt = torch.float16
    else:
        xq, xs = quantize_sym(x)
        wq, ws = quantize_sym(wt)
        t = [xq, off, msk, wq, b]
        ydt = torch.float32
    t = [v.to(DEV).contiguous() for v in t]
    desc = capi.make_desc(n, c, h, w, o, k, s, p, d, dg, dtype)
    return desc, t, (n, o, ho, wo), ydt, xs, ws


def _reference(desc, t, oshape, ydt, xs, ws, stream):
    y = torch.empty(oshape, dtype=ydt, device=DEV)
    wsp = torch.empty(capi.workspace_size(desc), dtype=torch.uint8, device=DEV)
    st = capi.forward_raw(desc, *[v.data_ptr() for v in t], y.data_ptr(), wsp.data_ptr(),
                          wsp.numel(), xs, ws, stream)
    assert st == Status.OK
    return y


def test_static_scratch_matches_forward_on_two_calls_in_a_row():
    stream = torch.cuda.current_stream().cuda_stream
    cases = [
        _inputs(2, 64, 24, 20, 96, 3, 1, 1, 1, 1, DType.HALF, seed=11),
        _inputs(3, 32, 17, 15, 40, 3, 2, 2, 2, 2, DType.INT8, seed=12),
    ]
    refs = [_reference(*c[:5], c[5], stream) for c in cases]
    outs = []
    for desc, t, oshape, ydt, xs, ws in cases:  # two calls in a row, one shared buffer
        assert capi.workspace_size(desc) <= capi.STATIC_SCRATCH_BYTES
        y = torch.full(oshape, float("nan"), dtype=ydt, device=DEV)
        st = capi.forward_static_scratch_raw(desc, *[v.data_ptr() for v in t], y.data_ptr(),
                                             xs, ws, stream)
        assert st == Status.OK, capi.status_string(st)
        outs.append(y)
    torch.cuda.synchronize()
    y16, r16 = outs[0].double(), refs[0].double()
    assert torch.isfinite(y16).all()
    assert float((y16 - r16).abs().sum() / r16.abs().sum()) <= 1e-3
    y8, r8 = outs[1].cpu().numpy().astype(np.float64), refs[1].cpu().numpy().astype(np.float64)
    bound = 1e-6 * (np.abs(r8) + 1.0)
    assert np.all(np.abs(y8 - r8) <= bound)
    assert capi.read_static_scratch_error(stream) == 0
    # the same outputs against the oracle
    d16, t16 = cases[0][0], [v.float().cpu().numpy() for v in cases[0][1]]
    ref16 = oracle.forward_ref(*t16, d16.stride, d16.padding, d16.dilation,
                               d16.deformable_groups, precision="fp16")
    assert float(np.abs(y16.cpu().numpy() - ref16).sum() / np.abs(ref16).sum()) <= 1e-3
    d8, t8 = cases[1][0], [v.cpu().numpy() for v in cases[1][1]]
    xs8, ws8 = cases[1][4], cases[1][5]
    yx, acc = oracle.forward_i8_exact(t8[0], t8[1], t8[2], t8[3], t8[4], xs8, ws8, d8.stride,
                                      d8.padding, d8.dilation, d8.deformable_groups)
    s = float(np.float32(xs8) * np.float32(ws8))
    denom = np.abs(acc.astype(np.float64) * s) + np.abs(t8[4]).reshape(1, -1, 1, 1)
    assert np.all(np.abs(y8 - yx) <= 1e-6 * denom + 1e-30)


def test_static_scratch_rejects_oversized_problem():
    desc = capi.make_desc(64, 256, 64, 64, 256, dtype=DType.HALF)
    assert capi.workspace_size(desc) > capi.STATIC_SCRATCH_BYTES
    y = torch.full((1,), 3.0, device=DEV)
    st = capi.forward_static_scratch_raw(desc, 256, 256, 256, 256, 256, y.data_ptr())
    assert st == Status.ERR_SCRATCH_LIMIT
    torch.cuda.synchronize()
    assert float(y.item()) == 3.0
