"""The DCNv2 block with its offset / mask head (dcnv2_forward_with_head) against the PyTorch
composition the reference's detector runs (python/detector.py:44,50-52; the same split in
python/01_oracle_and_export.py:46-48): om = conv2d(x, head_weight, head_bias, padding=(K-1)//2),
offset = om[:, :2*dg*K*K], mask = sigmoid(om[:, 2*dg*K*K:]), then the deformable layer.

Tolerances:
  offset      |off - off_ref| <= 1e-3 * (1 + |off_ref|)   (fp32 accumulation, one fp16 rounding)
  mask        |m - m_ref| <= 1e-3                          (values in (0, 1), one fp16 rounding)
  y           mean relative error <= 1e-3 against the oracle's fp16 layer evaluated on the
              head's own offset and mask, and <= 2e-3 against torchvision's fp64 layer on the
              fp64 head outputs (the offsets differ by their fp16 rounding)
"""
import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

from dcnv2_b200 import capi, dcnv2_forward_with_head  # noqa: E402
from dcnv2_b200 import workloads as wl  # noqa: E402

DEV = "cuda:0"


def composition(x, hw, hb, dg, K):
    """fp64 PyTorch head on the fp16-rounded operands."""
    om = torch.nn.functional.conv2d(x.double(), hw.double(), hb.double(), padding=(K - 1) // 2)
    n_off = 2 * dg * K * K
    return om[:, :n_off], torch.sigmoid(om[:, n_off:])


def mean_rel(y, ref):
    return float(np.abs(y.astype(np.float64) - ref).sum() / np.abs(ref).sum())


@pytest.mark.parametrize("n,c,o,h,w,k,dg,picks", [
    (2, 64, 48, 24, 24, 3, 1, (0, 1)),        # W = 24 < tile width 32: columns past W discarded
    (3, 128, 64, 19, 37, 3, 2, (0, 2)),       # two groups, odd sizes, tiles of 64 x 2
    (1, 32, 40, 9, 150, 3, 1, (0,)),          # W > 128: tiles of one row
    (2, 64, 64, 16, 16, 5, 1, (0, 1)),        # 5 x 5 head and layer (padding 2)
    (64, 256, 256, 64, 64, 3, 1, (0, 63)),    # the fp16 workload's layer, whole batch
])
def test_layer_with_head_matches_composition(n, c, o, h, w, k, dg, picks):
    L = wl.Layer(n, c, h, w, o, k, 1, (k - 1) // 2, 1, dg)
    inp = wl.make_layer_inputs(L, "fp16", 0.1, 3.0, 0.5, seed=n + c)
    hw32, hb32 = wl.head_inputs(L, offset_std=0.4 if n < 64 else 0.1, seed=c)
    x, hw, hb = inp.x, hw32.half(), hb32.half()
    y, off, msk = dcnv2_forward_with_head(x.to(DEV), hw.to(DEV), hb.to(DEV),
                                          inp.weight.to(DEV), inp.bias.to(DEV),
                                          deformable_groups=dg, return_offsets=True)
    torch.cuda.synchronize()
    off, msk, y = off.cpu(), msk.cpu(), y.float().cpu().numpy()
    for i in picks:
        off_r, msk_r = composition(x[i:i + 1], hw, hb, dg, k)
        d_off = (off[i:i + 1].double() - off_r).abs()
        assert bool((d_off <= 1e-3 * (1 + off_r.abs())).all()), float(d_off.max())
        assert float((msk[i:i + 1].double() - msk_r).abs().max()) <= 1e-3
        # the layer on the head's own outputs: the oracle's fp16 path
        a = (1, (k - 1) // 2, 1, dg)
        ref = oracle.forward_ref(x[i:i + 1].float().numpy(), off[i:i + 1].float().numpy(),
                                 msk[i:i + 1].float().numpy(), inp.weight.float().numpy(),
                                 inp.bias.float().numpy(), *a, precision="fp16")
        assert mean_rel(y[i:i + 1], ref) <= 1e-3
        if n < 64:  # the whole composition in fp64 (torchvision), small cases
            tv = pytest.importorskip("torchvision.ops")
            yt = tv.deform_conv2d(x[i:i + 1].double(), off_r, inp.weight.double(),
                                  inp.bias.double(), padding=(k - 1) // 2, mask=msk_r).numpy()
            assert mean_rel(y[i:i + 1], yt) <= 2e-3


def test_layer_with_head_keeps_outputs_in_workspace_and_matches_two_step_call():
    """Without output buffers the head's offset / mask stay in the workspace; the result equals,
    bit for bit, dcnv2_forward on the offsets and mask the head wrote."""
    from dcnv2_b200 import dcnv2_forward
    L = wl.Layer(4, 64, 20, 20, 64)
    inp = wl.make_layer_inputs(L, "fp16", 0.1, 3.0, 0.5, seed=3).to(DEV)
    hw32, hb32 = wl.head_inputs(L, offset_std=0.5, seed=3)
    hw, hb = hw32.half().to(DEV), hb32.half().to(DEV)
    y1 = dcnv2_forward_with_head(inp.x, hw, hb, inp.weight, inp.bias)
    y2, off, msk = dcnv2_forward_with_head(inp.x, hw, hb, inp.weight, inp.bias,
                                           return_offsets=True)
    y3 = dcnv2_forward(inp.x, off, msk, inp.weight, inp.bias)
    torch.cuda.synchronize()
    assert torch.equal(y1, y2) and torch.equal(y2, y3)
