"""Parity of the default dispatch on the benchmarked workloads themselves: the shapes, batch sizes
and input distributions that bench.py times (dcnv2_b200.workloads), checked against the oracle
on whole images (or on bands of output pixels where one image of the layer is too large for the
oracle to finish in seconds): the first, a middle and the last image of each batch.

Tolerances are those of test_gpu_parity.py:
  fp32   max |y - y_ref| <= 1e-5 against the oracle and against torchvision in float64
  fp16   mean relative error <= 1e-3 against the reference fp16 path (fp16 columns, fp32
         accumulation, the reference's two fp16 roundings of the output)
  int8   identical quantised operands; |y - y_exact| <= 1e-6 * (|acc * s| + |b|) against the
         exact int32-domain result
The reference's own load/run/compare tests (src/test_dcn_gemm.cu:28-72) are the model.
"""
import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

from dcnv2_b200 import capi, dcnv2_forward  # noqa: E402
from dcnv2_b200 import workloads as wl  # noqa: E402
from dcnv2_b200.capi import Math  # noqa: E402
from dcnv2_b200.shard import shard_range  # noqa: E402

DEV = "cuda:0"
FP32_TOL = 1e-5
FP16_MEAN_REL = 1e-3
INT8_REL = 1e-6


def attrs(L):
    return dict(stride=L.stride, padding=L.padding, dilation=L.dilation,
                deformable_groups=L.groups)


def oattrs(L):
    return (L.stride, L.padding, L.dilation, L.groups)


def run(inp, math=Math.DEFAULT):
    t = [v.to(DEV).contiguous() for v in inp.tensors()]
    y = dcnv2_forward(*t, x_scale=inp.x_scale, w_scale=inp.w_scale, math=math, **attrs(inp.layer))
    torch.cuda.synchronize()
    return y.float().cpu().numpy()


def desc_of(inp, math=Math.DEFAULT):
    L = inp.layer
    dt = {"fp32": capi.DType.FLOAT, "fp16": capi.DType.HALF, "int8": capi.DType.INT8}[inp.precision]
    return capi.make_desc(L.n, L.c, L.h, L.w, L.out_c, L.kernel, L.stride, L.padding,
                          L.dilation, L.groups, dt, math)


def picks(n):
    return sorted({0, n // 2, n - 1})


def bands(P, width):
    if P <= 3 * width:
        return [(0, P)]
    return [(0, width), (P // 2 - width // 2, P // 2 + width // 2), (P - width, P)]


def one(inp, i):
    """numpy float32 x / offset / mask of image i, shared weight and bias."""
    x, off, m, w, b = inp.tensors()
    return (x[i:i + 1].float().numpy(), off[i:i + 1].float().numpy(),
            m[i:i + 1].float().numpy(), w.float().numpy(), b.float().numpy())


def mean_rel(y, ref):
    return float(np.abs(y.astype(np.float64) - ref).sum() / np.abs(ref).sum())


def check_fp16_images(inp, ys, width=None):
    """ys: {math: y [N, O, Ho, Wo]} from the GPU; oracle fp16 reference per picked image/band."""
    L = inp.layer
    P = L.ho * L.wo
    for i in picks(L.n):
        x, off, m, w, b = one(inp, i)
        for p0, p1 in bands(P, width or P):
            ref = oracle.forward_ref_band(x, off, m, w, b, p0, p1, *oattrs(L), precision="fp16")
            for math, y in ys.items():
                got = y[i].reshape(L.out_c, P)[:, p0:p1]
                err = mean_rel(got, ref[0])
                assert err <= FP16_MEAN_REL, (math, i, p0, err)


def check_int8_images(inp, y, width=None):
    L = inp.layer
    P = L.ho * L.wo
    xq, off, m, wq, b = inp.tensors()
    s = float(np.float32(inp.x_scale) * np.float32(inp.w_scale))
    for i in picks(L.n):
        for p0, p1 in bands(P, width or P):
            yx, acc = oracle.forward_i8_exact_band(
                xq[i:i + 1].numpy(), off[i:i + 1].numpy(), m[i:i + 1].numpy(), wq.numpy(),
                b.numpy(), inp.x_scale, inp.w_scale, p0, p1, *oattrs(L))
            got = y[i].reshape(L.out_c, P)[:, p0:p1].astype(np.float64)
            denom = np.abs(acc[0].astype(np.float64) * s) + np.abs(b.numpy()).reshape(-1, 1)
            err = np.abs(got - yx[0])
            assert np.all(err <= INT8_REL * denom + 1e-30), (i, p0, float((err / denom).max()))


# ---------------------------------------------------------------- config 0: fp32, N=1
def test_fp32_n1_exact_shape_against_torchvision_and_oracle():
    """fp32 N=1 256->256 64x64 with ~5 % of the offsets at +-70 (out-of-image samples)."""
    tv = pytest.importorskip("torchvision.ops")
    inp = wl.workload("fp32_n1_256c_64", seed=0)
    assert capi.main_kernel(desc_of(inp)) == "dcnv2_f32_exact_kernel"
    y = run(inp)
    x, off, m, w, b = inp.tensors()
    yt = tv.deform_conv2d(x.double(), off.double(), w.double(), b.double(), padding=(1, 1),
                          mask=m.double()).numpy()
    assert np.abs(y - yt).max() <= FP32_TOL
    ref = oracle.forward_ref(*[t.numpy() for t in inp.tensors()], *oattrs(inp.layer))
    assert np.abs(y - ref).max() <= FP32_TOL


# ---------------------------------------------------------------- config 1: fp16, N=64
def test_headline_fp16_full_batch():
    """fp16 N=64 256->256 64x64 with identity-like offsets N(0, 0.1^2) and
    mask = sigmoid(N(3, 0.5^2)): the benchmarked batch, default and fp32-sampler modes."""
    inp = wl.workload("fp16_n64_256c_64", seed=0)
    assert capi.main_kernel(desc_of(inp)) == "dcnv2_fused_ta_kernel"
    ys = {m: run(inp, m) for m in (Math.DEFAULT, Math.PRECISE)}
    check_fp16_images(inp, ys)


# ---------------------------------------------------------------- config 2: int8, N=64
def test_int8_full_batch():
    inp = wl.workload("int8_n64_256c_64", seed=0)
    assert capi.main_kernel(desc_of(inp)) == "dcnv2_fused_ta_kernel"
    check_int8_images(inp, run(inp))


# ---------------------------------------------------------------- config 3: FPN levels, B=32
def test_fpn_levels_graph_against_oracle():
    """The five FPN levels (256 channels, 64x64 .. 4x4, B=32) as the benchmark runs them: one
    CUDA graph with one stream per level."""
    from dcnv2_b200.levels import LevelsRunner
    parts = wl.workload_parts("fpn_fp16_b32", seed=0)
    dev = [p.to(DEV) for p in parts]
    runner = LevelsRunner([dict(x=p.x, offset=p.offset, mask=p.mask, weight=p.weight,
                                bias=p.bias) for p in dev])
    outs = [y.float().cpu().numpy() for y in runner.run()]
    torch.cuda.synchronize()
    for p, y in zip(parts, outs):
        check_fp16_images(p, {Math.DEFAULT: y})


# ---------------------------------------------------------------- config 4: 512ch dg8 d2
@pytest.mark.parametrize("n", [1, 16])
def test_big_512c_128_dg8_fp16(n):
    """512->512, 128x128, dilation 2, padding 2, deformable_groups 8, offsets N(0, 2^2): the
    A-in-shared-memory kernel (512 output channels as two sub-MMAs), several channel blocks per
    group. N=16 is one GPU's share of the N=128 batch over 8 GPUs."""
    inp = wl.workload("big_512c_128_dg8", n=n, seed=0)
    assert capi.main_kernel(desc_of(inp)) == "dcnv2_fused_kernel"
    ys = {m: run(inp, m) for m in (Math.DEFAULT, Math.PRECISE)}
    check_fp16_images(inp, ys, width=512)


@pytest.mark.parametrize("n", [1, 16])
def test_big_512c_128_dg8_int8(n):
    inp = wl.workload("big_512c_128_dg8_int8", n=n, seed=0)
    assert capi.main_kernel(desc_of(inp)) == "dcnv2_fused_kernel"
    check_int8_images(inp, run(inp), width=512)


def test_big_layer_plan_at_small_size():
    """The same plan as the 512-channel layer (no x window at W=128, smem-A kernel, O=512,
    d2, dg8, several channel blocks) on a few rows, against the whole-image oracle."""
    L = wl.Layer(1, 512, 6, 128, 512, 3, 1, 2, 2, 8)
    for prec in ("fp16", "int8"):
        inp = wl.make_layer_inputs(L, prec, 2.0, 0.0, 1.0, seed=5)
        assert capi.main_kernel(desc_of(inp)) == "dcnv2_fused_kernel"
        if prec == "fp16":
            check_fp16_images(inp, {m: run(inp, m) for m in (Math.DEFAULT, Math.PRECISE)})
        else:
            check_int8_images(inp, run(inp))


# ---------------------------------------------------------------- the batch split
def test_batch_split_over_ranks_is_the_batch():
    """Each rank's slice (shard_range of the 64-image batch over 8 ranks) run on its own gives,
    bit for bit, the slice of the whole batch's forward."""
    inp = wl.workload("fp16_n64_256c_64", seed=0)
    full = run(inp)
    for r in range(8):
        a, b = shard_range(64, 8, r)
        assert np.array_equal(run(inp.images(a, b)), full[a:b])
