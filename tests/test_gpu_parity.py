"""Parity of the sm_100a kernels (through the C ABI) with the oracle, the reference's own GPU
path and torchvision.

Tolerances (stated per precision):
  fp32 (fused, fp32-exact)    max |y - y_ref| <= 1e-5 (absolute, outputs O(0.1-1))
  fp32 3xTF32 tensor cores    max |y - y_ref| <= 2e-4 * max(1, max|y_ref|)  (opt-in mode)
  fp32 single-pass TF32       max |y - y_ref| <= 2e-2 * max|y_ref|   (opt-in mode)
  fp16                        mean relative error sum|y - y_ref| / sum|y_ref| <= 1e-3 against
                              the reference fp16 path (fp16 columns, fp32 accumulation)
  int8                        identical quantised operands; |y - y_exact| <= 1e-6 *
                              (|acc * s| + |b|) against the exact int32-domain result
"""
import glob
import os

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

from dcnv2_b200 import DCNv2Error, Math, Status, dcnv2_forward  # noqa: E402
from dcnv2_b200 import capi  # noqa: E402
from dcnv2_b200.workloads import quantize_sym  # noqa: E402

DEV = "cuda:0"
FP32_TOL = 1e-5
TF32X3_REL = 2e-4
FP16_MEAN_REL = 1e-3
INT8_REL = 1e-6


def load(name):
    d = dict(np.load(os.path.join(os.path.dirname(__file__), "golden", name)))
    for k in ("stride", "padding", "dilation", "groups"):
        d[k] = int(d[k])
    return d


def attrs(fx):
    return dict(stride=fx["stride"], padding=fx["padding"], dilation=fx["dilation"],
                deformable_groups=fx["groups"])


def oattrs(fx):
    return (fx["stride"], fx["padding"], fx["dilation"], fx["groups"])


def cuda(a, dtype):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV).to(dtype).contiguous()


def run_fp32(fx, math=Math.DEFAULT):
    t = [cuda(fx[k], torch.float32) for k in ("x", "offset", "mask", "weight", "bias")]
    y = dcnv2_forward(*t, math=math, **attrs(fx))
    torch.cuda.synchronize()
    return y.cpu().numpy()


def run_fp16(fx, math=Math.DEFAULT):
    t = [cuda(fx[k], torch.float16) for k in ("x", "offset", "mask", "weight", "bias")]
    y = dcnv2_forward(*t, math=math, **attrs(fx))
    torch.cuda.synchronize()
    return y.float().cpu().numpy()


def half_inputs(fx):
    return {k: fx[k].astype(np.float16).astype(np.float32) for k in
            ("x", "offset", "mask", "weight", "bias")}


def quantized(fx):
    xq, xs = quantize_sym(torch.from_numpy(fx["x"]))
    wq, ws = quantize_sym(torch.from_numpy(fx["weight"]))
    return xq.numpy(), xs, wq.numpy(), ws


def run_int8(fx, xq, xs, wq, ws, math=Math.DEFAULT):
    y = dcnv2_forward(cuda(xq, torch.int8), cuda(fx["offset"], torch.float32),
                      cuda(fx["mask"], torch.float32), cuda(wq, torch.int8),
                      cuda(fx["bias"], torch.float32), x_scale=xs, w_scale=ws, math=math,
                      **attrs(fx))
    torch.cuda.synchronize()
    return y.cpu().numpy()


def mean_rel(y, ref):
    return float(np.abs(y.astype(np.float64) - ref).sum() / np.abs(ref).sum())


def check_int8(fx, y, xq, xs, wq, ws):
    yx, acc = oracle.forward_i8_exact(xq, fx["offset"], fx["mask"], wq, fx["bias"], xs, ws,
                                      *oattrs(fx))
    s = float(np.float32(xs) * np.float32(ws))
    denom = np.abs(acc.astype(np.float64) * s) + np.abs(fx["bias"]).reshape(1, -1, 1, 1)
    err = np.abs(y.astype(np.float64) - yx)
    assert np.all(err <= INT8_REL * denom + 1e-30), float((err / (denom + 1e-30)).max())


ALL_FIXTURES = ["kat_16c_32.npz"] + sorted(os.path.basename(p) for p in glob.glob(
    os.path.join(os.path.dirname(__file__), "golden", "tv_*.npz")))


@pytest.mark.parametrize("name", ALL_FIXTURES)
def test_fp32_golden(name):
    fx = load(name)
    y = run_fp32(fx)
    assert np.abs(y - fx["y"]).max() <= FP32_TOL


@pytest.mark.parametrize("name", ALL_FIXTURES)
def test_fp16_golden(name):
    fx = load(name)
    h = half_inputs(fx)
    ref = oracle.forward_ref(h["x"], h["offset"], h["mask"], h["weight"], h["bias"], *oattrs(fx),
                             precision="fp16")
    for math in (Math.DEFAULT, Math.PRECISE):
        y = run_fp16(fx, math)
        assert mean_rel(y, ref) <= FP16_MEAN_REL, (math, mean_rel(y, ref))


@pytest.mark.parametrize("name", ALL_FIXTURES)
def test_int8_golden(name):
    fx = load(name)
    xq, xs, wq, ws = quantized(fx)
    y = run_int8(fx, xq, xs, wq, ws)
    check_int8(fx, y, xq, xs, wq, ws)


@pytest.mark.parametrize("name", ["kat_16c_32.npz", "tv_oob.npz", "tv_n2_dg2_s2.npz",
                                  "tv_d2_p2_dg8.npz"])
def test_int8_precise_is_the_reference_rounding_rule(name):
    """int8 with DCNV2_MATH_PRECISE: each column is clamp(rint(m * bilinear(x_q)), -127, 127)
    in the reference's fp32 order (src/dcn_kernel.cu:19-30, :234) — the oracle's "rint" rule —
    so the integer accumulators match it exactly (|y - y_exact| <= 1e-6 * (|acc * s| + |b|))."""
    fx = load(name)
    xq, xs, wq, ws = quantized(fx)
    y = run_int8(fx, xq, xs, wq, ws, Math.PRECISE)
    n, o, ho, wo = y.shape
    yx, acc = oracle.forward_i8_exact_band(xq, fx["offset"], fx["mask"], wq, fx["bias"], xs, ws,
                                           0, ho * wo, *oattrs(fx), rule="rint")
    s = float(np.float32(xs) * np.float32(ws))
    denom = np.abs(acc.astype(np.float64) * s) + np.abs(fx["bias"]).reshape(1, -1, 1)
    err = np.abs(y.reshape(n, o, -1).astype(np.float64) - yx)
    assert np.all(err <= INT8_REL * denom + 1e-30), float((err / (denom + 1e-30)).max())


@pytest.mark.parametrize("name", ["kat_16c_32.npz", "tv_n2_dg2_s2.npz", "tv_odd.npz"])
def test_simt_path_matches(name):
    fx = load(name)
    assert np.abs(run_fp32(fx, Math.SIMT) - fx["y"]).max() <= FP32_TOL
    xq, xs, wq, ws = quantized(fx)
    check_int8(fx, run_int8(fx, xq, xs, wq, ws, Math.SIMT), xq, xs, wq, ws)
    h = half_inputs(fx)
    ref = oracle.forward_ref(h["x"], h["offset"], h["mask"], h["weight"], h["bias"], *oattrs(fx),
                             precision="fp16")
    assert mean_rel(run_fp16(fx, Math.SIMT), ref) <= FP16_MEAN_REL


@pytest.mark.parametrize("name", ["kat_16c_32.npz", "tv_d2_p2_dg8.npz", "tv_odd.npz"])
def test_tf32x3_tensor_core_bound(name):
    fx = load(name)
    y = run_fp32(fx, Math.TF32X3)
    assert np.abs(y - fx["y"]).max() <= TF32X3_REL * max(1.0, np.abs(fx["y"]).max())


def test_tf32_single_pass_reported_separately():
    fx = load("kat_16c_32.npz")
    y = run_fp32(fx, Math.TF32)
    assert np.abs(y - fx["y"]).max() <= 2e-2 * np.abs(fx["y"]).max()


def random_case(n, c, o, h, w, k=3, s=1, p=1, d=1, dg=1, ostd=0.5, outl=0.0, seed=0):
    g = np.random.default_rng(seed)
    ho = (h + 2 * p - d * (k - 1) - 1) // s + 1
    wo = (w + 2 * p - d * (k - 1) - 1) // s + 1
    off = (g.standard_normal((n, 2 * dg * k * k, ho, wo)) * ostd).astype(np.float32)
    if outl:
        sel = g.random(off.shape) < outl
        off[sel] = np.sign(g.standard_normal(sel.sum())) * 70.0
    return dict(
        x=g.standard_normal((n, c, h, w)).astype(np.float32),
        offset=off,
        mask=(1 / (1 + np.exp(-g.standard_normal((n, dg * k * k, ho, wo))))).astype(np.float32),
        weight=((g.random((o, c, k, k)) * 2 - 1) / np.sqrt(c * k * k)).astype(np.float32),
        bias=((g.random(o) * 2 - 1) * 0.05).astype(np.float32),
        stride=s, padding=p, dilation=d, groups=dg)


SHAPES = {
    "c256_o256_hw64_n2": dict(n=2, c=256, o=256, h=64, w=64, ostd=0.1),
    "c256_o256_oob": dict(n=1, c=256, o=256, h=32, w=48, ostd=0.5, outl=0.05),
    "c64_o320": dict(n=2, c=64, o=320, h=20, w=18),
    "c128_o512_dg8_d2": dict(n=1, c=128, o=512, h=24, w=24, p=2, d=2, dg=8, ostd=2.0),
    "c32_o24_s2": dict(n=3, c=32, o=24, h=33, w=29, s=2),
    "c512_o64_p4096": dict(n=1, c=512, o=64, h=64, w=64),
    "c16_o1200": dict(n=1, c=16, o=1200, h=12, w=12),
}


@pytest.mark.parametrize("shape", sorted(SHAPES))
def test_random_shapes_all_precisions(shape):
    fx = random_case(**SHAPES[shape])
    ref32 = oracle.forward_ref(fx["x"], fx["offset"], fx["mask"], fx["weight"], fx["bias"],
                               *oattrs(fx))
    assert np.abs(run_fp32(fx) - ref32).max() <= FP32_TOL
    assert np.abs(run_fp32(fx, Math.TF32X3) - ref32).max() <= \
        TF32X3_REL * max(1.0, np.abs(ref32).max())
    h = half_inputs(fx)
    ref16 = oracle.forward_ref(h["x"], h["offset"], h["mask"], h["weight"], h["bias"],
                               *oattrs(fx), precision="fp16")
    assert mean_rel(run_fp16(fx), ref16) <= FP16_MEAN_REL
    xq, xs, wq, ws = quantized(fx)
    check_int8(fx, run_int8(fx, xq, xs, wq, ws), xq, xs, wq, ws)


@pytest.mark.skipif(not oracle.ref_gpu_available(), reason="reference GPU build not present")
@pytest.mark.parametrize("name", ["kat_16c_32.npz", "npref_n3.npz", "npref_n2_s2_d2.npz"])
def test_against_reference_gpu_path(name):
    """Same inputs through the reference's own im2col + cuBLAS path on this GPU."""
    fx = load(name)
    t32 = [cuda(fx[k], torch.float32) for k in ("x", "offset", "mask", "weight", "bias")]
    yr = oracle.ref_gpu_forward(*t32, stride=fx["stride"], padding=fx["padding"],
                                dilation=fx["dilation"]).cpu().numpy()
    assert np.abs(run_fp32(fx) - yr).max() <= FP32_TOL
    t16 = [cuda(fx[k], torch.float16) for k in ("x", "offset", "mask", "weight", "bias")]
    yr16 = oracle.ref_gpu_forward(*t16, stride=fx["stride"], padding=fx["padding"],
                                  dilation=fx["dilation"]).float().cpu().numpy()
    assert mean_rel(run_fp16(fx), yr16) <= FP16_MEAN_REL
    xq, xs, wq, ws = quantized(fx)
    yr8 = oracle.ref_gpu_forward(cuda(xq, torch.int8), t32[1], t32[2], cuda(wq, torch.int8),
                                 t32[4], stride=fx["stride"], padding=fx["padding"],
                                 dilation=fx["dilation"], x_scale=xs, w_scale=ws).cpu().numpy()
    y8 = run_int8(fx, xq, xs, wq, ws)
    # int8 column rule: |c - m*bilinear(x)| <= 0.5 + 2^-7 per column value
    bound = (0.5 + 2.0 ** -7) * xs * ws * np.abs(wq).reshape(wq.shape[0], -1).sum(1).reshape(
        1, -1, 1, 1)
    assert np.all(np.abs(y8 - yr8) <= bound * 1.001 + 1e-5)


def test_torchvision_cuda_fp32():
    tv = pytest.importorskip("torchvision.ops")
    fx = random_case(n=2, c=64, o=64, h=24, w=24, dg=2, ostd=1.0, outl=0.05, seed=7)
    t = [cuda(fx[k], torch.float32) for k in ("x", "offset", "mask", "weight", "bias")]
    yt = tv.deform_conv2d(t[0].double(), t[1].double(), t[3].double(), t[4].double(),
                          padding=(1, 1), mask=t[2].double()).cpu().numpy()
    assert np.abs(run_fp32(fx) - yt).max() <= FP32_TOL


def test_device_error_word_clear_and_batch_consistency():
    fx = random_case(n=4, c=64, o=64, h=16, w=16, seed=3)
    t = [cuda(fx[k], torch.float16) for k in ("x", "offset", "mask", "weight", "bias")]
    desc = capi.make_desc(4, 64, 16, 16, 64, dtype=capi.DType.HALF)
    ws = torch.empty(capi.workspace_size(desc), dtype=torch.uint8, device=DEV)
    y = dcnv2_forward(*t, workspace=ws)
    assert capi.read_device_error(ws.data_ptr()) == 0
    # image n of a batched call equals a batch-1 call on image n
    for n in range(4):
        yn = dcnv2_forward(*(t[0][n:n + 1].contiguous(), t[1][n:n + 1].contiguous(),
                             t[2][n:n + 1].contiguous(), t[3], t[4]))
        torch.cuda.synchronize()
        assert torch.equal(yn[0], y[n])


def test_plugin_enqueue_matches_forward():
    from dcnv2_b200 import DCNv2Creator, tensor_desc
    fx = load("tv_n2_dg2_s2.npz")
    plug = DCNv2Creator().create_plugin("DCNv2", {"stride": 2, "padding": 1, "dilation": 1,
                                                  "kernel": 3, "deformable_groups": 2})
    t = [cuda(fx[k], torch.float16) for k in ("x", "offset", "mask", "weight", "bias")]
    (oshape,) = plug.get_output_shapes(t[0].shape, t[3].shape)
    y = torch.empty(oshape, dtype=torch.float16, device=DEV)
    ind = [tensor_desc(v.shape, capi.DType.HALF) for v in t]
    outd = [tensor_desc(oshape, capi.DType.HALF)]
    wsz = plug.get_workspace_size(ind, outd)
    ws = torch.empty(wsz, dtype=torch.uint8, device=DEV)
    rc = plug.clone().enqueue(ind, outd, [v.data_ptr() for v in t], [y.data_ptr()],
                              ws.data_ptr(), wsz, torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    ref = dcnv2_forward(*t, **attrs(fx))
    torch.cuda.synchronize()
    assert torch.equal(y, ref)


def test_short_workspace_is_rejected_without_launch():
    fx = load("kat_16c_32.npz")
    t = [cuda(fx[k], torch.float32) for k in ("x", "offset", "mask", "weight", "bias")]
    y = torch.full((1, 16, 32, 32), 7.0, device=DEV)
    desc = capi.make_desc(1, 16, 32, 32, 16, dtype=capi.DType.FLOAT)
    need = capi.workspace_size(desc)
    small = torch.empty(need - 1, dtype=torch.uint8, device=DEV)
    st = capi.forward_raw(desc, *[v.data_ptr() for v in t], y.data_ptr(), small.data_ptr(),
                          small.numel())
    assert st == Status.ERR_WORKSPACE
    torch.cuda.synchronize()
    assert bool((y == 7.0).all())  # nothing was launched


def test_device_code_is_sm100():
    """The runtime reports the library's device code as built for sm_100."""
    assert capi.binary_arch() == 100


def test_timeout_selftest_keeps_context_usable():
    st, code = capi.timeout_selftest(2000)  # a wait that nothing completes, 2 ms limit
    assert st == Status.ERR_DEVICE_TIMEOUT and code != 0
    fx = load("kat_16c_32.npz")
    assert np.abs(run_fp32(fx) - fx["y"]).max() <= FP32_TOL


PAIR_SHAPES = {
    # P = 33*29 = 957 (not a multiple of 256: the last pair tile's second CTA has no pixels)
    "c32_o24_s2": dict(n=3, c=32, o=24, h=33, w=29, s=2),
    "c128_o512_dg8_d2": dict(n=1, c=128, o=512, h=24, w=24, p=2, d=2, dg=8, ostd=2.0),
    "c256_o256_oob": dict(n=1, c=256, o=256, h=32, w=48, ostd=0.5, outl=0.05),
    "c64_o48_hw40": dict(n=2, c=64, o=48, h=40, w=40),
}


@pytest.fixture
def kernel_override():
    """Sets the library's kernel selection for one test and restores automatic selection."""
    yield capi.set_kernel_override
    capi.set_kernel_override(capi.Kernel.AUTO, capi.Pair.AUTO)


@pytest.mark.parametrize("shape", sorted(PAIR_SHAPES))
def test_cta_pair_and_single_cta_paths_agree(shape, kernel_override):
    """The shared-memory A kernel runs fp16 / int8 tiles on one CTA (128 pixels) or on a CTA
    pair (cta_group::2, 256 pixels; automatic above 256 output channels), forced here both ways.
    Both meet the stated bounds and agree with each other."""
    fx = random_case(**PAIR_SHAPES[shape])
    h = half_inputs(fx)
    ref16 = oracle.forward_ref(h["x"], h["offset"], h["mask"], h["weight"], h["bias"],
                               *oattrs(fx), precision="fp16")
    xq, xs, wq, ws = quantized(fx)
    kernel_override(capi.Kernel.SMEM, capi.Pair.PAIRS)
    y16_pair = run_fp16(fx)
    y8_pair = run_int8(fx, xq, xs, wq, ws)
    kernel_override(capi.Kernel.SMEM, capi.Pair.SINGLE)
    y16_one = run_fp16(fx)
    y8_one = run_int8(fx, xq, xs, wq, ws)
    for y in (y16_pair, y16_one):
        assert mean_rel(y, ref16) <= FP16_MEAN_REL
    for y in (y8_pair, y8_one):
        check_int8(fx, y, xq, xs, wq, ws)
    # same A and B operands and K order: the two paths differ at most by fp32 accumulation order
    assert mean_rel(y16_pair, y16_one) <= 1e-4
    np.testing.assert_allclose(y8_pair, y8_one, rtol=1e-6, atol=1e-6)


TA_SHAPES = {
    # identity-like offsets: every corner in the x window (fp16 3x3 fast path)
    "c256_o256_hw64_idlike": dict(n=2, c=256, o=256, h=64, w=64, ostd=0.1),
    # more tiles than SMs: CTAs take two tiles, window buffers are reused across tiles
    "c128_o64_n10_multitile": dict(n=10, c=128, o=64, h=48, w=48, ostd=0.3),
    # out-of-image offsets: corners outside the window come from global memory
    "c256_o256_oob": dict(n=1, c=256, o=256, h=32, w=48, ostd=0.5, outl=0.05),
    # partial channel block (16 of 64 / 128 channels), 5x5 taps
    "c16_o24_k5": dict(n=2, c=16, o=24, h=19, w=23, k=5, p=2),
    "c64_o48_k1": dict(n=2, c=64, o=48, h=20, w=20, k=1, p=0),
    # two output-channel chunks of 256, groups, dilation 2
    "c128_o512_dg8_d2": dict(n=1, c=128, o=512, h=24, w=24, p=2, d=2, dg=8, ostd=2.0),
    # odd pixel count (single-pixel epilogue stores), stride 2
    "c32_o24_s2": dict(n=3, c=32, o=24, h=33, w=29, s=2),
    # W > 256: no x window, every corner from global memory
    "c16_o32_w300": dict(n=1, c=16, o=32, h=5, w=300),
    # no window, int8 groups of 64 channels: the shared-memory A kernel packs two taps per
    # K-block (the TMEM-A kernel does not); both give the same integers
    "c128_o48_dg2_w300": dict(n=2, c=128, o=48, h=5, w=300, dg=2, ostd=1.5),
}


@pytest.mark.parametrize("pair", [False, True], ids=["cta", "pair"])
@pytest.mark.parametrize("shape", sorted(TA_SHAPES))
def test_tmem_a_kernel_matches_smem_a_kernel(shape, pair, kernel_override):
    """fp16 / int8 default to the kernel with the A operand in tensor memory (the "ta" override
    also forces it for > 256 output channels); the "smem" override selects the shared-memory A
    kernel (here with CTA pairs forced on or off; the TMEM-A kernel always runs one CTA per tile).
    Both meet the stated bounds against the oracle and agree with each other (same A values,
    same K order)."""
    fx = random_case(**TA_SHAPES[shape])
    h = half_inputs(fx)
    ref16 = oracle.forward_ref(h["x"], h["offset"], h["mask"], h["weight"], h["bias"],
                               *oattrs(fx), precision="fp16")
    xq, xs, wq, ws = quantized(fx)
    out = {}
    for name, kern in (("smem", capi.Kernel.SMEM), ("ta", capi.Kernel.TA)):
        kernel_override(kern, capi.Pair.PAIRS if pair else capi.Pair.SINGLE)
        out[name] = (run_fp16(fx), run_fp16(fx, Math.PRECISE), run_int8(fx, xq, xs, wq, ws))
    for kern, (y16, y16p, y8) in out.items():
        assert mean_rel(y16, ref16) <= FP16_MEAN_REL, kern
        assert mean_rel(y16p, ref16) <= FP16_MEAN_REL, kern
        check_int8(fx, y8, xq, xs, wq, ws)
    assert mean_rel(out["ta"][0], out["smem"][0]) <= 1e-4
    assert mean_rel(out["ta"][1], out["smem"][1]) <= 1e-4
    np.testing.assert_allclose(out["ta"][2], out["smem"][2], rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("chunk", [0, 1, 2, 5])
def test_host_buffer_forward_matches_device_forward(chunk):
    """dcnv2_forward_host (x, offset, mask, y on the host; uploads, forwards and downloads of
    image chunks overlapped) gives bit-identical results to dcnv2_forward, for every precision
    and for chunk sizes that leave a ragged last chunk."""
    from dcnv2_b200 import dcnv2_forward_host
    fx = random_case(n=5, c=64, o=48, h=20, w=18, ostd=0.6, outl=0.02, seed=11)
    cases = [(torch.float32, {}), (torch.float16, {})]
    xq, xs, wq, ws = quantized(fx)
    for dt, kw in cases:
        host = [torch.from_numpy(fx[k]).to(dt).contiguous().pin_memory()
                for k in ("x", "offset", "mask")]
        w = cuda(fx["weight"], dt)
        b = cuda(fx["bias"], dt)
        ref = dcnv2_forward(*[h.to(DEV) for h in host], w, b, **attrs(fx))
        y = dcnv2_forward_host(*host, w, b, images_per_chunk=chunk, **attrs(fx))
        assert torch.equal(y, ref.cpu())
    host = [torch.from_numpy(np.ascontiguousarray(xq)).pin_memory(),
            torch.from_numpy(fx["offset"]).pin_memory(), torch.from_numpy(fx["mask"]).pin_memory()]
    w8, b32 = cuda(wq, torch.int8), cuda(fx["bias"], torch.float32)
    ref8 = dcnv2_forward(*[h.to(DEV) for h in host], w8, b32, x_scale=xs, w_scale=ws, **attrs(fx))
    y8 = dcnv2_forward_host(*host, w8, b32, x_scale=xs, w_scale=ws, images_per_chunk=chunk,
                            **attrs(fx))
    assert torch.equal(y8, ref8.cpu())


@pytest.mark.parametrize("chunk", [4, 8])
def test_host_buffer_forward_short_edge_chunks(chunk):
    """A batch of more than two chunks runs with a first and a last chunk of a quarter of the
    others (20 images in chunks of 4: 1, 4, 4, 4, 4, 2, 1; of 8: 2, 8, 8, 2); the result stays
    bit-identical to dcnv2_forward."""
    from dcnv2_b200 import dcnv2_forward_host
    fx = random_case(n=20, c=32, o=32, h=12, w=12, ostd=0.6, outl=0.02, seed=13)
    host = [torch.from_numpy(fx[k]).to(torch.float16).contiguous().pin_memory()
            for k in ("x", "offset", "mask")]
    w = cuda(fx["weight"], torch.float16)
    b = cuda(fx["bias"], torch.float16)
    ref = dcnv2_forward(*[h.to(DEV) for h in host], w, b, **attrs(fx))
    y = dcnv2_forward_host(*host, w, b, images_per_chunk=chunk, **attrs(fx))
    assert torch.equal(y, ref.cpu())


def test_levels_runner_graph_matches_per_level_forward():
    """The FPN levels run as one CUDA graph with one stream per level give the same outputs,
    bit for bit, as one dcnv2_forward per level."""
    from dcnv2_b200.levels import LevelsRunner
    levels = []
    for i, s in enumerate((32, 16, 8, 4)):
        fx = random_case(n=3, c=64, o=64, h=s, w=s, ostd=0.3, seed=20 + i)
        levels.append({k: cuda(fx[k], torch.float16) for k in ("x", "offset", "mask", "weight",
                                                               "bias")})
    refs = [dcnv2_forward(lv["x"], lv["offset"], lv["mask"], lv["weight"], lv["bias"])
            for lv in levels]
    runner = LevelsRunner(levels)
    for _ in range(2):  # replay twice: outputs are rewritten, not accumulated
        outs = runner.run()
        torch.cuda.synchronize()
        for y, r in zip(outs, refs):
            assert torch.equal(y, r)
