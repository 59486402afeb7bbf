"""Pins the CPU oracle (oracle/dcnv2_oracle.c) before anything is checked against it.

* the reference's known-answer case (python/01_oracle_and_export.py:51-70, y.sum = -30.9894 at
  src/test_dcn.cu:64, max|err| < 1e-3 at :66) through both the im2col path and the naive path;
* torchvision float64 answers on batch/groups/stride/dilation/out-of-image/odd-size cases;
* the reference's own numpy forward (python/dcn_ort_op.py:68-92) on batch > 1 cases;
* the INT8 quantiser (src/test_dcn_int8.cu:31-42) and the exact int32-domain INT8 definition.
"""
import glob
import os

import numpy as np
import pytest

import oracle


def load(golden_dir, name):
    d = dict(np.load(os.path.join(golden_dir, name)))
    for k in ("stride", "padding", "dilation", "groups"):
        d[k] = int(d[k])
    return d


def run_ref(fx, precision="fp32"):
    return oracle.forward_ref(fx["x"], fx["offset"], fx["mask"], fx["weight"], fx["bias"],
                              fx["stride"], fx["padding"], fx["dilation"], fx["groups"],
                              precision=precision)


def test_known_answer_sum(golden_dir):
    fx = load(golden_dir, "kat_16c_32.npz")
    y = run_ref(fx)
    assert abs(float(y.sum()) - (-30.9894)) < 5e-4
    assert np.abs(y - fx["y"]).max() < 1e-5  # reference tolerance 1e-3 (src/test_dcn.cu:66)


def test_known_answer_naive_path(golden_dir):
    fx = load(golden_dir, "kat_16c_32.npz")
    y = oracle.forward_direct(fx["x"], fx["offset"], fx["mask"], fx["weight"], fx["bias"])
    assert np.abs(y - fx["y"]).max() < 1e-5


@pytest.mark.parametrize("name", sorted(os.path.basename(p) for p in glob.glob(
    os.path.join(os.path.dirname(__file__), "golden", "tv_*.npz"))))
def test_torchvision_edge_cases(golden_dir, name):
    fx = load(golden_dir, name)
    y = run_ref(fx)
    scale = np.abs(fx["y"]).max()
    assert np.abs(y - fx["y"]).max() <= 2e-6 * max(1.0, scale)
    yd = oracle.forward_direct(fx["x"], fx["offset"], fx["mask"], fx["weight"], fx["bias"],
                               fx["stride"], fx["padding"], fx["dilation"], fx["groups"])
    assert np.abs(yd - fx["y"]).max() <= 2e-6 * max(1.0, scale)


@pytest.mark.parametrize("name", sorted(os.path.basename(p) for p in glob.glob(
    os.path.join(os.path.dirname(__file__), "golden", "npref_*.npz"))))
def test_reference_numpy_forward(golden_dir, name):
    fx = load(golden_dir, name)
    y = run_ref(fx)
    assert np.abs(y - fx["y"]).max() <= 1e-5


def test_fp16_path_rounding(golden_dir):
    fx = load(golden_dir, "kat_16c_32.npz")
    h = {k: fx[k].astype(np.float16).astype(np.float32) for k in ("x", "offset", "mask",
                                                                   "weight", "bias")}
    y16 = oracle.forward_ref(h["x"], h["offset"], h["mask"], h["weight"], h["bias"],
                             precision="fp16")
    # outputs are fp16 values
    assert np.array_equal(y16, y16.astype(np.float16).astype(np.float32))
    # reference FP16 tolerance: mean relative error < 2% (src/test_dcn_half_gemm.cu:80-83)
    rel = np.abs(y16 - fx["y"]).sum() / np.abs(fx["y"]).sum()
    assert rel < 2e-3


def test_quantizer_matches_reference_rule():
    rng = np.random.default_rng(0)
    v = rng.standard_normal(1000).astype(np.float32)
    v[3] = 0.5 * np.abs(v).max()  # exact ties go away from zero
    q, s = oracle.quantize_sym(v)
    assert s == np.float32(np.abs(v).max()) / np.float32(127)
    r = v / np.float32(s)
    expect = np.clip(np.sign(r) * np.floor(np.abs(r) + 0.5), -127, 127).astype(np.int8)
    assert np.array_equal(q, expect)
    q0, s0 = oracle.quantize_sym(np.zeros(4, np.float32))
    assert s0 == 1.0 and not q0.any()


def test_int8_exact_definition(golden_dir):
    fx = load(golden_dir, "kat_16c_32.npz")
    xq, xs = oracle.quantize_sym(fx["x"])
    wq, ws = oracle.quantize_sym(fx["weight"])
    y, acc, cols = oracle.forward_i8_exact(xq, fx["offset"], fx["mask"], wq, fx["bias"], xs, ws,
                                           want_cols=True)
    assert cols.min() >= -127 and cols.max() <= 127
    # acc is the exact integer product of the integer operands
    wmat = wq.reshape(wq.shape[0], -1).astype(np.int64)
    assert np.array_equal(acc[0].reshape(wq.shape[0], -1), wmat @ cols[0].astype(np.int64))
    # deviation from the reference INT8 path (fp32 columns) is bounded by the column rounding:
    # |y_exact - y_ref| <= (0.5 + 2^-7) * xs * ws * sum|w_q| (+ fp32 slack)
    yref = oracle.forward_i8_ref(xq, fx["offset"], fx["mask"], wq, fx["bias"], xs, ws)
    bound = I8_COL_DEV * xs * ws * np.abs(wq).reshape(wq.shape[0], -1).sum(1)
    dev = np.abs(y - yref).max(axis=(0, 2, 3))
    assert np.all(dev <= bound * 1.0001 + 1e-5)
    # and the INT8 result stays within the reference INT8 tolerance of the fp32 answer
    # (mean relative error < 10%, src/test_dcn_int8_gemm.cu:89)
    rel = np.abs(y - fx["y"]).sum() / np.abs(fx["y"]).sum()
    assert rel < 0.05


I8_COL_DEV = 0.5 + 2.0 ** -7  # |c - m*bilinear(x)| of the fixed-point int8 column rule


def i8_cols_numpy(xq, off, mask, stride=1, padding=1, dilation=1, k=3):
    """Independent numpy statement of the int8 column rule (one image, one group):
    m' = clip(m, 0, 1), a_k = m' * (fy * fx) in float32, w_k = min(rint(a_k * 2^16), 65535),
    c = floor((sum_k w_k x_k + 2^15) / 2^16). Returns int cols [C*k*k, Ho*Wo]."""
    C, H, W = xq.shape
    Ho = (H + 2 * padding - dilation * (k - 1) - 1) // stride + 1
    Wo = (W + 2 * padding - dilation * (k - 1) - 1) // stride + 1
    f32 = np.float32
    oh, ow = np.meshgrid(np.arange(Ho), np.arange(Wo), indexing="ij")
    cols = np.zeros((C, k * k, Ho * Wo), np.int64)
    for t in range(k * k):
        i, j = divmod(t, k)
        dh = off[2 * t].astype(f32)
        dw = off[2 * t + 1].astype(f32)
        m = np.nan_to_num(mask[t].astype(f32), nan=0.0).clip(0, 1).astype(f32)
        hf = (oh * stride - padding + i * dilation).astype(f32) + dh
        wf = (ow * stride - padding + j * dilation).astype(f32) + dw
        inside = ~((hf <= -1) | (hf >= H) | (wf <= -1) | (wf >= W))
        h0f, w0f = np.floor(hf), np.floor(wf)
        lh, lw = (hf - h0f).astype(f32), (wf - w0f).astype(f32)
        hh, hw = (f32(1) - lh).astype(f32), (f32(1) - lw).astype(f32)
        h0, w0 = h0f.astype(np.int64), w0f.astype(np.int64)
        s = np.full((C, Ho, Wo), 32768, np.int64)
        for dy, dx, fy, fx in ((0, 0, hh, hw), (0, 1, hh, lw), (1, 0, lh, hw), (1, 1, lh, lw)):
            hc, wc = h0 + dy, w0 + dx
            ok = inside & (hc >= 0) & (hc <= H - 1) & (wc >= 0) & (wc <= W - 1)
            a = (m * (fy * fx).astype(f32)).astype(f32)
            w = np.minimum(np.rint(a.astype(np.float64) * 65536.0), 65535).astype(np.int64)
            w = np.where(ok & (a > 0), w, 0)
            xv = xq[:, np.clip(hc, 0, H - 1), np.clip(wc, 0, W - 1)].astype(np.int64)
            s += w[None] * np.where(ok[None], xv, 0)
        cols[:, t] = np.floor_divide(s, 65536).reshape(C, -1)
    return cols.reshape(C * k * k, -1)


def test_int8_column_rule_matches_numpy_statement(golden_dir):
    fx = load(golden_dir, "tv_oob.npz")  # out-of-image offsets exercise the zero corners
    xq, xs = oracle.quantize_sym(fx["x"])
    wq, ws = oracle.quantize_sym(fx["weight"])
    mask = fx["mask"].copy()
    mask.reshape(-1)[::7] = 1.0   # weight 65536 -> 65535
    mask.reshape(-1)[3::11] = 1.7  # clipped to 1
    mask.reshape(-1)[5::13] = -0.3  # clipped to 0
    _, _, cols = oracle.forward_i8_exact(xq, fx["offset"], mask, wq, fx["bias"], xs, ws,
                                         fx["stride"], fx["padding"], fx["dilation"],
                                         fx["groups"], want_cols=True)
    assert int(fx["groups"]) == 1
    for n in range(xq.shape[0]):
        ref = i8_cols_numpy(xq[n], fx["offset"][n], mask[n], fx["stride"], fx["padding"],
                            fx["dilation"], k=int(np.sqrt(fx["offset"].shape[1] // 2)))
        assert np.array_equal(cols[n].astype(np.int64), ref)


def test_int8_reference_path_tolerance(golden_dir):
    fx = load(golden_dir, "kat_16c_32.npz")
    xq, xs = oracle.quantize_sym(fx["x"])
    wq, ws = oracle.quantize_sym(fx["weight"])
    y = oracle.forward_i8_ref(xq, fx["offset"], fx["mask"], wq, fx["bias"], xs, ws)
    rel = np.abs(y - fx["y"]).sum() / np.abs(fx["y"]).sum()
    assert rel < 0.1  # src/test_dcn_int8_gemm.cu:89 (README reports 1.27%)


def test_band_matches_full(golden_dir):
    fx = load(golden_dir, "tv_n2_dg2_s2.npz")
    full = run_ref(fx)
    ho, wo = full.shape[2:]
    band = oracle.forward_ref_band(fx["x"], fx["offset"], fx["mask"], fx["weight"], fx["bias"],
                                   5, 23, fx["stride"], fx["padding"], fx["dilation"],
                                   fx["groups"])
    assert np.array_equal(band, full.reshape(full.shape[0], full.shape[1], -1)[:, :, 5:23])


def test_int8_column_rules_agree_on_the_int8_workload():
    """The kernels' int8 column rule (16-bit fixed-point corner weights, integer rounding) against
    the reference-rounding definition clamp(rint(m * bilinear(x_q)), -127, 127) in the reference's fp32
    arithmetic (src/dcn_kernel.cu:218-235), on one image of the benchmarked int8 workload
    (256 -> 256, 64x64, offsets N(0, 0.5^2) with 5 % at +-70, mask sigmoid(N(0, 1))).
    Measured: 0.017 % of the 9.4 M column values differ, each by 1; mean relative error against
    fp32 torchvision is 3.23 % for both rules (the reference's non-integer fp32 columns: 1.14 %,
    the reference reports 1.27 % on its own data, README.md:43)."""
    import sys
    import torch
    tv = pytest.importorskip("torchvision.ops")
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(__file__)),
                                    "tensorrt-dcnv2-plugin_b200"))
    from dcnv2_b200 import workloads as wl
    inp = wl.workload("int8_n64_256c_64", n=1, seed=0)
    L = inp.layer
    P = L.ho * L.wo
    x, off, m, w, b = [t.numpy() for t in inp.tensors()]
    yf, _, cf = oracle.forward_i8_exact_band(x, off, m, w, b, inp.x_scale, inp.w_scale, 0, P,
                                             rule="fixed", want_cols=True)
    yr, _, cr = oracle.forward_i8_exact_band(x, off, m, w, b, inp.x_scale, inp.w_scale, 0, P,
                                             rule="rint", want_cols=True)
    d = cf.astype(np.int32) - cr.astype(np.int32)
    assert np.abs(d).max() <= 1
    assert (d != 0).mean() < 1e-3
    yt = tv.deform_conv2d(inp.extra["x_f32"], torch.from_numpy(off), inp.extra["w_f32"],
                          torch.from_numpy(b), padding=1, mask=torch.from_numpy(m)).numpy()
    yt = yt.reshape(1, L.out_c, P)
    mr = lambda a: float(np.abs(a - yt).sum() / np.abs(yt).sum())
    assert abs(mr(yf) - mr(yr)) <= 0.01 * mr(yr)
    assert mr(yf) < 0.05


def test_int8_exact_band_matches_whole_image(golden_dir):
    fx = load(golden_dir, "tv_n2_dg2_s2.npz")
    xq, xs = oracle.quantize_sym(fx["x"])
    wq, ws = oracle.quantize_sym(fx["weight"])
    a = (fx["stride"], fx["padding"], fx["dilation"], fx["groups"])
    y, acc = oracle.forward_i8_exact(xq, fx["offset"], fx["mask"], wq, fx["bias"], xs, ws, *a)
    n, o = acc.shape[:2]
    P = acc.shape[2] * acc.shape[3]
    yb, accb = oracle.forward_i8_exact_band(xq, fx["offset"], fx["mask"], wq, fx["bias"], xs,
                                            ws, 5, P - 3, *a)
    assert np.array_equal(accb, acc.reshape(n, o, P)[:, :, 5:P - 3])
    assert np.array_equal(yb, y.reshape(n, o, P)[:, :, 5:P - 3])
