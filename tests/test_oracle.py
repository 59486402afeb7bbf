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
    # |y_exact - y_ref| <= 0.5 * xs * ws * sum|w_q| (+ fp32 slack)
    yref = oracle.forward_i8_ref(xq, fx["offset"], fx["mask"], wq, fx["bias"], xs, ws)
    bound = 0.5 * xs * ws * np.abs(wq).reshape(wq.shape[0], -1).sum(1)
    dev = np.abs(y - yref).max(axis=(0, 2, 3))
    assert np.all(dev <= bound * 1.0001 + 1e-5)
    # and the INT8 result stays within the reference INT8 tolerance of the fp32 answer
    # (mean relative error < 10%, src/test_dcn_int8_gemm.cu:89)
    rel = np.abs(y - fx["y"]).sum() / np.abs(fx["y"]).sum()
    assert rel < 0.05


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
