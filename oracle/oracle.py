"""Test infrastructure (the oracle): ctypes bindings of

  * _build/liboracle.so  — the CPU restatement of the reference DCNv2 forward (dcnv2_oracle.c);
  * _ref/libdcnv2_ref.so — the reference's own kernels (src/dcn_kernel.cu) + cuBLAS, replayed
                           through enqueue's three precision branches (ref_enqueue.cu).

Only the tests, __graft_entry__.smoke() and bench.py's CPU-baseline / reference legs use this
module, and only as the checker or the timed baseline; libdcnv2 never calls it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_LIB = os.path.join(HERE, "_build", "liboracle.so")
REF_LIB = os.path.join(HERE, "_ref", "libdcnv2_ref.so")


class Shape(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in (
        "n", "c", "h", "w", "out_c", "kernel", "stride", "padding", "dilation", "groups")]


def build() -> None:
    """Compiles liboracle.so (and _ref when the reference tree is present)."""
    subprocess.run(["make", "-C", HERE, "-s"], check=True)


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(ORACLE_LIB):
            build()
        L = ctypes.CDLL(ORACLE_LIB)
        fp = ctypes.POINTER(ctypes.c_float)
        i8p = ctypes.POINTER(ctypes.c_int8)
        Sp = ctypes.POINTER(Shape)
        L.oracle_forward_ref.argtypes = [Sp, ctypes.c_int, fp, fp, fp, fp, fp, fp, ctypes.c_int]
        L.oracle_forward_ref.restype = ctypes.c_int
        L.oracle_forward_ref_band.argtypes = [Sp, ctypes.c_int, fp, fp, fp, fp, fp, fp,
                                              ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.oracle_forward_ref_band.restype = ctypes.c_int
        L.oracle_forward_i8_ref.argtypes = [Sp, i8p, fp, fp, i8p, fp, ctypes.c_float,
                                            ctypes.c_float, fp, ctypes.c_int]
        L.oracle_forward_i8_ref.restype = ctypes.c_int
        L.oracle_forward_i8_exact.argtypes = [Sp, i8p, fp, fp, i8p, fp, ctypes.c_float,
                                              ctypes.c_float, ctypes.POINTER(ctypes.c_double),
                                              ctypes.POINTER(ctypes.c_int64), i8p, ctypes.c_int]
        L.oracle_forward_i8_exact.restype = ctypes.c_int
        L.oracle_forward_i8_exact_band.argtypes = [
            Sp, i8p, fp, fp, i8p, fp, ctypes.c_float, ctypes.c_float,
            ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_int64), i8p, ctypes.c_int,
            ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.oracle_forward_i8_exact_band.restype = ctypes.c_int
        L.oracle_quantize_sym.argtypes = [fp, ctypes.c_int64, i8p]
        L.oracle_quantize_sym.restype = ctypes.c_float
        L.oracle_forward_direct.argtypes = [Sp, fp, fp, fp, fp, fp, fp]
        L.oracle_forward_direct.restype = ctypes.c_int
        _lib = L
    return _lib


def _f32(a):
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def _i8(a):
    return np.ascontiguousarray(np.asarray(a, dtype=np.int8))


def _p(a, t):
    return a.ctypes.data_as(ctypes.POINTER(t))


def out_hw(h, w, k, s, p, d):
    return (h + 2 * p - d * (k - 1) - 1) // s + 1, (w + 2 * p - d * (k - 1) - 1) // s + 1


def _shape(x, weight, stride, padding, dilation, groups):
    n, c, h, w = x.shape
    o, _, k, _ = weight.shape
    return Shape(n, c, h, w, o, k, stride, padding, dilation, groups)


def forward_ref(x, offset, mask, weight, bias, stride=1, padding=1, dilation=1, groups=1,
                precision="fp32", threads=None):
    """Reference fast path: precision "fp32" (dcn_plugin.cpp:162-174) or "fp16" (:148-161)."""
    x, offset, mask, weight = _f32(x), _f32(offset), _f32(mask), _f32(weight)
    b = _f32(bias) if bias is not None else None
    s = _shape(x, weight, stride, padding, dilation, groups)
    ho, wo = out_hw(s.h, s.w, s.kernel, stride, padding, dilation)
    y = np.empty((s.n, s.out_c, ho, wo), np.float32)
    fp = ctypes.c_float
    rc = lib().oracle_forward_ref(ctypes.byref(s), 1 if precision == "fp16" else 0, _p(x, fp),
                                  _p(offset, fp), _p(mask, fp), _p(weight, fp),
                                  _p(b, fp) if b is not None else None, _p(y, fp),
                                  threads or os.cpu_count() or 1)
    if rc:
        raise ValueError("oracle_forward_ref failed")
    return y


def forward_ref_band(x, offset, mask, weight, bias, p_begin, p_end, stride=1, padding=1,
                     dilation=1, groups=1, precision="fp32", threads=None):
    """Reference fast path restricted to output pixels [p_begin, p_end) of every image (the
    bounded CPU-baseline sample). Returns y[N, O, p_end - p_begin]."""
    x, offset, mask, weight = _f32(x), _f32(offset), _f32(mask), _f32(weight)
    b = _f32(bias) if bias is not None else None
    s = _shape(x, weight, stride, padding, dilation, groups)
    y = np.empty((s.n, s.out_c, p_end - p_begin), np.float32)
    fp = ctypes.c_float
    rc = lib().oracle_forward_ref_band(ctypes.byref(s), 1 if precision == "fp16" else 0,
                                       _p(x, fp), _p(offset, fp), _p(mask, fp), _p(weight, fp),
                                       _p(b, fp) if b is not None else None, _p(y, fp),
                                       threads or os.cpu_count() or 1, int(p_begin), int(p_end))
    if rc:
        raise ValueError("oracle_forward_ref_band failed")
    return y


def forward_i8_ref(xq, offset, mask, wq, bias, x_scale, w_scale, stride=1, padding=1,
                   dilation=1, groups=1, threads=None):
    """Reference INT8 fast path (dcn_plugin.cpp:135-147): fp32 columns, fp32 output."""
    xq, wq, offset, mask = _i8(xq), _i8(wq), _f32(offset), _f32(mask)
    b = _f32(bias) if bias is not None else None
    s = _shape(xq, wq, stride, padding, dilation, groups)
    ho, wo = out_hw(s.h, s.w, s.kernel, stride, padding, dilation)
    y = np.empty((s.n, s.out_c, ho, wo), np.float32)
    fp, i8 = ctypes.c_float, ctypes.c_int8
    rc = lib().oracle_forward_i8_ref(ctypes.byref(s), _p(xq, i8), _p(offset, fp), _p(mask, fp),
                                     _p(wq, i8), _p(b, fp) if b is not None else None,
                                     float(x_scale), float(w_scale), _p(y, fp),
                                     threads or os.cpu_count() or 1)
    if rc:
        raise ValueError("oracle_forward_i8_ref failed")
    return y


def forward_i8_exact(xq, offset, mask, wq, bias, x_scale, w_scale, stride=1, padding=1,
                     dilation=1, groups=1, want_cols=False, threads=None):
    """Exact int32-domain INT8 definition: returns (y float64, acc int64[, cols int8])."""
    xq, wq, offset, mask = _i8(xq), _i8(wq), _f32(offset), _f32(mask)
    b = _f32(bias) if bias is not None else None
    s = _shape(xq, wq, stride, padding, dilation, groups)
    ho, wo = out_hw(s.h, s.w, s.kernel, stride, padding, dilation)
    y = np.empty((s.n, s.out_c, ho, wo), np.float64)
    acc = np.empty((s.n, s.out_c, ho, wo), np.int64)
    cols = np.empty((s.n, s.c * s.kernel ** 2, ho * wo), np.int8) if want_cols else None
    fp, i8 = ctypes.c_float, ctypes.c_int8
    rc = lib().oracle_forward_i8_exact(
        ctypes.byref(s), _p(xq, i8), _p(offset, fp), _p(mask, fp), _p(wq, i8),
        _p(b, fp) if b is not None else None, float(x_scale), float(w_scale),
        _p(y, ctypes.c_double), _p(acc, ctypes.c_int64), _p(cols, i8) if want_cols else None,
        threads or os.cpu_count() or 1)
    if rc:
        raise ValueError("oracle_forward_i8_exact failed")
    return (y, acc, cols) if want_cols else (y, acc)


I8_RULES = {"fixed": 0, "rint": 1}


def forward_i8_exact_band(xq, offset, mask, wq, bias, x_scale, w_scale, p_begin, p_end,
                          stride=1, padding=1, dilation=1, groups=1, rule="fixed",
                          want_cols=False, threads=None):
    """Exact INT8 on output pixels [p_begin, p_end) of every image. rule "fixed": the column
    rule the kernels implement (16-bit fixed-point corner weights); rule "rint": the reference's
    fp32 column m*bilinear(x_q) (src/dcn_kernel.cu:218-235) rounded to nearest, clamped to
    +-127. Returns (y float64 [N,O,np], acc int64 [N,O,np][, cols int8 [N,C*K*K,np]])."""
    xq, wq, offset, mask = _i8(xq), _i8(wq), _f32(offset), _f32(mask)
    b = _f32(bias) if bias is not None else None
    s = _shape(xq, wq, stride, padding, dilation, groups)
    npx = int(p_end) - int(p_begin)
    y = np.empty((s.n, s.out_c, npx), np.float64)
    acc = np.empty((s.n, s.out_c, npx), np.int64)
    cols = np.empty((s.n, s.c * s.kernel ** 2, npx), np.int8) if want_cols else None
    fp, i8 = ctypes.c_float, ctypes.c_int8
    rc = lib().oracle_forward_i8_exact_band(
        ctypes.byref(s), _p(xq, i8), _p(offset, fp), _p(mask, fp), _p(wq, i8),
        _p(b, fp) if b is not None else None, float(x_scale), float(w_scale),
        _p(y, ctypes.c_double), _p(acc, ctypes.c_int64), _p(cols, i8) if want_cols else None,
        threads or os.cpu_count() or 1, int(p_begin), int(p_end), I8_RULES[rule])
    if rc:
        raise ValueError("oracle_forward_i8_exact_band failed")
    return (y, acc, cols) if want_cols else (y, acc)


def quantize_sym(v):
    v = _f32(v)
    q = np.empty(v.shape, np.int8)
    scale = lib().oracle_quantize_sym(_p(v, ctypes.c_float), v.size, _p(q, ctypes.c_int8))
    return q, float(scale)


def forward_direct(x, offset, mask, weight, bias, stride=1, padding=1, dilation=1, groups=1):
    """Naive-kernel semantics (src/dcn_kernel.cu:33-65), double accumulation; small cases only."""
    x, offset, mask, weight = _f32(x), _f32(offset), _f32(mask), _f32(weight)
    b = _f32(bias) if bias is not None else None
    s = _shape(x, weight, stride, padding, dilation, groups)
    ho, wo = out_hw(s.h, s.w, s.kernel, stride, padding, dilation)
    y = np.empty((s.n, s.out_c, ho, wo), np.float32)
    fp = ctypes.c_float
    rc = lib().oracle_forward_direct(ctypes.byref(s), _p(x, fp), _p(offset, fp), _p(mask, fp),
                                     _p(weight, fp), _p(b, fp) if b is not None else None,
                                     _p(y, fp))
    if rc:
        raise ValueError("oracle_forward_direct failed")
    return y


# ---------------------------------------------------------------- reference GPU path
_ref = None


def ref_gpu_available() -> bool:
    return os.path.exists(REF_LIB)


def ref_lib() -> ctypes.CDLL:
    global _ref
    if _ref is None:
        L = ctypes.CDLL(REF_LIB)
        P = ctypes.c_void_p
        L.ref_enqueue.argtypes = [ctypes.c_int] * 10 + [P] * 7 + [ctypes.c_float,
                                                                  ctypes.c_float, P]
        L.ref_enqueue.restype = ctypes.c_int
        L.ref_workspace_size.argtypes = [ctypes.c_int] * 5
        L.ref_workspace_size.restype = ctypes.c_size_t
        _ref = L
    return _ref


def ref_gpu_forward(x, offset, mask, weight, bias, stride=1, padding=1, dilation=1,
                    x_scale=1.0, w_scale=1.0):
    """Runs the reference's own im2col + cuBLAS path on the GPU (torch CUDA tensors, dg = 1)."""
    import torch
    n, c, h, w = x.shape
    o, _, k, _ = weight.shape
    ho, wo = out_hw(h, w, k, stride, padding, dilation)
    dtype = {torch.float32: 0, torch.float16: 1, torch.int8: 2}[x.dtype]
    ydt = torch.float16 if dtype == 1 else torch.float32
    y = torch.empty((n, o, ho, wo), dtype=ydt, device=x.device)
    L = ref_lib()
    ws = torch.empty(L.ref_workspace_size(c, k, o, ho, wo), dtype=torch.uint8, device=x.device)
    st = torch.cuda.current_stream(x.device).cuda_stream
    rc = L.ref_enqueue(dtype, n, c, h, w, o, k, stride, padding, dilation, x.data_ptr(),
                       offset.data_ptr(), mask.data_ptr(), weight.data_ptr(), bias.data_ptr(),
                       y.data_ptr(), ws.data_ptr(), float(x_scale), float(w_scale), st)
    if rc:
        raise RuntimeError(f"ref_enqueue failed rc={rc}")
    return y
