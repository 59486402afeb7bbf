"""Host-side checks of libdcnv2.so that need no GPU: the library loads, exports every symbol the
headers declare, and its plugin logic (identity, attributes, serialisation, shape inference,
precision negotiation, workspace rule, argument validation) behaves like the reference plugin
(src/dcn_plugin.cpp). No kernel is launched here."""
import ctypes
import os
import re

import pytest

from dcnv2_b200 import DCNv2Creator, tensor_desc
from dcnv2_b200 import capi
from dcnv2_b200.capi import DType, Math, Status

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for h in ("dcnv2.h", "dcnv2_diag.h"):
        src = open(os.path.join(ROOT, "include", h)).read()
        names |= set(re.findall(r"DCNV2_API\s+[\w\s\*]+?\b(dcnv2_\w+)\s*\(", src))
    return names


def test_library_exports_every_declared_symbol():
    names = declared_symbols()
    assert len(names) >= 20
    lib = ctypes.CDLL(capi.LIB_PATH)
    for n in sorted(names):
        assert hasattr(lib, n), n
    assert names == set(capi.EXPORTED)


def test_library_build_targets_sm100a_only():
    """The build recipe compiles every device object for sm_100a and nothing else (the device
    code's architecture is checked at run time on the GPU: test_gpu_parity's
    test_device_code_is_sm100)."""
    mk = open(os.path.join(ROOT, "tensorrt-dcnv2-plugin_b200", "csrc", "Makefile")).read()
    arch = re.findall(r"-gencode\s+arch=(\S+),code=(\S+)", mk)
    assert arch == [("compute_100a", "sm_100a")]


def test_package_import_maps_no_library():
    """Importing the package (e.g. for the seeded workload generators) maps no libdcnv2.so; the
    first library call does. The reference benchmark arm relies on this."""
    import subprocess
    import sys
    code = ("import sys; sys.path.insert(0, %r)\n"
            "import dcnv2_b200.workloads, dcnv2_b200\n"
            "maps = open('/proc/self/maps').read()\n"
            "assert 'libdcnv2.so' not in maps, 'mapped at import'\n"
            "from dcnv2_b200 import capi\n"
            "capi.lib.dcnv2_plugin_name()\n"
            "assert 'libdcnv2.so' in open('/proc/self/maps').read()\n"
            % os.path.join(ROOT, "tensorrt-dcnv2-plugin_b200"))
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-2000:]


def test_plugin_identity_and_fields():
    cr = DCNv2Creator()
    assert (cr.get_plugin_name(), cr.get_plugin_version(), cr.get_plugin_namespace()) == \
        ("DCNv2", "1", "")
    assert cr.get_field_names() == ["stride", "padding", "dilation", "kernel",
                                    "deformable_groups"]
    p = cr.create_plugin("DCNv2", {})
    assert p.get_fields_to_serialize() == {"stride": 1, "padding": 1, "dilation": 1,
                                           "kernel": 3, "deformable_groups": 1}
    p2 = cr.create_plugin("DCNv2", {"stride": 2, "padding": 2, "dilation": 2, "kernel": 5,
                                    "deformable_groups": 8, "unknown": 7})
    f = p2.get_fields_to_serialize()
    assert f == {"stride": 2, "padding": 2, "dilation": 2, "kernel": 5, "deformable_groups": 8}
    # a field without data reads as 0 (src/dcn_plugin.cpp:227)
    assert cr.create_plugin("DCNv2", {"padding": None}).get_fields_to_serialize()["padding"] == 0
    # serialize -> create round trip
    assert cr.create_plugin("DCNv2", f).get_fields_to_serialize() == f
    assert p2.clone().get_fields_to_serialize() == f
    assert p2.attach_to_context().get_fields_to_serialize() == f
    assert p.get_nb_outputs() == 1


@pytest.mark.parametrize("attrs,x,w,expect", [
    (dict(), (1, 256, 64, 64), (256, 256, 3, 3), (1, 256, 64, 64)),
    (dict(stride=2), (2, 16, 11, 13), (24, 16, 3, 3), (2, 24, 6, 7)),
    (dict(padding=2, dilation=2), (1, 512, 128, 128), (512, 512, 3, 3), (1, 512, 128, 128)),
    (dict(kernel=1, padding=0), (3, 8, 7, 9), (4, 8, 1, 1), (3, 4, 7, 9)),
    (dict(kernel=5, padding=2, stride=3), (1, 8, 10, 17), (8, 8, 5, 5), (1, 8, 4, 6)),
])
def test_output_shapes(attrs, x, w, expect):
    p = DCNv2Creator().create_plugin("DCNv2", attrs)
    assert p.get_output_shapes(x, w) == [expect]
    d = capi.make_desc(*x, w[0], kernel=attrs.get("kernel", 3), stride=attrs.get("stride", 1),
                       padding=attrs.get("padding", 1), dilation=attrs.get("dilation", 1))
    assert capi.output_shape(d) == expect


def test_supports_format_combination():
    p = DCNv2Creator().create_plugin("DCNv2", {})
    F, H, I = DType.FLOAT, DType.HALF, DType.INT8

    def combo(types, fmt=0):
        return [tensor_desc((1, 1, 1, 1), t, fmt) for t in types]

    for t in (F, H, I):
        assert p.supports_format_combination(0, combo([t] * 6))
    assert not p.supports_format_combination(0, combo([F] * 6, fmt=1))  # non-linear format
    assert all(p.supports_format_combination(i, combo([H] * 6)) for i in range(6))
    assert not p.supports_format_combination(3, combo([H, H, H, F, H, H]))
    int8 = combo([I, F, F, I, F, F])
    assert all(p.supports_format_combination(i, int8) for i in range(6))
    assert not p.supports_format_combination(5, combo([I, F, F, I, F, I]))
    assert not p.supports_format_combination(1, combo([I, I, F, I, F, F]))
    # output dtype follows x, except INT8 -> FLOAT (agrees with the combination above)
    assert p.get_output_data_types([F]) == [F]
    assert p.get_output_data_types([H]) == [H]
    assert p.get_output_data_types([I]) == [F]


def test_workspace_rule():
    d = capi.make_desc(64, 256, 64, 64, 256, dtype=DType.HALF)
    ws = capi.workspace_size(d)
    x_bytes = 64 * 256 * 64 * 64 * 2
    w_bytes = 9 * 4 * 256 * 128  # 36 K-blocks x 256 rows x 128 B
    assert x_bytes + w_bytes <= ws <= x_bytes + w_bytes + 4096
    assert capi.uses_tensor_cores(d)
    assert capi.launch_count(d) == 2  # one pre-pass launch (transpose + packing), main kernel
    # scales with N (the reference's rule ignored N)
    d1 = capi.make_desc(1, 256, 64, 64, 256, dtype=DType.HALF)
    assert capi.workspace_size(d1) < ws
    # plugin path agrees with the desc path
    p = DCNv2Creator().create_plugin("DCNv2", {})
    ins = [tensor_desc((64, 256, 64, 64), DType.HALF), tensor_desc((64, 18, 64, 64), DType.HALF),
           tensor_desc((64, 9, 64, 64), DType.HALF), tensor_desc((256, 256, 3, 3), DType.HALF),
           tensor_desc((256,), DType.HALF)]
    outs = [tensor_desc((64, 256, 64, 64), DType.HALF)]
    assert p.get_workspace_size(ins, outs) == ws
    # SIMT-only shapes need just the error word
    odd = capi.make_desc(1, 6, 9, 9, 4, dtype=DType.HALF)
    assert not capi.uses_tensor_cores(odd) and capi.workspace_size(odd) <= 1024
    assert capi.launch_count(odd) == 1


@pytest.mark.parametrize("kw", [
    dict(n=0), dict(c=0), dict(h=0), dict(out_c=0), dict(kernel=0), dict(stride=0),
    dict(padding=-1), dict(dilation=0), dict(deformable_groups=0), dict(deformable_groups=3),
    dict(h=1, w=1, padding=0), dict(math=9), dict(math=-1),
])
def test_invalid_descs(kw):
    base = dict(n=1, c=16, h=8, w=8, out_c=8)
    base.update(kw)
    n, c, h, w, o = (base.pop(k) for k in ("n", "c", "h", "w", "out_c"))
    d = capi.make_desc(n, c, h, w, o, **base)
    assert capi.workspace_size(d) == 0
    st = capi.forward_raw(d, 16, 16, 16, 16, 16, 16, 256, 1 << 20)
    assert st == Status.ERR_INVALID_ARG


def test_forward_argument_errors_before_any_launch():
    d = capi.make_desc(1, 16, 8, 8, 8, dtype=DType.FLOAT)
    wsz = capi.workspace_size(d)
    assert capi.forward_raw(d, None, 256, 256, 256, 256, 256, 256, wsz) == Status.ERR_INVALID_ARG
    assert capi.forward_raw(d, 258, 256, 256, 256, 256, 256, 256, wsz) == Status.ERR_INVALID_ARG
    assert capi.forward_raw(d, 256, 256, 256, 256, 256, 256, None, wsz) == Status.ERR_WORKSPACE
    assert capi.forward_raw(d, 256, 256, 256, 256, 256, 256, 256, wsz - 1) == Status.ERR_WORKSPACE
    d8 = capi.make_desc(1, 16, 8, 8, 8, dtype=DType.INT8)
    for xs, ws in ((0.0, 1.0), (1.0, -1.0), (float("nan"), 1.0), (float("inf"), 1.0)):
        assert capi.forward_raw(d8, 256, 256, 256, 256, 256, 256, 256,
                                capi.workspace_size(d8), xs, ws) == Status.ERR_INVALID_ARG
    bad = capi.make_desc(1, 16, 8, 8, 8, dtype=7)
    assert capi.forward_raw(bad, 256, 256, 256, 256, 256, 256, 256, 1 << 20) == \
        Status.ERR_UNSUPPORTED
    assert capi.status_string(Status.ERR_WORKSPACE).startswith("workspace")


def test_math_modes_select_kernels():
    f32 = capi.make_desc(1, 256, 64, 64, 256, dtype=DType.FLOAT)
    assert capi.uses_tensor_cores(f32) == 2  # fp32-exact fused CUDA-core kernel
    assert capi.launch_count(f32) == 2
    for m in (Math.TF32, Math.TF32X3):
        assert capi.uses_tensor_cores(capi.make_desc(1, 256, 64, 64, 256, dtype=DType.FLOAT,
                                                     math=m)) == 1
    simt = capi.make_desc(1, 256, 64, 64, 256, dtype=DType.FLOAT, math=Math.SIMT)
    assert not capi.uses_tensor_cores(simt)
    for bad in ((DType.HALF, Math.TF32), (DType.INT8, Math.TF32X3), (DType.FLOAT, Math.PRECISE)):
        d = capi.make_desc(1, 256, 64, 64, 256, dtype=bad[0], math=bad[1])
        assert capi.workspace_size(d) == 0
    # int8 needs 16-channel groups for the tensor-core path
    assert capi.uses_tensor_cores(capi.make_desc(1, 32, 8, 8, 8, dtype=DType.INT8))
    assert not capi.uses_tensor_cores(capi.make_desc(1, 24, 8, 8, 8, dtype=DType.INT8))
    assert capi.uses_tensor_cores(capi.make_desc(1, 24, 8, 8, 8, dtype=DType.HALF))


def test_enqueue_rejects_mismatched_output_and_combination():
    p = DCNv2Creator().create_plugin("DCNv2", {})
    H = DType.HALF
    ins = [tensor_desc((1, 16, 8, 8), H), tensor_desc((1, 18, 8, 8), H),
           tensor_desc((1, 9, 8, 8), H), tensor_desc((8, 16, 3, 3), H), tensor_desc((8,), H)]
    bad_out = [tensor_desc((1, 8, 7, 8), H)]
    assert p.enqueue(ins, bad_out, [256] * 5, [256], 256, 1 << 20) == Status.ERR_INVALID_ARG
    mixed = list(ins)
    mixed[1] = tensor_desc((1, 18, 8, 8), DType.FLOAT)
    assert p.enqueue(mixed, [tensor_desc((1, 8, 8, 8), H)], [256] * 5, [256], 256, 1 << 20) == \
        Status.ERR_UNSUPPORTED


def test_forward_with_head_support_rules():
    """The layer-with-head entry point takes fp16 "same" layers (stride 1, dilation 1, padding
    (K-1)/2, C a multiple of 8, 3*dg*K*K <= 256) on the tensor-core path; its workspace holds the
    layer's workspace plus the head's packed weights and its offset / mask outputs."""
    ok = capi.make_desc(2, 64, 24, 24, 48, 3, 1, 1, 1, 1, DType.HALF)
    need = capi.forward_with_head_workspace_size(ok)
    assert need > capi.workspace_size(ok) + 2 * 27 * 24 * 24 * 2
    for bad in (capi.make_desc(2, 64, 24, 24, 48, 3, 1, 1, 1, 1, DType.FLOAT),
                capi.make_desc(2, 64, 24, 24, 48, 3, 1, 1, 1, 1, DType.INT8),
                capi.make_desc(2, 64, 24, 24, 48, 3, 2, 1, 1, 1, DType.HALF),
                capi.make_desc(2, 64, 24, 24, 48, 3, 1, 2, 2, 1, DType.HALF),
                capi.make_desc(2, 60, 24, 24, 48, 3, 1, 1, 1, 1, DType.HALF),
                capi.make_desc(2, 64, 24, 24, 48, 3, 1, 0, 1, 1, DType.HALF),
                capi.make_desc(2, 640, 24, 24, 48, 3, 1, 1, 1, 10, DType.HALF)):
        assert capi.forward_with_head_workspace_size(bad) == 0
    assert capi.forward_with_head_workspace_size(
        capi.make_desc(1, 256, 64, 64, 256, 3, 1, 1, 1, 8, DType.HALF)) > 0


def test_kernel_override_validation_and_plan_effect():
    """The measurement override changes the planned kernel and rejects out-of-range values; the
    automatic selection picks CTA pairs only for the A-in-shared-memory kernel above 256 output
    channels (the plan is visible through the kernel name and the workspace size)."""
    d = capi.make_desc(2, 256, 32, 32, 256, dtype=DType.HALF)
    try:
        assert capi.main_kernel(d) == "dcnv2_fused_ta_kernel"
        capi.set_kernel_override(capi.Kernel.SMEM)
        assert capi.main_kernel(d) == "dcnv2_fused_kernel"
        capi.set_kernel_override(capi.Kernel.TA, capi.Pair.PAIRS)
        assert capi.main_kernel(d) == "dcnv2_fused_ta_kernel"
        for bad in ((3, 0), (-1, 0), (0, 3), (0, -1)):
            assert capi.lib.dcnv2_diag_set_kernel_override(*bad) == Status.ERR_INVALID_ARG
    finally:
        capi.set_kernel_override(capi.Kernel.AUTO, capi.Pair.AUTO)
    assert capi.main_kernel(d) == "dcnv2_fused_ta_kernel"
    wide = capi.make_desc(1, 512, 16, 16, 512, 3, 1, 2, 2, 8, DType.INT8)
    assert capi.main_kernel(wide) == "dcnv2_fused_kernel"


def test_binary_arch_without_device():
    """Without a usable sm_100 device the architecture query reports no device instead of
    failing."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present (the GPU test covers the query)")
    v = ctypes.c_int32(0)
    assert capi.lib.dcnv2_diag_binary_arch(ctypes.byref(v)) == Status.ERR_NO_DEVICE


def test_int8_precise_takes_the_reference_rounding_kernel():
    """int8 with DCNV2_MATH_PRECISE computes each column as the reference's fp32 sample rounded
    to nearest, on the one-thread-per-output kernel; fp32 has no PRECISE mode."""
    d = capi.make_desc(2, 64, 16, 16, 32, dtype=DType.INT8, math=Math.PRECISE)
    assert capi.uses_tensor_cores(d) == 0
    assert capi.main_kernel(d) == "dcnv2_simt_kernel"
    assert capi.uses_tensor_cores(capi.make_desc(2, 64, 16, 16, 32, dtype=DType.INT8)) == 1
