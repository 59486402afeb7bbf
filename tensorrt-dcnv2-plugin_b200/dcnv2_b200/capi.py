"""ctypes binding of libdcnv2.so (include/dcnv2.h).

This is the Python-side FFI a caller of the reference would write around libdcnv2.so
(python/02_build_and_validate.py:29 loads it with ctypes.CDLL). It adds nothing to the compute
path: every forward goes through the C ABI into the sm_100a kernels. The library is mapped on the
first call that needs it (so that importing the package's pure-Python parts, such as the
workload generators, maps nothing); if it is missing that call raises ImportError. There is no
fallback.
"""
from __future__ import annotations

import ctypes
import enum
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.normpath(os.path.join(_HERE, "..", "lib", "libdcnv2.so"))


class Status(enum.IntEnum):
    OK = 0
    ERR_INVALID_ARG = 1
    ERR_UNSUPPORTED = 2
    ERR_WORKSPACE = 3
    ERR_CUDA = 4
    ERR_NO_DEVICE = 5
    ERR_DEVICE_TIMEOUT = 6
    ERR_SCRATCH_LIMIT = 7


#: Size of the library's static scratch buffer (DCNV2_STATIC_SCRATCH_BYTES in include/dcnv2.h).
STATIC_SCRATCH_BYTES = 32 * 1024 * 1024


class DType(enum.IntEnum):
    """Values of nvinfer1::DataType used by the plugin."""
    FLOAT = 0
    HALF = 1
    INT8 = 2


class Math(enum.IntEnum):
    DEFAULT = 0
    PRECISE = 1
    TF32 = 2
    SIMT = 3
    TF32X3 = 4


FORMAT_LINEAR = 0


class Desc(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in (
        "n", "c", "h", "w", "out_c", "kernel", "stride", "padding", "dilation",
        "deformable_groups", "dtype", "math")]


class TensorDesc(ctypes.Structure):
    _fields_ = [("nb_dims", ctypes.c_int32), ("d", ctypes.c_int64 * 8), ("type", ctypes.c_int32),
                ("format", ctypes.c_int32), ("scale", ctypes.c_float)]


class DCNv2Error(RuntimeError):
    def __init__(self, status: int, what: str = ""):
        self.status = Status(status) if status in Status._value2member_map_ else status
        super().__init__(f"{what}: {self.status!r}" if what else repr(self.status))


def _load() -> ctypes.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"libdcnv2.so not built at {LIB_PATH}; run __graft_entry__.build()")
    lib = ctypes.CDLL(LIB_PATH, mode=ctypes.RTLD_GLOBAL)
    P = ctypes.c_void_p
    Dp = ctypes.POINTER(Desc)
    TDp = ctypes.POINTER(TensorDesc)
    sig = {
        "dcnv2_output_shape": (ctypes.c_int, [Dp, ctypes.POINTER(ctypes.c_int64)]),
        "dcnv2_workspace_size": (ctypes.c_size_t, [Dp]),
        "dcnv2_forward": (ctypes.c_int, [Dp, P, P, P, P, P, P, P, ctypes.c_size_t, ctypes.c_float,
                                         ctypes.c_float, P]),
        "dcnv2_forward_static_scratch": (ctypes.c_int, [Dp, P, P, P, P, P, P, ctypes.c_float,
                                                        ctypes.c_float, P]),
        "dcnv2_read_device_error": (ctypes.c_int, [P, P, ctypes.POINTER(ctypes.c_int32)]),
        "dcnv2_read_static_scratch_error": (ctypes.c_int, [P, ctypes.POINTER(ctypes.c_int32)]),
        "dcnv2_diag_set_kernel_override": (ctypes.c_int, [ctypes.c_int32, ctypes.c_int32]),
        "dcnv2_diag_binary_arch": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int32)]),
        "dcnv2_forward_with_head_workspace_size": (ctypes.c_size_t, [Dp]),
        "dcnv2_forward_with_head": (ctypes.c_int, [Dp, P, P, P, P, P, P, P, P, P,
                                                   ctypes.c_size_t, P]),
        "dcnv2_forward_host_workspace_size": (ctypes.c_size_t, [Dp, ctypes.c_int32]),
        "dcnv2_forward_host": (ctypes.c_int, [Dp, P, P, P, P, P, P, P, ctypes.c_size_t,
                                              ctypes.c_float, ctypes.c_float, ctypes.c_int32, P]),
        "dcnv2_uses_tensor_cores": (ctypes.c_int32, [Dp]),
        "dcnv2_launch_count": (ctypes.c_int32, [Dp]),
        "dcnv2_diag_main_kernel": (ctypes.c_char_p, [Dp]),
        "dcnv2_status_string": (ctypes.c_char_p, [ctypes.c_int]),
        "dcnv2_plugin_name": (ctypes.c_char_p, []),
        "dcnv2_plugin_version": (ctypes.c_char_p, []),
        "dcnv2_plugin_namespace": (ctypes.c_char_p, []),
        "dcnv2_plugin_field_names": (ctypes.c_int32, [ctypes.POINTER(ctypes.POINTER(ctypes.c_char_p))]),
        "dcnv2_plugin_create": (P, [ctypes.POINTER(ctypes.c_char_p),
                                    ctypes.POINTER(ctypes.POINTER(ctypes.c_int32)), ctypes.c_int32]),
        "dcnv2_plugin_clone": (P, [P]),
        "dcnv2_plugin_destroy": (None, [P]),
        "dcnv2_plugin_serialize": (ctypes.c_int32, [P, ctypes.POINTER(ctypes.c_char_p),
                                                    ctypes.POINTER(ctypes.c_int32)]),
        "dcnv2_plugin_nb_outputs": (ctypes.c_int32, [P]),
        "dcnv2_plugin_output_dtype": (ctypes.c_int32, [P, ctypes.c_int32]),
        "dcnv2_plugin_output_shape": (ctypes.c_int, [P, ctypes.POINTER(ctypes.c_int64),
                                                     ctypes.POINTER(ctypes.c_int64),
                                                     ctypes.POINTER(ctypes.c_int64)]),
        "dcnv2_plugin_supports_format": (ctypes.c_int32, [P, ctypes.c_int32, TDp, ctypes.c_int32,
                                                          ctypes.c_int32]),
        "dcnv2_plugin_workspace_size": (ctypes.c_size_t, [P, TDp, ctypes.c_int32, TDp,
                                                          ctypes.c_int32]),
        "dcnv2_plugin_enqueue": (ctypes.c_int32, [P, TDp, TDp, ctypes.POINTER(P),
                                                  ctypes.POINTER(P), P, ctypes.c_size_t, P]),
        "dcnv2_diag_timeout_selftest": (ctypes.c_int, [ctypes.c_uint32,
                                                       ctypes.POINTER(ctypes.c_int32)]),
        "dcnv2_diag_forward_events": (ctypes.c_int, [Dp, P, P, P, P, P, P, P, ctypes.c_size_t,
                                                     ctypes.c_float, ctypes.c_float, P,
                                                     ctypes.POINTER(P), ctypes.c_int32]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


class _LazyLib:
    """libdcnv2.so, mapped on first attribute access (ImportError if it is not built)."""

    def __init__(self):
        self._lib = None

    def __getattr__(self, name):
        if name.startswith("__"):
            raise AttributeError(name)
        if self._lib is None:
            self._lib = _load()
        return getattr(self._lib, name)

    @property
    def loaded(self) -> bool:
        return self._lib is not None


lib = _LazyLib()

#: Every entry point include/dcnv2.h and include/dcnv2_diag.h declare.
EXPORTED = (
    "dcnv2_output_shape", "dcnv2_workspace_size", "dcnv2_forward",
    "dcnv2_forward_static_scratch", "dcnv2_read_static_scratch_error", "dcnv2_read_device_error",
    "dcnv2_forward_with_head_workspace_size", "dcnv2_forward_with_head",
    "dcnv2_forward_host_workspace_size", "dcnv2_forward_host",
    "dcnv2_uses_tensor_cores", "dcnv2_launch_count", "dcnv2_status_string", "dcnv2_plugin_name",
    "dcnv2_plugin_version", "dcnv2_plugin_namespace", "dcnv2_plugin_field_names",
    "dcnv2_plugin_create", "dcnv2_plugin_clone", "dcnv2_plugin_destroy",
    "dcnv2_plugin_serialize", "dcnv2_plugin_nb_outputs", "dcnv2_plugin_output_dtype",
    "dcnv2_plugin_output_shape", "dcnv2_plugin_supports_format", "dcnv2_plugin_workspace_size",
    "dcnv2_plugin_enqueue", "dcnv2_diag_timeout_selftest", "dcnv2_diag_forward_events",
    "dcnv2_diag_main_kernel", "dcnv2_diag_set_kernel_override", "dcnv2_diag_binary_arch",
)


def make_desc(n, c, h, w, out_c, kernel=3, stride=1, padding=1, dilation=1,
              deformable_groups=1, dtype=DType.HALF, math=Math.DEFAULT) -> Desc:
    return Desc(int(n), int(c), int(h), int(w), int(out_c), int(kernel), int(stride),
                int(padding), int(dilation), int(deformable_groups), int(dtype), int(math))


def output_shape(desc: Desc):
    out = (ctypes.c_int64 * 4)()
    st = lib.dcnv2_output_shape(ctypes.byref(desc), out)
    if st != Status.OK:
        raise DCNv2Error(st, "dcnv2_output_shape")
    return tuple(out)


def workspace_size(desc: Desc) -> int:
    return int(lib.dcnv2_workspace_size(ctypes.byref(desc)))


def uses_tensor_cores(desc: Desc) -> int:
    """1 = fused tcgen05 kernel, 2 = fused fp32-exact CUDA-core kernel, 0 = per-output kernel."""
    return int(lib.dcnv2_uses_tensor_cores(ctypes.byref(desc)))


def main_kernel(desc: Desc) -> str:
    """Name of the main kernel dcnv2_forward launches for this desc."""
    name = lib.dcnv2_diag_main_kernel(ctypes.byref(desc))
    if name is None:
        raise DCNv2Error(Status.ERR_INVALID_ARG, "dcnv2_diag_main_kernel")
    return name.decode()


def launch_count(desc: Desc) -> int:
    return int(lib.dcnv2_launch_count(ctypes.byref(desc)))


def forward_raw(desc: Desc, x, offset, mask, weight, bias, y, workspace, workspace_bytes,
                x_scale=1.0, w_scale=1.0, stream=0) -> int:
    """Raw C call with integer device addresses; returns the dcnv2_status value."""
    return int(lib.dcnv2_forward(ctypes.byref(desc), x, offset, mask, weight, bias, y, workspace,
                                 workspace_bytes, float(x_scale), float(w_scale), stream))


def forward_host_workspace_size(desc: Desc, images_per_chunk: int = 0) -> int:
    return int(lib.dcnv2_forward_host_workspace_size(ctypes.byref(desc), int(images_per_chunk)))


def forward_host_raw(desc: Desc, x_host, offset_host, mask_host, weight, bias, y_host, workspace,
                     workspace_bytes, x_scale=1.0, w_scale=1.0, images_per_chunk=0,
                     stream=0) -> int:
    """Raw call of the host-buffer forward (x, offset, mask, y host addresses; weight, bias and
    workspace device addresses); returns the dcnv2_status value."""
    return int(lib.dcnv2_forward_host(ctypes.byref(desc), x_host, offset_host, mask_host, weight,
                                      bias, y_host, workspace, workspace_bytes, float(x_scale),
                                      float(w_scale), int(images_per_chunk), stream))


def read_device_error(workspace, stream=0) -> int:
    code = ctypes.c_int32(0)
    st = lib.dcnv2_read_device_error(workspace, stream, ctypes.byref(code))
    if st not in (Status.OK, Status.ERR_DEVICE_TIMEOUT):
        raise DCNv2Error(st, "dcnv2_read_device_error")
    return int(code.value)


def status_string(st: int) -> str:
    return lib.dcnv2_status_string(int(st)).decode()


def timeout_selftest(timeout_us: int):
    code = ctypes.c_int32(0)
    st = lib.dcnv2_diag_timeout_selftest(int(timeout_us), ctypes.byref(code))
    return int(st), int(code.value)


def forward_events_raw(desc: Desc, x, offset, mask, weight, bias, y, workspace, workspace_bytes,
                       x_scale, w_scale, stream, events) -> int:
    """dcnv2_forward with cudaEvent_t handles (ints) recorded around each launch."""
    arr = (ctypes.c_void_p * len(events))(*[int(e) for e in events])
    return int(lib.dcnv2_diag_forward_events(ctypes.byref(desc), x, offset, mask, weight, bias,
                                             y, workspace, workspace_bytes, float(x_scale),
                                             float(w_scale), stream, arr, len(events)))


def forward_static_scratch_raw(desc: Desc, x, offset, mask, weight, bias, y, x_scale=1.0,
                               w_scale=1.0, stream=0) -> int:
    """Raw call of the allocation-free forward (scratch in the library's static buffer)."""
    return int(lib.dcnv2_forward_static_scratch(ctypes.byref(desc), x, offset, mask, weight, bias,
                                                y, float(x_scale), float(w_scale), stream))


def read_static_scratch_error(stream=0) -> int:
    """Error word of the last dcnv2_forward_static_scratch call on the current device."""
    code = ctypes.c_int32(0)
    st = lib.dcnv2_read_static_scratch_error(stream, ctypes.byref(code))
    if st not in (Status.OK, Status.ERR_DEVICE_TIMEOUT):
        raise DCNv2Error(st, "dcnv2_read_static_scratch_error")
    return int(code.value)


class Kernel(enum.IntEnum):
    """Kernel selection of dcnv2_diag_set_kernel_override."""
    AUTO = 0
    TA = 1     # A operand in tensor memory (dcnv2_fused_ta_kernel)
    SMEM = 2   # A operand in shared memory (dcnv2_fused_kernel)


class Pair(enum.IntEnum):
    """CTA-pair selection of dcnv2_diag_set_kernel_override (A-in-shared-memory kernel only)."""
    AUTO = 0     # pairs for tiles of more than 256 output channels
    PAIRS = 1    # every fp16 / int8 tile on a CTA pair (tcgen05 cta_group::2)
    SINGLE = 2   # one CTA per tile


def set_kernel_override(kernel: int = Kernel.AUTO, pair: int = Pair.AUTO) -> None:
    st = lib.dcnv2_diag_set_kernel_override(int(kernel), int(pair))
    if st != Status.OK:
        raise DCNv2Error(st, "dcnv2_diag_set_kernel_override")


def binary_arch() -> int:
    """cudaFuncAttributes::binaryVersion of the library's device code on the current device."""
    v = ctypes.c_int32(0)
    st = lib.dcnv2_diag_binary_arch(ctypes.byref(v))
    if st != Status.OK:
        raise DCNv2Error(st, "dcnv2_diag_binary_arch")
    return int(v.value)


def forward_with_head_workspace_size(desc: Desc) -> int:
    return int(lib.dcnv2_forward_with_head_workspace_size(ctypes.byref(desc)))


def forward_with_head_raw(desc: Desc, x, head_weight, head_bias, weight, bias, y, offset_out,
                          mask_out, workspace, workspace_bytes, stream=0) -> int:
    """Raw call of the layer with its offset / mask head; returns the dcnv2_status value."""
    return int(lib.dcnv2_forward_with_head(ctypes.byref(desc), x, head_weight, head_bias, weight,
                                           bias, y, offset_out, mask_out, workspace,
                                           workspace_bytes, stream))
