"""Python mirror of the dcn::DCNv2 plugin interface, backed by libdcnv2.so.

Method names follow the reference plugin (src/dcn_plugin.cpp of flairziv/tensorrt-dcnv2-plugin):
DCNv2Creator.create_plugin  <- DCNv2Creator::createPlugin        (:222-235)
DCNv2Plugin.get_output_shapes  <- getOutputShapes                (:72-89)
DCNv2Plugin.supports_format_combination <- supportsFormatCombination (:94-104)
DCNv2Plugin.get_output_data_types <- getOutputDataTypes          (:64-68, INT8 -> FLOAT)
DCNv2Plugin.get_workspace_size <- getWorkspaceSize               (:110-118)
DCNv2Plugin.enqueue           <- enqueue                         (:122-176)
DCNv2Plugin.get_fields_to_serialize <- getFieldsToSerialize      (:184-194)
DCNv2Plugin.clone / attach_to_context <- clone / attachToContext (:51-53, :181)

`dcnv2_forward` is the tensor-level convenience used by tests and the benchmark: it takes torch
CUDA tensors, allocates the workspace and output if not given, and calls the C ABI on the
current torch stream.
"""
from __future__ import annotations

import ctypes
from typing import Dict, Optional, Sequence

from . import capi
from .capi import DCNv2Error, DType, FORMAT_LINEAR, Math, Status, TensorDesc, lib

PLUGIN_NAME = "DCNv2"
PLUGIN_VERSION = "1"
PLUGIN_NAMESPACE = ""
FIELD_NAMES = ("stride", "padding", "dilation", "kernel", "deformable_groups")


def tensor_desc(shape: Sequence[int], dtype: int, fmt: int = FORMAT_LINEAR,
                scale: float = 1.0) -> TensorDesc:
    td = TensorDesc()
    td.nb_dims = len(shape)
    for i, v in enumerate(shape):
        td.d[i] = int(v)
    td.type = int(dtype)
    td.format = int(fmt)
    td.scale = float(scale)
    return td


class DCNv2Plugin:
    """One plugin instance (attributes only; no device state)."""

    def __init__(self, handle: int):
        if not handle:
            raise MemoryError("dcnv2_plugin_create failed")
        self._h = ctypes.c_void_p(handle)

    def __del__(self):
        h = getattr(self, "_h", None)
        if h and h.value:
            lib.dcnv2_plugin_destroy(h)
            self._h = None

    # -- IPluginV3OneCore
    def get_plugin_name(self) -> str:
        return lib.dcnv2_plugin_name().decode()

    def get_plugin_version(self) -> str:
        return lib.dcnv2_plugin_version().decode()

    def get_plugin_namespace(self) -> str:
        return lib.dcnv2_plugin_namespace().decode()

    # -- IPluginV3
    def clone(self) -> "DCNv2Plugin":
        return DCNv2Plugin(lib.dcnv2_plugin_clone(self._h))

    def attach_to_context(self, _resource_context=None) -> "DCNv2Plugin":
        return self.clone()

    # -- IPluginV3OneBuild
    def get_nb_outputs(self) -> int:
        return int(lib.dcnv2_plugin_nb_outputs(self._h))

    def get_output_data_types(self, input_types: Sequence[int]):
        return [int(lib.dcnv2_plugin_output_dtype(self._h, int(input_types[0])))]

    def get_output_shapes(self, x_shape: Sequence[int], w_shape: Sequence[int]):
        xs = (ctypes.c_int64 * 4)(*[int(v) for v in x_shape])
        ws = (ctypes.c_int64 * 4)(*[int(v) for v in list(w_shape) + [0] * (4 - len(w_shape))])
        out = (ctypes.c_int64 * 4)()
        st = lib.dcnv2_plugin_output_shape(self._h, xs, ws, out)
        if st != Status.OK:
            raise DCNv2Error(st, "getOutputShapes")
        return [tuple(out)]

    def supports_format_combination(self, pos: int, in_out: Sequence[TensorDesc],
                                     nb_inputs: int = 5, nb_outputs: int = 1) -> bool:
        arr = (TensorDesc * len(in_out))(*in_out)
        return bool(lib.dcnv2_plugin_supports_format(self._h, int(pos), arr, nb_inputs,
                                                     nb_outputs))

    def configure_plugin(self, *_args) -> int:
        return 0

    def get_workspace_size(self, inputs: Sequence[TensorDesc],
                           outputs: Sequence[TensorDesc]) -> int:
        ia = (TensorDesc * len(inputs))(*inputs)
        oa = (TensorDesc * len(outputs))(*outputs)
        return int(lib.dcnv2_plugin_workspace_size(self._h, ia, len(inputs), oa, len(outputs)))

    # -- IPluginV3OneRuntime
    def enqueue(self, input_desc: Sequence[TensorDesc], output_desc: Sequence[TensorDesc],
                inputs: Sequence[int], outputs: Sequence[int], workspace: int,
                workspace_bytes: int, stream: int = 0) -> int:
        ia = (TensorDesc * len(input_desc))(*input_desc)
        oa = (TensorDesc * len(output_desc))(*output_desc)
        ip = (ctypes.c_void_p * len(inputs))(*[int(v) if v else None for v in inputs])
        op = (ctypes.c_void_p * len(outputs))(*[int(v) for v in outputs])
        return int(lib.dcnv2_plugin_enqueue(self._h, ia, oa, ip, op, workspace, workspace_bytes,
                                            stream))

    def on_shape_change(self, *_args) -> int:
        return 0

    def get_fields_to_serialize(self) -> Dict[str, int]:
        names = (ctypes.c_char_p * 5)()
        vals = (ctypes.c_int32 * 5)()
        n = lib.dcnv2_plugin_serialize(self._h, names, vals)
        return {names[i].decode(): int(vals[i]) for i in range(n)}


class DCNv2Creator:
    """IPluginCreatorV3One mirror (src/dcn_plugin.cpp:207-241)."""

    def get_plugin_name(self) -> str:
        return lib.dcnv2_plugin_name().decode()

    def get_plugin_version(self) -> str:
        return lib.dcnv2_plugin_version().decode()

    def get_plugin_namespace(self) -> str:
        return lib.dcnv2_plugin_namespace().decode()

    def get_field_names(self):
        arr = ctypes.POINTER(ctypes.c_char_p)()
        n = lib.dcnv2_plugin_field_names(ctypes.byref(arr))
        return [arr[i].decode() for i in range(n)]

    def create_plugin(self, name: str = PLUGIN_NAME,
                      fields: Optional[Dict[str, Optional[int]]] = None,
                      phase: int = 0) -> DCNv2Plugin:
        fields = fields or {}
        keys = list(fields.keys())
        names = (ctypes.c_char_p * max(1, len(keys)))(*[k.encode() for k in keys])
        holders = [ctypes.c_int32(int(v)) if v is not None else None for v in fields.values()]
        ptrs = (ctypes.POINTER(ctypes.c_int32) * max(1, len(keys)))(
            *[ctypes.pointer(h) if h is not None else ctypes.POINTER(ctypes.c_int32)()
              for h in holders])
        return DCNv2Plugin(lib.dcnv2_plugin_create(names, ptrs, len(keys)))


_TORCH_DTYPES = None


def _dtype_of(t) -> int:
    import torch
    if t.dtype == torch.float32:
        return DType.FLOAT
    if t.dtype == torch.float16:
        return DType.HALF
    if t.dtype == torch.int8:
        return DType.INT8
    raise TypeError(f"unsupported x dtype {t.dtype}")


def dcnv2_forward(x, offset, mask, weight, bias=None, stride: int = 1, padding: int = 1,
                  dilation: int = 1, deformable_groups: int = 1, x_scale: float = 1.0,
                  w_scale: float = 1.0, math: int = Math.DEFAULT, out=None, workspace=None,
                  stream=None):
    """y = DCNv2(x, offset, mask, weight, bias) on the GPU through dcnv2_forward.

    Tensors must be contiguous CUDA tensors of one precision combination: all fp32, all fp16, or
    int8 x/weight with fp32 offset/mask/bias (output fp32). Raises DCNv2Error on any failure.
    """
    import torch
    dt = _dtype_of(x)
    K = int(weight.shape[2])
    N, C, H, W = (int(v) for v in x.shape)
    O = int(weight.shape[0])
    desc = capi.make_desc(N, C, H, W, O, K, stride, padding, dilation, deformable_groups, dt,
                          math)
    n, o, ho, wo = capi.output_shape(desc)
    ydtype = torch.float16 if dt == DType.HALF else torch.float32
    for t in (x, offset, mask, weight) + ((bias,) if bias is not None else ()):
        if not t.is_cuda or not t.is_contiguous():
            raise ValueError("dcnv2_forward expects contiguous CUDA tensors")
    if out is None:
        out = torch.empty((n, o, ho, wo), dtype=ydtype, device=x.device)
    ws_bytes = capi.workspace_size(desc)
    if workspace is None or workspace.numel() < ws_bytes:
        workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=x.device)
    if stream is None:
        stream = torch.cuda.current_stream(x.device).cuda_stream
    st = capi.forward_raw(desc, x.data_ptr(), offset.data_ptr(), mask.data_ptr(),
                          weight.data_ptr(), bias.data_ptr() if bias is not None else None,
                          out.data_ptr(), workspace.data_ptr(), workspace.numel(), x_scale,
                          w_scale, stream)
    if st != Status.OK:
        raise DCNv2Error(st, "dcnv2_forward")
    return out


def dcnv2_forward_host(x, offset, mask, weight, bias=None, stride: int = 1, padding: int = 1,
                       dilation: int = 1, deformable_groups: int = 1, x_scale: float = 1.0,
                       w_scale: float = 1.0, math: int = Math.DEFAULT, out=None, workspace=None,
                       images_per_chunk: int = 0, stream=None, synchronize: bool = True):
    """y = DCNv2(...) with x, offset, mask and y in host memory, through dcnv2_forward_host.

    x, offset and mask are contiguous CPU tensors (page-locked for overlapped copies); weight and
    bias are contiguous CUDA tensors. The batch is uploaded, computed and downloaded in chunks of
    images with the copies overlapped. Returns the host output (pinned when allocated here);
    with synchronize=False it is complete only once `stream` has completed.
    """
    import torch
    dt = _dtype_of(x)
    K = int(weight.shape[2])
    N, C, H, W = (int(v) for v in x.shape)
    O = int(weight.shape[0])
    desc = capi.make_desc(N, C, H, W, O, K, stride, padding, dilation, deformable_groups, dt,
                          math)
    n, o, ho, wo = capi.output_shape(desc)
    ydtype = torch.float16 if dt == DType.HALF else torch.float32
    for t in (x, offset, mask):
        if t.is_cuda or not t.is_contiguous():
            raise ValueError("dcnv2_forward_host expects contiguous host tensors x, offset, mask")
    for t in (weight,) + ((bias,) if bias is not None else ()):
        if not t.is_cuda or not t.is_contiguous():
            raise ValueError("dcnv2_forward_host expects contiguous CUDA weight and bias")
    if out is None:
        out = torch.empty((n, o, ho, wo), dtype=ydtype, pin_memory=True)
    ws_bytes = capi.forward_host_workspace_size(desc, images_per_chunk)
    if ws_bytes == 0:
        raise DCNv2Error(Status.ERR_INVALID_ARG, "dcnv2_forward_host_workspace_size")
    if workspace is None or workspace.numel() < ws_bytes:
        workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=weight.device)
    if stream is None:
        stream = torch.cuda.current_stream(weight.device).cuda_stream
    st = capi.forward_host_raw(desc, x.data_ptr(), offset.data_ptr(), mask.data_ptr(),
                               weight.data_ptr(), bias.data_ptr() if bias is not None else None,
                               out.data_ptr(), workspace.data_ptr(), workspace.numel(), x_scale,
                               w_scale, images_per_chunk, stream)
    if st != Status.OK:
        raise DCNv2Error(st, "dcnv2_forward_host")
    if synchronize:
        torch.cuda.ExternalStream(stream, device=weight.device).synchronize()
    return out


def dcnv2_forward_with_head(x, head_weight, head_bias, weight, bias=None, deformable_groups: int = 1,
                            math: int = Math.DEFAULT, return_offsets: bool = False, out=None,
                            workspace=None, stream=None):
    """The DCNv2 block with its offset / mask head (python/detector.py:44,50-52 of the
    reference): om = conv2d(x, head_weight, head_bias, padding=(K-1)//2), offset = om[:, :2*dg*K*K],
    mask = sigmoid(om[:, 2*dg*K*K:]), y = DCNv2(x, offset, mask, weight, bias), all on the GPU
    through dcnv2_forward_with_head (fp16, stride 1, dilation 1). Returns y, or
    (y, offset, mask) with return_offsets."""
    import torch
    if x.dtype != torch.float16:
        raise TypeError("dcnv2_forward_with_head runs fp16 layers")
    N, C, H, W = (int(v) for v in x.shape)
    O, K = int(weight.shape[0]), int(weight.shape[2])
    desc = capi.make_desc(N, C, H, W, O, K, 1, (K - 1) // 2, 1, deformable_groups, DType.HALF,
                          math)
    tens = (x, head_weight, weight) + tuple(t for t in (head_bias, bias) if t is not None)
    for t in tens:
        if not t.is_cuda or not t.is_contiguous() or t.dtype != torch.float16:
            raise ValueError("dcnv2_forward_with_head expects contiguous fp16 CUDA tensors")
    ws_bytes = capi.forward_with_head_workspace_size(desc)
    if ws_bytes == 0:
        raise DCNv2Error(Status.ERR_UNSUPPORTED, "dcnv2_forward_with_head_workspace_size")
    n, o, ho, wo = capi.output_shape(desc)
    if out is None:
        out = torch.empty((n, o, ho, wo), dtype=torch.float16, device=x.device)
    T = K * K
    off = msk = None
    if return_offsets:
        off = torch.empty((N, 2 * deformable_groups * T, H, W), dtype=torch.float16,
                          device=x.device)
        msk = torch.empty((N, deformable_groups * T, H, W), dtype=torch.float16, device=x.device)
    if workspace is None or workspace.numel() < ws_bytes:
        workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=x.device)
    if stream is None:
        stream = torch.cuda.current_stream(x.device).cuda_stream
    st = capi.forward_with_head_raw(
        desc, x.data_ptr(), head_weight.data_ptr(),
        head_bias.data_ptr() if head_bias is not None else None, weight.data_ptr(),
        bias.data_ptr() if bias is not None else None, out.data_ptr(),
        off.data_ptr() if off is not None else None, msk.data_ptr() if msk is not None else None,
        workspace.data_ptr(), workspace.numel(), stream)
    if st != Status.OK:
        raise DCNv2Error(st, "dcnv2_forward_with_head")
    return (out, off, msk) if return_offsets else out
