"""dcnv2_b200 — sm_100a DCNv2 forward behind the dcn::DCNv2 plugin interface.

The first call into the library maps libdcnv2.so (built by __graft_entry__.build()); that call
raises ImportError if the library is missing, so no caller can silently run without the CUDA
kernels. Importing the package alone (e.g. for the seeded workload generators) maps nothing.
"""
from .capi import DCNv2Error, DType, Math, Status, LIB_PATH  # noqa: F401
from .plugin import (DCNv2Creator, DCNv2Plugin, FIELD_NAMES, PLUGIN_NAME,  # noqa: F401
                     PLUGIN_NAMESPACE, PLUGIN_VERSION, dcnv2_forward, dcnv2_forward_host,
                     dcnv2_forward_with_head, tensor_desc)

__all__ = ["DCNv2Error", "DType", "Math", "Status", "DCNv2Creator", "DCNv2Plugin",
           "dcnv2_forward", "dcnv2_forward_host", "dcnv2_forward_with_head", "tensor_desc", "PLUGIN_NAME", "PLUGIN_VERSION", "PLUGIN_NAMESPACE",
           "FIELD_NAMES", "LIB_PATH"]
