"""dragonwing_edge_rs_b200 -- B200 (sm_100a) backend for the fused quantized
convolution path of dragonwing-edge-rs.

``CudaBackend`` mirrors the reference's ``Backend`` trait; ``ops`` holds the op
free functions (reference names and argument order) over the C ABI in
include/dw_cuda.h, implemented by libdragonwing_cuda.so (hand-written CUDA for
sm_100a).  There is no CPU fallback: without the built library or a GPU every
call raises.
"""
from . import ops, quantization
from ._lib import EPI_NONE, EPI_RELU, EPI_RELU6, EPI_SILU, PATH_AUTO, PATH_DIRECT, PATH_UMMA
from ._lib import DWV_AUTO, DWV_SLAB, DWV_STREAM2, DWV_STREAM2X2, DWV_STREAM4
from .backend import BackendError, BufferKind, CudaBackend, CudaBuffer, device_count
from .ops import ConvDesc

__all__ = [
    "BackendError", "BufferKind", "CudaBackend", "CudaBuffer", "ConvDesc", "device_count", "ops", "quantization",
    "EPI_NONE", "EPI_RELU", "EPI_RELU6", "EPI_SILU", "PATH_AUTO", "PATH_DIRECT", "PATH_UMMA", "DWV_AUTO", "DWV_SLAB", "DWV_STREAM2", "DWV_STREAM2X2", "DWV_STREAM4",
]
