"""B200-native (sm_100a) backend for ModelSharp's com.microsoft.MatMulNBits operator.

The compute lives in libms_cuda_nbits.so (C ABI: include/ms_cuda_nbits.h); this package is
the host-side mirror of the reference's operator plugin API plus the multi-GPU column split.
"""
from .errors import ModelSharpException
from .kernels import CudaMatMulNBitsKernel, GraphContext, GraphNode, IKernel, KernelRegistry, ModelGraph
from .engine import CudaEngine, UnsupportedOperatorException
from .weights import QuantizedWeights

__all__ = [
    "ModelSharpException", "CudaMatMulNBitsKernel", "GraphContext", "GraphNode", "IKernel", "KernelRegistry",
    "ModelGraph", "CudaEngine", "UnsupportedOperatorException", "QuantizedWeights",
]
