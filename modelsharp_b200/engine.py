"""A node-loop engine over the kernel registry, with the reference engine's run contract.

ManagedCpuEngine.Run (src/ModelSharp/Cpu/ManagedCpuEngine.cs:36-84): seed the environment
with the graph's initializers, then the caller's feeds (a missing feed is an error), run the
nodes in order through the registry by op type (an unknown op type is an error), and return
the requested outputs. Here the registry's kernels are the CUDA ones, so a graph whose
MatMulNBits nodes come from an ONNX export dispatches them to libms_cuda_nbits.so unchanged.
"""
from __future__ import annotations

from .errors import ModelSharpException
from .kernels import GraphContext, KernelRegistry, ModelGraph


class UnsupportedOperatorException(ModelSharpException):
    def __init__(self, op_type: str, where: str):
        super().__init__(f"Operator '{op_type}' is not supported ({where}).")
        self.op_type = op_type


class CudaEngine:
    """preload=True packs every MatMulNBits node's weight initializers on the device when the
    engine is built (load time) instead of on the node's first run."""

    def __init__(self, graph: ModelGraph, kernels: KernelRegistry | None = None, device=None,
                 preload: bool = False):
        if graph is None:
            raise ValueError("graph")
        self.graph = graph
        self.kernels = kernels or KernelRegistry.create_default(device)
        self.preloaded = 0
        if preload:
            from .onnx_loader import preload_matmulnbits
            ok, k = self.kernels.try_get("MatMulNBits")
            if ok and hasattr(k, "preload"):
                self.preloaded = preload_matmulnbits(graph, k, device)

    def run(self, feeds: dict) -> dict:
        env = dict(self.graph.initializers)
        for name in self.graph.inputs:
            if name not in feeds:
                raise ModelSharpException(f"Missing feed for required input '{name}'.")
            env[name] = feeds[name]
        ctx = GraphContext(env)
        for node in self.graph.nodes:
            ok, kernel = self.kernels.try_get(node.op_type)
            if not ok or kernel is None:
                raise UnsupportedOperatorException(node.op_type, f"node '{node.name}'")
            kernel.execute(node, ctx)
        return {name: ctx.values[name] for name in self.graph.outputs}
