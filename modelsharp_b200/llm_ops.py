"""CUDA kernels for the op types of an INT4 decoder graph, behind the plugin API.

With these registered beside MatMulNBits, the engine's node loop (CudaEngine.run, the
contract of ManagedCpuEngine.Run) runs a Llama-shaped decoder graph one token at a time with
every value on the device. Op types, inputs, outputs and attributes follow the reference's
CPU kernels:

* Gather                          ShapeOps.cs:54 (an embedding-row lookup: data [V, H],
                                  int64 indices)
* SimplifiedLayerNormalization    SimplifiedLayerNormalizationKernel.cs:19-64 (epsilon, last
                                  axis): msq_add_rmsnorm
* SkipSimplifiedLayerNormalization SkipSimplifiedLayerNormalizationKernel.cs:24-86 (outputs
                                  [output, mean, inv_std_var, input_skip_bias_sum]; beta and
                                  bias inputs are not supported here): msq_add_rmsnorm
* GroupQueryAttention             GroupQueryAttentionKernel.cs:55-202 (packed QKV, do_rotary,
                                  cos_cache / sin_cache, seqlens_k): msq_rope_gqa_decode, and
                                  for a prompt msq_rope_append_rows + msq_gqa_prefill
* Sigmoid, Mul                    SigmoidKernel.cs:11, MulKernel.cs:8 (same-shape operands)
* ArgMax                          ArgReduceKernels.cs:77 (last axis): msq_argmax

GroupQueryAttention takes batch 1, packed QKV, rotary in the op, and past_key / past_value
preallocated to [1, kv_num_heads, max_seq, head_dim] and shared with present_key /
present_value: the tokens' rotated k and v are written into the past buffers (rows up to
seqlens_k) and the present outputs are those buffers. One query token runs as one
msq_rope_gqa_decode launch; several (a prompt ending at seqlens_k) as msq_rope_append_rows and
msq_gqa_prefill. (The reference
returns a fresh concatenated present each step; sharing the buffer keeps a decode step free
of per-token copies of the cache.) Inputs outside these forms raise ModelSharpException.
"""
from __future__ import annotations

import math

import torch

from . import _native as N
from .errors import ModelSharpException
from .kernels import CudaMatMulNBitsKernel, GraphContext, GraphNode, KernelRegistry


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _cuda_f32(ctx: GraphContext, name: str, op: str) -> torch.Tensor:
    t = ctx.get(name)
    if not t.is_cuda:
        raise ModelSharpException(f"{op}: input '{name}' must be on the CUDA device.")
    if t.dtype != torch.float32:
        t = t.float()
    return t.contiguous()


def _ok(rc: int, what: str) -> None:
    if rc != N.MSQ_OK:
        N.check(rc, what)


def _attr(node: GraphNode, name: str, default):
    return node.attributes.get(name, default)


class GatherKernel:
    """Rows of data [V, H] selected by int64 indices of any shape -> indices.shape + [H]."""

    op_type = "Gather"

    def execute(self, node: GraphNode, ctx: GraphContext) -> None:
        data = ctx.get_tensor(node.inputs[0])
        idx = ctx.get_tensor(node.inputs[1])
        if int(_attr(node, "axis", 0)) != 0 or data.dim() != 2:
            raise ModelSharpException("Gather: only axis 0 of a 2-D table is supported on this backend.")
        flat = idx.reshape(-1).to(torch.int64)
        out = torch.index_select(data, 0, flat)
        ctx.set(node.outputs[0], out.reshape(*idx.shape, data.shape[1]))


class SimplifiedLayerNormalizationKernel:
    op_type = "SimplifiedLayerNormalization"

    def execute(self, node: GraphNode, ctx: GraphContext) -> None:
        x = _cuda_f32(ctx, node.inputs[0], self.op_type)
        gamma = _cuda_f32(ctx, node.inputs[1], self.op_type)
        if int(_attr(node, "axis", -1)) not in (-1, x.dim() - 1):
            raise ModelSharpException("SimplifiedLayerNormalization: only the last axis is supported.")
        n = x.shape[-1]
        if gamma.numel() != n:
            raise ModelSharpException(f"SimplifiedLayerNormalization: scale has {gamma.numel()} values, expected {n}.")
        y = torch.empty_like(x)
        _ok(N.lib().msq_add_rmsnorm(None, _stream(x), x.data_ptr(), None, gamma.data_ptr(), y.data_ptr(),
                                    x.numel() // n, n, float(_attr(node, "epsilon", 1e-5))), self.op_type)
        ctx.set(node.outputs[0], y)


class SkipSimplifiedLayerNormalizationKernel:
    op_type = "SkipSimplifiedLayerNormalization"

    def execute(self, node: GraphNode, ctx: GraphContext) -> None:
        if (len(node.inputs) > 3 and node.inputs[3]) or (len(node.inputs) > 4 and node.inputs[4]):
            raise ModelSharpException("SkipSimplifiedLayerNormalization: beta / bias inputs are not supported.")
        if len(node.outputs) > 1 and any(node.outputs[1:3]):
            raise ModelSharpException("SkipSimplifiedLayerNormalization: mean / inv_std_var outputs are not supported.")
        x = _cuda_f32(ctx, node.inputs[0], self.op_type)
        skip = _cuda_f32(ctx, node.inputs[1], self.op_type)
        gamma = _cuda_f32(ctx, node.inputs[2], self.op_type)
        if skip.shape != x.shape:
            raise ModelSharpException(f"SkipSimplifiedLayerNormalization: skip shape {tuple(skip.shape)} "
                                      f"differs from input {tuple(x.shape)}.")
        n = x.shape[-1]
        s = x.clone()  # input + skip lands here; the graph's input value stays as it was
        y = torch.empty_like(x)
        _ok(N.lib().msq_add_rmsnorm(None, _stream(x), s.data_ptr(), skip.data_ptr(), gamma.data_ptr(), y.data_ptr(),
                                    x.numel() // n, n, float(_attr(node, "epsilon", 1e-5))), self.op_type)
        ctx.set(node.outputs[0], y)
        if len(node.outputs) > 3 and node.outputs[3]:
            ctx.set(node.outputs[3], s)


class GroupQueryAttentionKernel:
    op_type = "GroupQueryAttention"

    def execute(self, node: GraphNode, ctx: GraphContext) -> None:
        op = self.op_type
        heads, kvh = int(_attr(node, "num_heads", 0)), int(_attr(node, "kv_num_heads", 0))
        if heads <= 0 or kvh <= 0:
            raise ModelSharpException(f"{op}: num_heads and kv_num_heads must be positive.")
        ins = list(node.inputs) + [""] * (9 - len(node.inputs))
        if ins[1] or ins[2]:
            raise ModelSharpException(f"{op}: only packed QKV (empty key / value inputs) is supported here.")
        if int(_attr(node, "do_rotary", 0)) != 1 or int(_attr(node, "rotary_interleaved", 0)) != 0:
            raise ModelSharpException(f"{op}: the decode form needs do_rotary=1 with half-split rotary.")
        if int(_attr(node, "local_window_size", -1)) != -1:
            raise ModelSharpException(f"{op}: local_window_size is not supported here.")
        if not (ins[3] and ins[4] and ins[5] and ins[7] and ins[8]):
            raise ModelSharpException(f"{op}: past_key, past_value, seqlens_k, cos_cache and sin_cache are required.")
        qkv = _cuda_f32(ctx, ins[0], op)
        if qkv.dim() != 3 or qkv.shape[0] != 1:
            raise ModelSharpException(f"{op}: batch 1 query [1, S, hidden] only; got {list(qkv.shape)}.")
        unit = heads + 2 * kvh
        if qkv.shape[2] % unit:
            raise ModelSharpException(f"GroupQueryAttention packed-QKV hidden {qkv.shape[2]} not divisible by "
                                      f"(num_heads + 2·kv_num_heads) = {unit}.")
        d = qkv.shape[2] // unit
        scale = float(_attr(node, "scale", 0.0))
        if scale != 0.0 and not math.isclose(scale, 1.0 / math.sqrt(d), rel_tol=1e-6):
            raise ModelSharpException(f"{op}: only the default 1/sqrt(head_dim) scale is supported.")
        pk, pv = ctx.get_tensor(ins[3]), ctx.get_tensor(ins[4])
        for name, t in ((ins[3], pk), (ins[4], pv)):
            if (not t.is_cuda or t.dtype != torch.float32 or t.dim() != 4 or t.shape[0] != 1 or t.shape[1] != kvh
                    or t.shape[3] != d or not t.is_contiguous()):
                raise ModelSharpException(f"{op}: '{name}' must be a contiguous float32 CUDA buffer "
                                          f"[1, {kvh}, max_seq, {d}].")
        max_seq = pk.shape[2]
        if pv.shape[2] != max_seq:
            raise ModelSharpException(f"{op}: past_key and past_value lengths differ.")
        cos, sin = _cuda_f32(ctx, ins[7], op), _cuda_f32(ctx, ins[8], op)
        if cos.shape != (max_seq, d // 2) or sin.shape != (max_seq, d // 2):
            raise ModelSharpException(f"{op}: cos_cache / sin_cache must be [{max_seq}, {d // 2}].")
        pos = ctx.get_tensor(ins[5])
        if not pos.is_cuda or pos.numel() != 1:
            raise ModelSharpException(f"{op}: seqlens_k must be one index on the CUDA device.")
        if pos.dtype != torch.int64:
            pos = pos.to(torch.int64)
        if qkv.shape[1] > 1:
            out = self._prompt(qkv, pos, pk, pv, cos, sin, heads, kvh, d, max_seq)
        else:
            out = torch.empty(1, 1, heads * d, dtype=torch.float32, device=qkv.device)
            _ok(N.lib().msq_rope_gqa_decode(None, _stream(qkv), qkv.data_ptr(), heads, kvh, d, cos.data_ptr(),
                                            sin.data_ptr(), pos.data_ptr(), pk.data_ptr(), pv.data_ptr(),
                                            out.data_ptr(), max_seq), op)
        ctx.set(node.outputs[0], out)
        if len(node.outputs) > 1 and node.outputs[1]:
            ctx.set(node.outputs[1], pk)
        if len(node.outputs) > 2 and node.outputs[2]:
            ctx.set(node.outputs[2], pv)


    @staticmethod
    def _prompt(qkv, pos, pk, pv, cos, sin, heads, kvh, d, max_seq):
        """S > 1 query tokens ending at position seqlens_k (a prompt): half-split rotary of q and k
        at positions p0..p0+S-1 with k and v appended to the cache (msq_rope_append_rows, qkv left
        unchanged), then causal attention of each query over cache rows 0..its position with the
        1/sqrt(d) scale (msq_gqa_prefill). Reads seqlens_k on the host."""
        S = qkv.shape[1]
        last = int(pos.reshape(-1)[0])
        p0 = last - S + 1
        if p0 < 0 or last >= max_seq:
            raise ModelSharpException(f"GroupQueryAttention: {S} query tokens ending at position {last} do not fit "
                                      f"a cache of {max_seq}.")
        st = _stream(qkv)
        q = torch.empty(S, heads * d, dtype=torch.float32, device=qkv.device)
        _ok(N.lib().msq_rope_append_rows(None, st, qkv.data_ptr(), S, p0, heads, kvh, d, cos.data_ptr(),
                                         sin.data_ptr(), q.data_ptr(), pk.data_ptr(), pv.data_ptr(), max_seq),
            "GroupQueryAttention")
        out = torch.empty(1, S, heads * d, dtype=torch.float32, device=qkv.device)
        _ok(N.lib().msq_gqa_prefill(None, st, q.data_ptr(), pk.data_ptr(), pv.data_ptr(), S, p0, out.data_ptr(), heads,
                                    kvh, d, max_seq), "GroupQueryAttention")
        return out


class SigmoidKernel:
    op_type = "Sigmoid"

    def execute(self, node: GraphNode, ctx: GraphContext) -> None:
        ctx.set(node.outputs[0], torch.sigmoid(_cuda_f32(ctx, node.inputs[0], self.op_type)))


class MulKernel:
    op_type = "Mul"

    def execute(self, node: GraphNode, ctx: GraphContext) -> None:
        a = _cuda_f32(ctx, node.inputs[0], self.op_type)
        b = _cuda_f32(ctx, node.inputs[1], self.op_type)
        if a.shape != b.shape:
            raise ModelSharpException(f"Mul: shapes {list(a.shape)} and {list(b.shape)} differ "
                                      "(broadcasting is not supported on this backend).")
        ctx.set(node.outputs[0], a * b)


class ArgMaxKernel:
    """Index of the first maximum along the last axis (int64), keepdims as the attribute says:
    msq_argmax for one row, torch.argmax for several."""

    op_type = "ArgMax"

    def execute(self, node: GraphNode, ctx: GraphContext) -> None:
        x = _cuda_f32(ctx, node.inputs[0], self.op_type)
        if int(_attr(node, "axis", 0)) not in (-1, x.dim() - 1):
            raise ModelSharpException("ArgMax: only the last axis is supported on this backend.")
        if int(_attr(node, "select_last_index", 0)) != 0:
            raise ModelSharpException("ArgMax: select_last_index is not supported.")
        n = x.shape[-1]
        rows = x.numel() // n
        if rows == 1:
            idx = torch.empty(1, dtype=torch.int64, device=x.device)
            _ok(N.lib().msq_argmax(None, _stream(x), x.data_ptr(), n, idx.data_ptr(), None), "ArgMax")
        else:  # a prompt's rows at once (torch also returns the first maximum)
            idx = torch.argmax(x.reshape(rows, n), dim=1)
        shape = list(x.shape[:-1]) + ([1] if int(_attr(node, "keepdims", 1)) else [])
        ctx.set(node.outputs[0], idx.reshape(shape))


class MatMulNBitsFusedKernel(CudaMatMulNBitsKernel):
    """MatMulNBits with decode-step glue folded in, the node graph_fusion writes.

    Inputs [A, B, scales, zero_points, gamma, residual] (gamma and residual optional), attributes
    of MatMulNBits plus `swiglu` and `epsilon`. With gamma, A rows are RMSNorm inputs (the norm is
    applied on the way in); with swiglu=1, A rows are [gate | up] of 2K and the product uses
    silu(gate) * up; with residual, the product is added into that tensor in place (the fusion
    pass proves no later node reads its old value) and the node's output is that tensor. Up to
    16 rows of fp32 A run as one msq_matmul_fused launch; larger M (a prompt) runs the same steps
    unfused (msq_add_rmsnorm or msq_swiglu_rows, the MatMulNBits path of the registry, a torch
    add into the residual)."""

    op_type = "MatMulNBitsFused"

    def execute(self, node: GraphNode, ctx: GraphContext) -> None:
        ins = list(node.inputs) + [""] * (6 - len(node.inputs))
        n, k = int(node.attributes["N"]), int(node.attributes["K"])
        bits, bs = int(node.attributes.get("bits", 4)), int(node.attributes.get("block_size", 0))
        swiglu = int(node.attributes.get("swiglu", 0))
        eps = float(node.attributes.get("epsilon", 1e-5))
        a = _cuda_f32(ctx, ins[0], self.op_type)
        kin = 2 * k if swiglu else k
        if a.shape[-1] != kin:
            raise ModelSharpException(f"MatMulNBitsFused: A rows of {a.shape[-1]}, expected {kin}.")
        m = a.numel() // kin
        gamma = _cuda_f32(ctx, ins[4], self.op_type) if ins[4] else None
        if gamma is not None and swiglu:
            raise ModelSharpException("MatMulNBitsFused: gamma and swiglu are exclusive.")
        zp_raw = ctx.get_tensor(ins[3]) if ins[3] else None
        w = self._weights(ctx.get_tensor(ins[1]), ctx.get_tensor(ins[2]), zp_raw, n, k, bits, bs, a.device)
        self.calls += 1
        if ins[5]:
            out = ctx.get_tensor(ins[5])
            if not out.is_cuda or out.dtype != torch.float32 or not out.is_contiguous() or out.numel() != m * n:
                raise ModelSharpException("MatMulNBitsFused: the residual must be a contiguous float32 CUDA "
                                          f"tensor of {m} x {n}.")
        else:
            out = torch.empty(*a.shape[:-1], n, dtype=torch.float32, device=a.device)
        a2, o2 = a.reshape(m, kin), out.view(m, n)
        aligned = k % 4 == 0 and a2.data_ptr() % 16 == 0 and (gamma is None or gamma.data_ptr() % 16 == 0)
        if m <= 16 and aligned and bits == 4 and bs in (32, 64, 128):  # the decode GEMV's forms
            w.matmul_fused(a2, o2, rms_gamma=gamma, rms_eps=eps, swiglu=bool(swiglu), accumulate=bool(ins[5]),
                           stream=_stream(a))
        else:
            x = a2
            if gamma is not None:
                x = torch.empty_like(a2)
                _ok(N.lib().msq_add_rmsnorm(None, _stream(a), a2.data_ptr(), None, gamma.data_ptr(), x.data_ptr(),
                                            m, k, eps), self.op_type)
            elif swiglu:
                x = torch.empty(m, k, dtype=torch.float32, device=a.device)
                _ok(N.lib().msq_swiglu_rows(None, _stream(a), a2.data_ptr(), x.data_ptr(), m, k), self.op_type)
            y = w.matmul(x, path=self.path)
            if ins[5]:
                o2.add_(y)
            else:
                o2.copy_(y)
        ctx.set(node.outputs[0], out)


def create_decoder_registry(device=None, path: int = N.PATH_AUTO_SPLIT) -> KernelRegistry:
    """The CUDA registry with MatMulNBits (plain and fused) and the decoder graph's other op
    types. `path` pins the MatMulNBits route (PATH_GEMV: the exact decode GEMV for every M)."""
    reg = KernelRegistry().register(CudaMatMulNBitsKernel(device, path)).register(MatMulNBitsFusedKernel(device, path))
    for k in (GatherKernel(), SimplifiedLayerNormalizationKernel(), SkipSimplifiedLayerNormalizationKernel(),
              GroupQueryAttentionKernel(), SigmoidKernel(), MulKernel(), ArgMaxKernel()):
        reg.register(k)
    return reg


__all__ = ["create_decoder_registry", "MatMulNBitsFusedKernel", "GatherKernel", "SimplifiedLayerNormalizationKernel",
           "SkipSimplifiedLayerNormalizationKernel", "GroupQueryAttentionKernel", "SigmoidKernel", "MulKernel",
           "ArgMaxKernel"]
