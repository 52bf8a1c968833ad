"""The library's kernels as torch operators (namespace ``ggemm``), registered with torch.library.

    torch.ops.ggemm.variable_k_wgrad(lhs, rhs, lhs_scale, rhs_scale, group_offs) -> out
        out[g] = sL_g * sR_g * lhs[off_g:off_{g+1}]^T @ rhs[off_g:off_{g+1}], bf16 [G, OUT_M, OUT_N]
        (the call the reference harness makes into Primus-Turbo, ggemm-asm bench.py:268)
    torch.ops.ggemm.grouped_fp8_fwd(a, b, a_scale, b_scale, group_offs, trans_b) -> out
        the fixed-K grouped GEMM of the forward / data-gradient sites, bf16 [M, N]
        (bench.py:154-181, 241-260)
    torch.ops.ggemm.quantize_fp8(x, group_offs, fmt, per_group) -> (q, scales)
        the producer step: per-expert (or per-tensor) amax scaling and fp8 quantisation

Each operator has a fake implementation that produces the output's shape, dtype and device
without running anything, so code built from them traces under FakeTensorMode, torch.compile
and torch.export, and the FP8 MoE layer (moe.GroupedLinearFP8Function, built on these operators)
traces through its forward and backward. The real implementation calls the C ABI on the current
CUDA stream; there is no CPU implementation (CPU tensors raise, as the plain functions do).
The plain functions (grouped_gemm_fp8_tensorwise_variable_k, grouped_gemm_fp8_tensorwise,
quantize_fp8) go through these operators whenever they are called without their eager-only
extras (``out=``, a path override, a caller status block).
"""
from __future__ import annotations

import torch

from .grouped_fwd import _grouped_fwd
from .grouped_gemm import _variable_k_wgrad
from .quantize import FORMATS, _quantize_fp8


@torch.library.custom_op("ggemm::variable_k_wgrad", mutates_args=())
def variable_k_wgrad(lhs: torch.Tensor, rhs: torch.Tensor, lhs_scale: torch.Tensor,
                     rhs_scale: torch.Tensor, group_offs: torch.Tensor) -> torch.Tensor:
    return _variable_k_wgrad(lhs, rhs, lhs_scale, rhs_scale, group_offs)


@variable_k_wgrad.register_fake
def _(lhs, rhs, lhs_scale, rhs_scale, group_offs):
    G = group_offs.shape[0] - 1
    return lhs.new_empty((G, lhs.shape[1], rhs.shape[1]), dtype=torch.bfloat16)


@torch.library.custom_op("ggemm::grouped_fp8_fwd", mutates_args=())
def grouped_fp8_fwd(a: torch.Tensor, b: torch.Tensor, a_scale: torch.Tensor,
                    b_scale: torch.Tensor, group_offs: torch.Tensor,
                    trans_b: bool) -> torch.Tensor:
    return _grouped_fwd(a, b, a_scale, b_scale, group_offs, trans_b)


@grouped_fp8_fwd.register_fake
def _(a, b, a_scale, b_scale, group_offs, trans_b):
    N = b.shape[1] if trans_b else b.shape[2]
    return a.new_empty((a.shape[0], N), dtype=torch.bfloat16)


@torch.library.custom_op("ggemm::quantize_fp8", mutates_args=())
def quantize_fp8(x: torch.Tensor, group_offs: torch.Tensor, fmt: str,
                 per_group: bool) -> tuple[torch.Tensor, torch.Tensor]:
    return _quantize_fp8(x, group_offs, fmt, "group" if per_group else "tensor")


@quantize_fp8.register_fake
def _(x, group_offs, fmt, per_group):
    units = group_offs.shape[0] - 1 if per_group else 1
    q = x.new_empty(x.shape, dtype=FORMATS[fmt][1])
    return q, x.new_empty((max(units, 1),), dtype=torch.float32)
