"""FP8 MoE expert linear layer with autograd, built on this library's kernels only.

For tokens grouped by expert (group_offs, as everywhere in this package) and weights W [E, K, N]
(bf16 master copy), the layer computes y[off_g:off_{g+1}] = x[off_g:off_{g+1}] @ W[g]:

  forward    x -> e4m3 and W -> e4m3 with one amax scale per expert (quantize_fp8), then the
             fixed-K grouped GEMM with B = W[g] stored [K, N] (trans_b=False)
  backward   dy -> e5m2 per expert (quantize_fp8), then
             dx = dy @ W[g]^T  the fixed-K grouped GEMM with B = W[g] read as [N_out=K, K_red=N]
                               (trans_b=True; the same quantised weights, no transpose copy)
             dW = x^T @ dy     the variable-K grouped wgrad (LHS = x e4m3, RHS = dy e5m2), whose
                               output [E, K, N] is W's own layout

These are the roles the reference harness benchmarks one by one (ggemm-asm bench.py:154-193:
x @ W_gu forward, dy @ W^T data gradient, dW_gu = x^T @ dy weight gradient); here they form one
autograd function. There is no CPU path.
"""
from __future__ import annotations

import torch

from .grouped_fwd import grouped_gemm_fp8_tensorwise
from .grouped_gemm import grouped_gemm_fp8_tensorwise_variable_k
from .quantize import quantize_fp8


def _weight_offsets(E: int, K: int, device) -> torch.Tensor:
    return torch.arange(0, (E + 1) * K, K, dtype=torch.int64, device=device)


class GroupedLinearFP8Function(torch.autograd.Function):
    """y = x @ W[g] per expert in FP8 (see the module docstring). Inputs: x [M, K] bf16,
    w [E, K, N] bf16, group_offs int64 [E + 1] (device). Returns y [M, N] bf16."""

    @staticmethod
    def forward(ctx, x: torch.Tensor, w: torch.Tensor, group_offs: torch.Tensor):
        E, K, N = w.shape
        if x.dim() != 2 or x.shape[1] != K:
            raise ValueError(f"x must be [M, {K}], got {tuple(x.shape)}")
        if group_offs.numel() != E + 1:
            raise ValueError(f"group_offs must have E+1={E + 1} entries")
        xq, sx = quantize_fp8(x.contiguous(), group_offs, "e4m3")
        wq, sw = quantize_fp8(w.contiguous().view(E * K, N), _weight_offsets(E, K, w.device), "e4m3")
        wq = wq.view(E, K, N)
        y = grouped_gemm_fp8_tensorwise(xq, wq, sx, sw, group_offs, trans_b=False)
        ctx.save_for_backward(xq, sx, wq, sw, group_offs)
        return y

    @staticmethod
    def backward(ctx, dy: torch.Tensor):
        xq, sx, wq, sw, group_offs = ctx.saved_tensors
        dyq, sdy = quantize_fp8(dy.contiguous().to(torch.bfloat16), group_offs, "e5m2")
        dx = dw = None
        if ctx.needs_input_grad[0]:
            dx = grouped_gemm_fp8_tensorwise(dyq, wq, sdy, sw, group_offs, trans_b=True)
        if ctx.needs_input_grad[1]:
            dw = grouped_gemm_fp8_tensorwise_variable_k(xq, dyq, sx, sdy, group_offs)
        return dx, dw, None


def grouped_linear_fp8(x: torch.Tensor, w: torch.Tensor, group_offs: torch.Tensor) -> torch.Tensor:
    """Functional form of GroupedLinearFP8Function."""
    return GroupedLinearFP8Function.apply(x, w, group_offs)


class GroupedLinearFP8(torch.nn.Module):
    """E expert weights [E, K, N] (bf16 parameters); forward(x, group_offs) -> y [M, N] bf16."""

    def __init__(self, num_experts: int, in_features: int, out_features: int, device=None):
        super().__init__()
        self.weight = torch.nn.Parameter(
            torch.empty(num_experts, in_features, out_features, dtype=torch.bfloat16,
                        device=device))
        torch.nn.init.normal_(self.weight, std=in_features ** -0.5)

    def forward(self, x: torch.Tensor, group_offs: torch.Tensor) -> torch.Tensor:
        return grouped_linear_fp8(x, self.weight, group_offs)
