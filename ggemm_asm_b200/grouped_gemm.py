"""PyTorch-facing API of the variable-K grouped FP8 wgrad.

``grouped_gemm_fp8_tensorwise_variable_k`` mirrors the call the reference harness makes into
Primus-Turbo, ``grouped_gemm_fp8_tensorwise_variable_k_triton_kernel(lhs, rhs, lhs_scale,
rhs_scale, group_offs) -> out`` (ggemm-asm bench.py:241-246, 268, 745): same argument order and
meaning, returns a freshly allocated ``[G, OUT_M, OUT_N]`` bf16 tensor (or fills ``out``).
It calls the C ABI (``ggemm_vark_fp8_wgrad_ex``) on the current CUDA stream; there is no
fallback path: a missing library or a non-sm_100 device raises.
"""
from __future__ import annotations

import torch

from . import _lib

LHS_DTYPE = torch.float8_e4m3fn
RHS_DTYPE = torch.float8_e5m2

_PATHS = {"auto": _lib.PATH_AUTO, "tcgen05": _lib.PATH_TCGEN05, "simt": _lib.PATH_SIMT,
          "tcgen05_1sm": _lib.PATH_TCGEN05_1SM}


def _check_inputs(lhs, rhs, lhs_scale, rhs_scale, group_offs):
    if not (isinstance(lhs, torch.Tensor) and isinstance(rhs, torch.Tensor)):
        raise TypeError("lhs and rhs must be tensors")
    if lhs.dtype != LHS_DTYPE or rhs.dtype != RHS_DTYPE:
        raise TypeError(f"expected lhs {LHS_DTYPE} and rhs {RHS_DTYPE}, got {lhs.dtype} and {rhs.dtype}")
    if lhs.dim() != 2 or rhs.dim() != 2:
        raise ValueError("lhs and rhs must be 2-D [tokens, features]")
    if lhs.shape[0] != rhs.shape[0]:
        raise ValueError(f"lhs and rhs token counts differ: {lhs.shape[0]} vs {rhs.shape[0]}")
    if lhs.stride(1) != 1 or rhs.stride(1) != 1:
        raise ValueError("lhs and rhs rows must be contiguous (stride(1) == 1)")
    if group_offs.dtype != torch.int64 or group_offs.dim() != 1 or group_offs.numel() < 1:
        raise ValueError("group_offs must be a 1-D int64 tensor of G+1 prefix sums")
    G = group_offs.numel() - 1
    if lhs_scale.dtype != torch.float32 or rhs_scale.dtype != torch.float32:
        raise TypeError("scales must be float32")
    if lhs_scale.numel() != rhs_scale.numel():
        raise ValueError("lhs_scale and rhs_scale must have the same number of elements")
    if lhs_scale.numel() == 1:
        scale_stride = 0
    elif lhs_scale.numel() == G:
        scale_stride = 1
    else:
        raise ValueError(f"scales must have 1 (tensorwise) or G={G} (per-group) elements")
    if not (lhs_scale.is_contiguous() and rhs_scale.is_contiguous() and group_offs.is_contiguous()):
        raise ValueError("scales and group_offs must be contiguous")
    for name, v in (("G", G), ("OUT_M", lhs.shape[1]), ("OUT_N", rhs.shape[1]),
                    ("stride_lhs_m", lhs.stride(0)), ("stride_rhs_m", rhs.stride(0))):
        if v >= 2**31:
            raise ValueError(f"{name}={v} does not fit the int32 ABI")
    dev = lhs.device
    if dev.type != "cuda":
        raise ValueError("inputs must be CUDA tensors (no CPU path)")
    for name, t in (("rhs", rhs), ("lhs_scale", lhs_scale), ("rhs_scale", rhs_scale),
                    ("group_offs", group_offs)):
        if t.device != dev:
            raise ValueError(f"{name} is on {t.device}, expected {dev}")
    return G, scale_stride


def grouped_gemm_fp8_tensorwise_variable_k(lhs: torch.Tensor, rhs: torch.Tensor,
                                           lhs_scale: torch.Tensor, rhs_scale: torch.Tensor,
                                           group_offs: torch.Tensor,
                                           out: torch.Tensor | None = None, *,
                                           path: str = "auto",
                                           status: torch.Tensor | None = None) -> torch.Tensor:
    """C[g] = lhs_scale * rhs_scale * lhs[off_g:off_g+1].T @ rhs[off_g:off_g+1], bf16.

    lhs: [M_total, OUT_M] float8_e4m3fn, rhs: [M_total, OUT_N] float8_e5m2 (token-major),
    lhs_scale / rhs_scale: float32 with 1 element (tensorwise, as the reference) or G elements
    (per group), group_offs: int64 [G+1]. ``out`` (optional) is a [G, OUT_M, OUT_N] bf16 tensor
    with contiguous rows; it is overwritten. ``path`` selects "auto" | "tcgen05" (CTA pairs) |
    "tcgen05_1sm" (single CTA) | "simt".
    ``status``: optional int32 CUDA tensor of >= 64 elements used as the device status block.
    Called without ``out``, ``path`` or ``status`` it runs as the registered operator
    torch.ops.ggemm.variable_k_wgrad (traceable; see ops.py).
    """
    if out is None and path == "auto" and status is None:
        from . import ops

        return ops.variable_k_wgrad(lhs, rhs, lhs_scale, rhs_scale, group_offs)
    return _variable_k_wgrad(lhs, rhs, lhs_scale, rhs_scale, group_offs, out, path, status)


def _variable_k_wgrad(lhs, rhs, lhs_scale, rhs_scale, group_offs, out=None, path="auto",
                      status=None) -> torch.Tensor:
    """The C-ABI call behind grouped_gemm_fp8_tensorwise_variable_k and its operator."""
    G, scale_stride = _check_inputs(lhs, rhs, lhs_scale, rhs_scale, group_offs)
    OUT_M, OUT_N = lhs.shape[1], rhs.shape[1]
    if out is None:
        out = torch.empty((G, OUT_M, OUT_N), dtype=torch.bfloat16, device=lhs.device)
    else:
        if out.dtype != torch.bfloat16 or tuple(out.shape) != (G, OUT_M, OUT_N):
            raise ValueError(f"out must be bf16 of shape {(G, OUT_M, OUT_N)}")
        if out.device != lhs.device:
            raise ValueError("out must be on the inputs' device")
        if any(s <= 0 for s in out.stride()):
            raise ValueError("out strides must be positive")
    if G == 0:
        return out
    if path not in _PATHS:
        raise ValueError(f"path must be one of {sorted(_PATHS)}")
    status_ptr = None
    if status is not None:
        if status.device != lhs.device or status.numel() * status.element_size() < 256:
            raise ValueError("status must be a >= 256-byte tensor on the inputs' device")
        status_ptr = status.data_ptr()
    with torch.cuda.device(lhs.device):
        stream = torch.cuda.current_stream(lhs.device).cuda_stream
        rc = _lib.lib().ggemm_vark_fp8_wgrad_ex(
            lhs.data_ptr(), rhs.data_ptr(), out.data_ptr(),
            lhs_scale.data_ptr(), rhs_scale.data_ptr(), group_offs.data_ptr(),
            G, OUT_M, OUT_N, lhs.stride(0), rhs.stride(0),
            out.stride(0), out.stride(1), out.stride(2),
            lhs.shape[0], scale_stride, _PATHS[path], status_ptr, 0, stream)
    _lib.check(rc, "grouped_gemm_fp8_tensorwise_variable_k")
    return out


# Short alias used by the MoE backward integration and the benchmarks.
variable_k_wgrad = grouped_gemm_fp8_tensorwise_variable_k


def launch_raw(lhs_ptr: int, rhs_ptr: int, c_ptr: int, lhs_scale_ptr: int, rhs_scale_ptr: int,
               group_offs_ptr: int, G: int, OUT_M: int, OUT_N: int, stride_lhs_m: int,
               stride_rhs_m: int, stride_cg: int, stride_cm: int, stride_cn: int,
               stream: int = 0) -> None:
    """The 14-argument drop-in entry point (ggemm_vark_fp8_wgrad) with raw device pointers,
    argument for argument as the reference packs its kernel arguments (bench.py:376-385)."""
    rc = _lib.lib().ggemm_vark_fp8_wgrad(lhs_ptr, rhs_ptr, c_ptr, lhs_scale_ptr, rhs_scale_ptr,
                                         group_offs_ptr, G, OUT_M, OUT_N, stride_lhs_m,
                                         stride_rhs_m, stride_cg, stride_cm, stride_cn, stream)
    _lib.check(rc, "ggemm_vark_fp8_wgrad")


def flops(group_offs_or_mtotal, OUT_M: int, OUT_N: int) -> float:
    """Algorithmic FLOP count 2 * M_total * OUT_M * OUT_N (launcher.cpp:76, bench.py:742)."""
    if isinstance(group_offs_or_mtotal, torch.Tensor):
        m_total = int(group_offs_or_mtotal[-1] - group_offs_or_mtotal[0])
    else:
        m_total = int(group_offs_or_mtotal)
    return 2.0 * m_total * OUT_M * OUT_N
