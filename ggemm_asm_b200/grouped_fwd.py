"""PyTorch-facing API of the fixed-K grouped FP8 GEMM (MoE forward and data-gradient sites).

``grouped_gemm_fp8_tensorwise(a, b, a_scale, b_scale, group_offs, trans_b=True)`` mirrors the
call the reference harness makes into Primus-Turbo, ``grouped_gemm_fp8_tensorwise_triton_kernel(
a, b, a_scale, b_scale, group_offs, trans_b=...)`` (ggemm-asm bench.py:241-260, the "persistent"
call sites of bench.py:154-181): for every token t of expert g,

    out[t, :] = a_scale * b_scale[g] * a[t, :] @ b[g].T                      (bf16 out)

a: [M_total, K] float8_e4m3fn (forward: x, swiglu) or float8_e5m2 (data gradient: dy);
b: [G, N, K] float8_e4m3fn (trans_b=True, the layout every harness site uses) or [G, K, N]
(trans_b=False: out = a @ b[g]). It calls ``ggemm_vark_grouped_fp8_fwd_ex`` on the current
stream; there is no CPU or fallback path.
"""
from __future__ import annotations

import torch

from . import _lib

A_FORMATS = {torch.float8_e4m3fn: 0, torch.float8_e5m2: 1}


def grouped_gemm_fp8_tensorwise(a: torch.Tensor, b: torch.Tensor, a_scale: torch.Tensor,
                                b_scale: torch.Tensor, group_offs: torch.Tensor,
                                trans_b: bool = True, out: torch.Tensor | None = None, *,
                                status: torch.Tensor | None = None,
                                timeout_ns: int = 0) -> torch.Tensor:
    """Fixed-K grouped GEMM: out[off_g:off_{g+1}] = sA_g * sB_g * a[off_g:off_{g+1}] @ B_g with
    B_g = b[g].T (trans_b=True, b [G, N, K]) or b[g] (trans_b=False, b [G, K, N]).

    a_scale / b_scale: float32, both 1 element (tensorwise, as the harness) or both G elements
    (per expert). ``out`` (optional): [M_total, N] bf16 with contiguous rows; rows of every
    expert are overwritten. Called without ``out``, ``status`` or ``timeout_ns`` it runs as the
    registered operator torch.ops.ggemm.grouped_fp8_fwd (traceable; see ops.py).
    """
    if out is None and status is None and timeout_ns == 0:
        from . import ops

        return ops.grouped_fp8_fwd(a, b, a_scale, b_scale, group_offs, bool(trans_b))
    return _grouped_fwd(a, b, a_scale, b_scale, group_offs, trans_b, out, status, timeout_ns)


def _grouped_fwd(a, b, a_scale, b_scale, group_offs, trans_b=True, out=None, status=None,
                 timeout_ns=0) -> torch.Tensor:
    """The C-ABI call behind grouped_gemm_fp8_tensorwise and its operator."""
    if a.dtype not in A_FORMATS or b.dtype != torch.float8_e4m3fn:
        raise TypeError(f"expected a float8_e4m3fn/float8_e5m2 and b float8_e4m3fn, got "
                        f"{a.dtype} and {b.dtype}")
    if a.dim() != 2 or b.dim() != 3:
        raise ValueError(f"expected a [M, K] and b [G, N, K] / [G, K, N], got {tuple(a.shape)} "
                         f"and {tuple(b.shape)}")
    if trans_b:
        G, N, K = b.shape
    else:
        G, K, N = b.shape
    if a.shape[1] != K:
        raise ValueError(f"a has K={a.shape[1]} but b has K={K}")
    if a.stride(1) != 1 or b.stride(2) != 1:
        raise ValueError("a and b must have their last dimension contiguous (stride 1)")
    if group_offs.dtype != torch.int64 or group_offs.dim() != 1 or not group_offs.is_contiguous():
        raise ValueError("group_offs must be a contiguous 1-D int64 tensor of G+1 prefix sums")
    if group_offs.numel() != G + 1:
        raise ValueError(f"group_offs has {group_offs.numel()} entries, expected G+1={G + 1}")
    if a_scale.dtype != torch.float32 or b_scale.dtype != torch.float32:
        raise TypeError("a_scale and b_scale must be float32")
    if a_scale.numel() != b_scale.numel() or a_scale.numel() not in (1, G) or not (
            a_scale.is_contiguous() and b_scale.is_contiguous()):
        raise ValueError(f"a_scale and b_scale must both have 1 or G={G} contiguous elements")
    dev = a.device
    if dev.type != "cuda":
        raise ValueError("inputs must be CUDA tensors (no CPU path)")
    for name, t in (("b", b), ("a_scale", a_scale), ("b_scale", b_scale), ("group_offs", group_offs)):
        if t.device != dev:
            raise ValueError(f"{name} is on {t.device}, expected {dev}")
    M = a.shape[0]
    if out is None:
        out = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
    if out.dtype != torch.bfloat16 or tuple(out.shape) != (M, N) or out.stride(1) != 1:
        raise ValueError(f"out must be [{M}, {N}] bf16 with contiguous rows")
    for name, v in (("N", N), ("K", K), ("stride_am", a.stride(0)), ("stride_bg", b.stride(0)),
                    ("stride_bn", b.stride(1)), ("stride_cm", out.stride(0))):
        if v >= 2**31:
            raise ValueError(f"{name}={v} does not fit the int32 ABI")
    status_ptr = None
    if status is not None:
        if status.dtype != torch.int32 or status.numel() < 64 or status.device != dev:
            raise ValueError("status must be an int32 tensor of >= 64 elements on a's device")
        status_ptr = status.data_ptr()
    with torch.cuda.device(dev):
        rc = _lib.lib().ggemm_vark_grouped_fp8_fwd_ex(
            a.data_ptr() if M else None, b.data_ptr(), out.data_ptr() if M else None,
            a_scale.data_ptr(), b_scale.data_ptr(), group_offs.data_ptr(), G, N, K, a.stride(0),
            b.stride(0), b.stride(1), out.stride(0), out.stride(1), M, A_FORMATS[a.dtype],
            0 if b_scale.numel() == 1 else 1, 0 if trans_b else 1, status_ptr, int(timeout_ns),
            torch.cuda.current_stream(dev).cuda_stream)
    _lib.check(rc, "ggemm_vark_grouped_fp8_fwd_ex")
    return out


def fwd_flops(M_total: int, N: int, K: int) -> float:
    """2 * M_total * N * K (the harness's TFLOPS numerator for the persistent sites)."""
    return 2.0 * M_total * N * K
