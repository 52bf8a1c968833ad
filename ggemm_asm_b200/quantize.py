"""Per-expert FP8 quantisation of token-major bf16 operands: the producer step of the wgrad.

``quantize_fp8(x, group_offs, "e4m3")`` turns the activations ``x`` into the wgrad's LHS and
``quantize_fp8(dy, group_offs, "e5m2")`` the output gradients into its RHS, each with one fp32
scale per expert (or per tensor), in a single kernel per operand (``ggemm_vark_quantize_fp8``):

    s_g = amax(|x[off_g:off_{g+1}]|) / FMAX      (1.0 for an empty expert or an all-zero slice)
    q   = fp8(x / s_g), round to nearest even, saturated to +-FMAX (448 e4m3fn, 57344 e5m2)

The reference harness builds its fp8 operands on the host (ggemm-asm bench.py:221-223, scales
fixed by bench.py:266-267); this op is the device-side producer of the amax-scaled operands the
wgrad's configurations use. There is no CPU path: inputs must be CUDA tensors on an sm_100 device.
"""
from __future__ import annotations

import torch

from . import _lib

FORMATS = {"e4m3": (0, torch.float8_e4m3fn, 448.0), "e5m2": (1, torch.float8_e5m2, 57344.0)}


def quantize_fp8(x: torch.Tensor, group_offs: torch.Tensor, fmt: str = "e4m3", *,
                 granularity: str = "group", out: torch.Tensor | None = None,
                 scales: torch.Tensor | None = None, status: torch.Tensor | None = None,
                 timeout_ns: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
    """Return ``(q, scales)``: q = fp8(x / s) per unit, s = amax/FMAX per unit.

    x: [tokens, F] bfloat16 CUDA tensor with contiguous rows (any row pitch).
    group_offs: int64 [G+1] prefix sums on the same device (offs[0] = 0, offs[G] = tokens).
    fmt: "e4m3" (float8_e4m3fn, the LHS/activation format) or "e5m2" (the RHS/gradient format).
    granularity: "group" (one scale per expert, G values) or "tensor" (one scale over all rows).
    out / scales: optional outputs ([tokens, F] fp8 with contiguous rows; fp32 [G] or [1]).
    status / timeout_ns: optional int32 status block (>= 64 elements) and wait limit (ns).
    Rows outside [offs[0], offs[G]) are left as they are in ``out`` (uninitialised if new).
    Called without ``out``, ``scales``, ``status`` or ``timeout_ns`` it runs as the registered
    operator torch.ops.ggemm.quantize_fp8 (traceable; see ops.py).
    """
    if out is None and scales is None and status is None and timeout_ns == 0 and \
            granularity in ("group", "tensor") and fmt in FORMATS:
        from . import ops

        return ops.quantize_fp8(x, group_offs, fmt, granularity == "group")
    return _quantize_fp8(x, group_offs, fmt, granularity, out, scales, status, timeout_ns)


def _quantize_fp8(x, group_offs, fmt="e4m3", granularity="group", out=None, scales=None,
                  status=None, timeout_ns=0) -> tuple[torch.Tensor, torch.Tensor]:
    """The C-ABI call behind quantize_fp8 and its operator."""
    if fmt not in FORMATS:
        raise ValueError(f"fmt must be one of {sorted(FORMATS)}, got {fmt!r}")
    if granularity not in ("group", "tensor"):
        raise ValueError("granularity must be 'group' or 'tensor'")
    code, dtype, _ = FORMATS[fmt]
    if x.dtype != torch.bfloat16 or x.dim() != 2 or x.stride(1) != 1:
        raise ValueError("x must be a 2-D bfloat16 tensor with contiguous rows")
    if group_offs.dtype != torch.int64 or group_offs.dim() != 1 or group_offs.numel() < 1:
        raise ValueError("group_offs must be a 1-D int64 tensor of G+1 prefix sums")
    if not group_offs.is_contiguous():
        raise ValueError("group_offs must be contiguous")
    G = group_offs.numel() - 1
    per_group = granularity == "group"
    units = G if per_group else 1
    if x.device.type != "cuda" or group_offs.device != x.device:
        raise ValueError("x and group_offs must be CUDA tensors on the same device (no CPU path)")
    rows, F = x.shape
    if out is None:
        out = torch.empty(rows, F, dtype=dtype, device=x.device)
    if out.dtype != dtype or tuple(out.shape) != (rows, F) or out.stride(1) != 1:
        raise ValueError(f"out must be [{rows}, {F}] {dtype} with contiguous rows")
    if scales is None:
        scales = torch.empty(max(units, 1), dtype=torch.float32, device=x.device)
    if scales.dtype != torch.float32 or scales.numel() < units or not scales.is_contiguous():
        raise ValueError(f"scales must be a contiguous float32 tensor of >= {units} elements")
    for name, v in (("G", G), ("F", F), ("stride_x", x.stride(0)), ("stride_q", out.stride(0))):
        if v >= 2**31:
            raise ValueError(f"{name}={v} does not fit the int32 ABI")
    ws = torch.empty(_lib.lib().ggemm_vark_quantize_workspace_bytes(units) + 16,
                     dtype=torch.uint8, device=x.device)
    ws_ptr = (ws.data_ptr() + 15) // 16 * 16
    status_ptr = None
    if status is not None:
        if status.dtype != torch.int32 or status.numel() < 64 or status.device != x.device:
            raise ValueError("status must be an int32 tensor of >= 64 elements on x's device")
        status_ptr = status.data_ptr()
    stream = torch.cuda.current_stream(x.device).cuda_stream
    with torch.cuda.device(x.device):
        rc = _lib.lib().ggemm_vark_quantize_fp8(
            x.data_ptr() if rows else None, out.data_ptr() if rows else None, scales.data_ptr(),
            group_offs.data_ptr(), G, F, x.stride(0), out.stride(0), code, int(per_group), rows,
            ws_ptr, status_ptr, int(timeout_ns), stream)
    _lib.check(rc, "ggemm_vark_quantize_fp8")
    return out, scales
