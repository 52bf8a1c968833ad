"""ggemm_asm_b200 - B200 (sm_100a) variable-K grouped FP8 GEMM (MoE expert weight gradient).

    C[g] = sL * sR * LHS[off_g:off_{g+1}]^T @ RHS[off_g:off_{g+1}]   (e4m3 x e5m2 -> fp32 -> bf16)

Public API:
  grouped_gemm_fp8_tensorwise_variable_k  torch entry point (mirrors the Primus-Turbo call the
                                          ggemm-asm harness makes, bench.py:268)
  variable_k_wgrad                        alias
  launch_raw                              the 14-argument C-ABI drop-in with raw pointers
  grouped_gemm_fp8_tensorwise             fixed-K grouped GEMM of the forward / data-gradient
                                          sites (mirrors the Primus-Turbo call, bench.py:260)
  quantize_fp8                            per-expert amax scaling + fp8 quantisation of x / dy
                                          (the producer step in front of the wgrad)
  moe.GroupedLinearFP8 / grouped_linear_fp8  FP8 MoE expert linear layer with autograd (forward,
                                          data gradient and weight gradient on these kernels)
  inputs / sharding                       seeded problems and expert sharding for 1..8 GPUs
  ops                                     the kernels as torch operators (torch.ops.ggemm.*) with
                                          fake implementations, so they trace
The C ABI itself is declared in include/ggemm_vark.h and lives in libggemm_vark.so.
"""
from .grouped_gemm import (  # noqa: F401
    flops,
    grouped_gemm_fp8_tensorwise_variable_k,
    launch_raw,
    variable_k_wgrad,
)
from ._lib import VarkError, read_status  # noqa: F401
from .grouped_fwd import grouped_gemm_fp8_tensorwise  # noqa: F401
from .quantize import quantize_fp8  # noqa: F401
from . import ops  # noqa: F401,E402  (registers torch.ops.ggemm.*)

__version__ = "0.1.0"
