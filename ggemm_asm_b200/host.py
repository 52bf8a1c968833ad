"""Grouped wgrad with host-resident operands: copies in, kernel and copies out overlapped.

For callers whose LHS/RHS live in pinned host memory and who want C back on the host (an offload
setting, or any measurement that includes the transfers). The experts are split into contiguous
chunks balanced by work (sharding.partition); for chunk i the host->device copy of its token rows,
the wgrad of its experts and the device->host copy of its C slices run on three streams, so the
copy of chunk i+1 and the read-back of chunk i-1 overlap the kernel of chunk i, and the two copy
directions overlap each other (PCIe is full duplex). Each chunk is one ordinary call of the
variable-K wgrad on the chunk's rows with rebased offsets, so C is bit-identical to a single call
over all experts (every expert's tiles are computed the same way whatever else is in the launch).
"""
from __future__ import annotations

import numpy as np
import torch

from . import sharding
from .grouped_gemm import grouped_gemm_fp8_tensorwise_variable_k


class HostWgrad:
    """Reusable device buffers and streams for problems up to (max_tokens, G, OUT_M, OUT_N).

    call(lhs_h, rhs_h, lhs_scale, rhs_scale, group_offs_h, out_h): lhs_h [M, OUT_M] e4m3 and
    rhs_h [M, OUT_N] e5m2 in pinned host memory, scales fp32 (1 or G elements; host or device),
    group_offs_h host int64 [G+1], out_h pinned host bf16 [G, OUT_M, OUT_N]. Returns out_h once
    its contents are on the host (the call synchronises with its last copy). One instance owns
    its device buffers and streams: calls on the same instance must not overlap (use one
    instance per thread).
    """

    def __init__(self, max_tokens: int, G: int, OUT_M: int, OUT_N: int, device="cuda",
                 chunks: int = 8):
        self.device = torch.device(device)
        self.chunks = max(1, int(chunks))
        self.d_lhs = torch.empty(max_tokens, OUT_M, dtype=torch.float8_e4m3fn, device=self.device)
        self.d_rhs = torch.empty(max_tokens, OUT_N, dtype=torch.float8_e5m2, device=self.device)
        self.d_out = torch.empty(G, OUT_M, OUT_N, dtype=torch.bfloat16, device=self.device)
        self.d_offs = torch.empty(G + 1 + self.chunks, dtype=torch.int64, device=self.device)
        self.h_offs = torch.empty(G + 1 + self.chunks, dtype=torch.int64, pin_memory=True)
        self.s_in = torch.cuda.Stream(self.device)
        self.s_run = torch.cuda.Stream(self.device)
        self.s_out = torch.cuda.Stream(self.device)

    def __call__(self, lhs_h, rhs_h, lhs_scale, rhs_scale, group_offs_h, out_h):
        for name, t in (("lhs_h", lhs_h), ("rhs_h", rhs_h), ("out_h", out_h)):
            if t.device.type != "cpu" or not t.is_pinned():
                raise ValueError(f"{name} must be a pinned host tensor")
        offs = np.asarray(group_offs_h, dtype=np.int64)
        G = offs.size - 1
        M = int(offs[-1])
        if M > self.d_lhs.shape[0] or G > self.d_out.shape[0]:
            raise ValueError("problem larger than the buffers this HostWgrad was built for")
        if lhs_h.dtype != torch.float8_e4m3fn or rhs_h.dtype != torch.float8_e5m2:
            raise TypeError("lhs_h must be float8_e4m3fn and rhs_h float8_e5m2")
        shards = [s for s in sharding.partition(np.diff(offs), self.chunks) if s.groups > 0]
        # Every chunk's offsets rebased to its first token, packed into one small host buffer.
        packed, where = [], []
        for s in shards:
            where.append(len(packed))
            packed.extend((offs[s.g_begin:s.g_end + 1] - offs[s.g_begin]).tolist())
        self.h_offs[:len(packed)] = torch.tensor(packed, dtype=torch.int64)
        dev = self.device
        ls = lhs_scale.to(dev, non_blocking=True)
        rs = rhs_scale.to(dev, non_blocking=True)
        cur = torch.cuda.current_stream(dev)
        for s in (self.s_in, self.s_run, self.s_out):
            s.wait_stream(cur)
        with torch.cuda.stream(self.s_in):
            self.d_offs[:len(packed)].copy_(self.h_offs[:len(packed)], non_blocking=True)
        per_group = ls.numel() > 1
        for i, s in enumerate(shards):
            t0, t1 = int(offs[s.g_begin]), int(offs[s.g_end])
            with torch.cuda.stream(self.s_in):
                self.d_lhs[t0:t1].copy_(lhs_h[t0:t1], non_blocking=True)
                self.d_rhs[t0:t1].copy_(rhs_h[t0:t1], non_blocking=True)
            self.s_run.wait_stream(self.s_in)
            with torch.cuda.stream(self.s_run):
                grouped_gemm_fp8_tensorwise_variable_k(
                    self.d_lhs[t0:t1], self.d_rhs[t0:t1],
                    ls[s.g_begin:s.g_end] if per_group else ls,
                    rs[s.g_begin:s.g_end] if per_group else rs,
                    self.d_offs[where[i]:where[i] + s.groups + 1],
                    out=self.d_out[s.g_begin:s.g_end])
            self.s_out.wait_stream(self.s_run)
            with torch.cuda.stream(self.s_out):
                out_h[s.g_begin:s.g_end].copy_(self.d_out[s.g_begin:s.g_end], non_blocking=True)
        # Experts with no chunk (all empty) still get zeros, like the device path.
        covered = np.zeros(G, dtype=bool)
        for s in shards:
            covered[s.g_begin:s.g_end] = True
        cur.wait_stream(self.s_out)
        self.s_out.synchronize()
        if not covered.all():
            out_h[torch.from_numpy(~covered)] = 0
        return out_h
