"""The allocation-free entry point (ggemm_vark_fp8_wgrad_noalloc).

It exists for callers that must not let a library call cudaMalloc: code that runs inside a
framework-owned memory pool or arena, allocators with strict accounting, and processes with a
fixed device footprint. It runs the same tensor-core kernel as the regular entry points with its
scratch in a fixed device array inside the library. This file is named so that pytest collects
it last; it must pass alone in a fresh process and after the other tests.
"""
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

from ggemm_asm_b200 import _lib, inputs
from oracle import vark_oracle as vo

pytestmark = pytest.mark.gpu


def _noalloc(d, out, status=None):
    """Call the C ABI entry point directly (no Python-side allocation on this path)."""
    stream = torch.cuda.current_stream().cuda_stream
    return _lib.lib().ggemm_vark_fp8_wgrad_noalloc(
        d.lhs.data_ptr(), d.rhs.data_ptr(), out.data_ptr(), d.lhs_scale.data_ptr(),
        d.rhs_scale.data_ptr(), d.group_offs.data_ptr(), d.G, d.OUT_M, d.OUT_N,
        d.lhs.stride(0), d.rhs.stride(0), out.stride(0), out.stride(1), out.stride(2),
        d.lhs.shape[0], 0 if d.lhs_scale.numel() == 1 else 1,
        None if status is None else status.data_ptr(), stream)


def _existing(d, out):
    stream = torch.cuda.current_stream().cuda_stream
    return _lib.lib().ggemm_vark_fp8_wgrad_ex(
        d.lhs.data_ptr(), d.rhs.data_ptr(), out.data_ptr(), d.lhs_scale.data_ptr(),
        d.rhs_scale.data_ptr(), d.group_offs.data_ptr(), d.G, d.OUT_M, d.OUT_N,
        d.lhs.stride(0), d.rhs.stride(0), out.stride(0), out.stride(1), out.stride(2),
        d.lhs.shape[0], 0 if d.lhs_scale.numel() == 1 else 1, _lib.PATH_AUTO, None, 0, stream)


def _tolerance_check(p, got, ref):
    """Within the parity tolerance used everywhere in this suite (1 bf16 ulp of the oracle's
    magnitude plus the fp32 reassociation bound), against the regular entry point's output."""
    ref32 = vo.wgrad_torch_f32(p.lhs, p.rhs, p.lhs_scale, p.rhs_scale, p.group_offs)
    tol = vo.tolerance(p.lhs, p.rhs, p.lhs_scale, p.rhs_scale, p.group_offs, ref32)
    err = (got.float().cpu() - ref.float().cpu()).abs()
    assert bool((err <= tol).all()), f"max diff {err.max().item()}"
    assert vo.cosine(got.float().cpu(), ref.float().cpu()) >= 0.99999


# (OUT_M, OUT_N): the last row tile has 224, 48 (32-byte LHS boxes) or 112 rows (64-byte LHS
# boxes); the transposed last column tile has 128 (64-byte RHS boxes) or 64 columns (32-byte).
SHAPES = [(480, 640), (304, 320), (368, 640), (368, 320)]


@pytest.mark.parametrize("shape", SHAPES, ids=[f"{m}x{n}" for m, n in SHAPES])
@pytest.mark.parametrize("scales", ["tensor", "group"])
def test_noalloc_matches_existing_entry_point_twice(scales, shape):
    m, n = shape
    problems = [
        inputs.make_problem("tiny", seed=41, lens=[700, 0, 129, 1500, 33], OUT_M=m, OUT_N=n,
                            scales=scales),
        inputs.make_problem("tiny", seed=42, lens=[64, 2000, 0, 0, 901], OUT_M=m, OUT_N=n,
                            scales=scales),
    ]
    for p in problems:  # two calls in a row, different data: no stale state carries over
        d = p.to("cuda")
        ref = torch.full((d.G, d.OUT_M, d.OUT_N), 5.0, dtype=torch.bfloat16, device="cuda")
        got = torch.full_like(ref, -5.0)
        assert _existing(d, ref) == _lib.OK
        assert _noalloc(d, got) == _lib.OK
        torch.cuda.synchronize()
        _tolerance_check(p, got, ref)
        assert torch.equal(got, ref)  # same kernel, same accumulation order


def test_noalloc_reports_status_in_caller_buffer():
    p = inputs.make_problem("tiny", seed=43, lens=[64, 64, 64, 64], OUT_M=256, OUT_N=256)
    d = p.to("cuda")
    d.group_offs = torch.tensor([0, 64, 40, 192, 256], dtype=torch.int64, device="cuda")
    status = torch.zeros(64, dtype=torch.int32, device="cuda")  # a 256-byte status block
    out = torch.full((4, 256, 256), 3.0, dtype=torch.bfloat16, device="cuda")
    assert _noalloc(d, out, status) == _lib.OK
    torch.cuda.synchronize()
    assert int(status[0].item()) & _lib.DEV_BAD_OFFS
    assert bool((out[1] == 0).all())


def test_noalloc_rejects_what_it_cannot_run():
    p = inputs.make_problem("tiny", seed=44, lens=[10, 20], OUT_M=64, OUT_N=128)
    d = p.to("cuda")
    out = torch.empty(2, 64, 128, dtype=torch.bfloat16, device="cuda")
    wide = torch.zeros(30, 72, dtype=torch.uint8, device="cuda")
    d.lhs = wide[:, :64].view(torch.float8_e4m3fn)  # row pitch 72: not a tensor-core layout
    assert _noalloc(d, out) == _lib.ELAYOUT
    assert _lib.lib().ggemm_vark_fp8_wgrad_noalloc(
        None, None, None, None, None, None, 1, 1, 1, 1, 1, 1, 1, 1, -1, 0, None, None) == \
        _lib.EINVAL_PTR
    header = (Path(__file__).resolve().parents[1] / "include" / "ggemm_vark.h").read_text()
    assert "#define GGEMM_VARK_NOALLOC_SCRATCH_BYTES 4096u" in header  # status words only


def test_noalloc_accepts_an_empty_batch_like_the_existing_entry_point():
    """m_total == 0 with NULL operands: every group is empty and C is zeroed, as for _ex."""
    p = inputs.make_problem("tiny", seed=46, lens=[0, 0, 0], OUT_M=64, OUT_N=128)
    d = p.to("cuda")
    out = torch.full((3, 64, 128), 5.0, dtype=torch.bfloat16, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    rc = _lib.lib().ggemm_vark_fp8_wgrad_noalloc(
        None, None, out.data_ptr(), d.lhs_scale.data_ptr(), d.rhs_scale.data_ptr(),
        d.group_offs.data_ptr(), 3, 64, 128, 64, 128, out.stride(0), out.stride(1), 1, 0, 0,
        None, stream)
    assert rc == _lib.OK
    torch.cuda.synchronize()
    assert bool((out == 0).all())


_ALLOC_FREE_SCRIPT = r"""
import sys, torch
sys.path.insert(0, sys.argv[1])
from ggemm_asm_b200 import _lib, inputs
p = inputs.make_problem("tiny", seed=47, lens=[300, 0, 77, 1500], OUT_M=480, OUT_N=640)
d = p.to("cuda")
out = torch.empty(d.G, d.OUT_M, d.OUT_N, dtype=torch.bfloat16, device="cuda")
stream = torch.cuda.current_stream().cuda_stream
def call():
    return _lib.lib().ggemm_vark_fp8_wgrad_noalloc(
        d.lhs.data_ptr(), d.rhs.data_ptr(), out.data_ptr(), d.lhs_scale.data_ptr(),
        d.rhs_scale.data_ptr(), d.group_offs.data_ptr(), d.G, d.OUT_M, d.OUT_N,
        d.lhs.stride(0), d.rhs.stride(0), out.stride(0), out.stride(1), out.stride(2),
        d.lhs.shape[0], 0, None, stream)
assert call() == 0  # first call: symbol lookup, kernel attributes, lazy module load
torch.cuda.synchronize()
free0 = torch.cuda.mem_get_info()[0]
assert call() == 0 and call() == 0
torch.cuda.synchronize()
free1 = torch.cuda.mem_get_info()[0]
held = _lib.device_bytes(torch.cuda.current_device())
print("free", free0, free1, "library bytes", held)
assert free1 == free0, "device memory changed across two calls"
assert held == 0, "the regular entry points' per-device state was set up"
"""


def test_noalloc_allocates_nothing_in_a_fresh_process():
    """A fresh process that calls only the allocation-free entry point: free device memory is
    unchanged across two calls, and the library reports no allocation of its own on the device
    (the regular entry points would have made their 4 KiB status block)."""
    root = str(Path(__file__).resolve().parents[1])
    res = subprocess.run([sys.executable, "-c", _ALLOC_FREE_SCRIPT, root], capture_output=True,
                         text=True, timeout=600, env={**os.environ, "PYTHONPATH": root})
    assert res.returncode == 0, res.stdout + res.stderr
    # The same query after a regular call in this process reports the status block.
    p = inputs.make_problem("tiny", seed=48, lens=[40], OUT_M=64, OUT_N=128)
    d = p.to("cuda")
    out = torch.empty(1, 64, 128, dtype=torch.bfloat16, device="cuda")
    assert _existing(d, out) == _lib.OK
    torch.cuda.synchronize()
    assert _lib.device_bytes(torch.cuda.current_device()) == 4096
