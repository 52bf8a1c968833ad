"""Failure detection on the GPU without a fault: a pipeline wait that runs out.

The tensor-core kernels bound every mbarrier wait. With the GGEMM_VARK_TEST_STALL_MAGIC hook in a
caller-provided status block, the producers withhold their first stage, so the MMA warp's wait on
it can never complete. The kernel must then stop by itself within the given limit, report
GGEMM_VARK_DEV_TIMEOUT in the status block, and leave the context usable for the next call.
Nothing here traps, faults or hangs the GPU.
"""
import time

import pytest
import torch

from ggemm_asm_b200 import _lib, grouped_gemm_fp8_tensorwise_variable_k as vark, inputs
from oracle import vark_oracle as vo

pytestmark = pytest.mark.gpu

STALL_MAGIC = 0x5374616C
PATHS = {"tcgen05": _lib.PATH_TCGEN05, "tcgen05_1sm": _lib.PATH_TCGEN05_1SM}


@pytest.mark.parametrize("path", sorted(PATHS))
def test_expired_wait_is_reported_and_context_survives(path):
    p = inputs.make_problem("tiny", seed=51, lens=[300, 0, 200], OUT_M=256, OUT_N=256)
    d = p.to("cuda")
    status = torch.zeros(64, dtype=torch.int32, device="cuda")
    status[3] = STALL_MAGIC
    out = torch.empty(3, 256, 256, dtype=torch.bfloat16, device="cuda")
    timeout_ns = 20_000_000  # 20 ms per wait
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    rc = _lib.lib().ggemm_vark_fp8_wgrad_ex(
        d.lhs.data_ptr(), d.rhs.data_ptr(), out.data_ptr(), d.lhs_scale.data_ptr(),
        d.rhs_scale.data_ptr(), d.group_offs.data_ptr(), d.G, d.OUT_M, d.OUT_N,
        d.lhs.stride(0), d.rhs.stride(0), out.stride(0), out.stride(1), out.stride(2),
        d.lhs.shape[0], 0, PATHS[path], status.data_ptr(), timeout_ns,
        torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.OK
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert elapsed < 5.0, f"the stalled launch took {elapsed:.2f} s to stop"
    bits = int(status[0].item())
    assert bits & _lib.DEV_TIMEOUT, f"status {bits:#x}: the expired wait was not reported"
    assert int(status[1].item()) != 0  # the wait site that expired

    # The context is intact: the next call on the same stream computes correct results.
    good = vark(d.lhs, d.rhs, d.lhs_scale, d.rhs_scale, d.group_offs, path=path)
    torch.cuda.synchronize()
    assert _lib.read_status(clear=True) == 0
    ref = vo.wgrad_torch_f32(p.lhs, p.rhs, p.lhs_scale, p.rhs_scale, p.group_offs)
    assert vo.cosine(good.float().cpu(), ref) >= 0.99999
    assert bool((good[1] == 0).all())


def test_status_read_in_stream_order_waits_for_its_stream_only():
    """ggemm_vark_read_status_stream waits for the given stream alone: with another stream busy
    for about a second it returns at once, and it sees the words of work queued before it on its
    own stream (a bad offset recorded by a call just before)."""
    p = inputs.make_problem("tiny", seed=52, lens=[64, 64], OUT_M=256, OUT_N=256)
    d = p.to("cuda")
    bad = torch.tensor([0, 64, 40], dtype=torch.int64, device="cuda")
    status = torch.zeros(64, dtype=torch.int32, device="cuda")
    out = torch.empty(2, 256, 256, dtype=torch.bfloat16, device="cuda")
    busy, mine = torch.cuda.Stream(), torch.cuda.Stream()
    torch.cuda.synchronize()
    with torch.cuda.stream(busy):
        torch.cuda._sleep(2_000_000_000)  # ~1 s of spinning on the other stream
    with torch.cuda.stream(mine):
        vark(d.lhs, d.rhs, d.lhs_scale, d.rhs_scale, bad, out=out, status=status)
        t0 = time.perf_counter()
        words = _lib.read_status_words(status.data_ptr(), 8, clear=True, stream=mine.cuda_stream)
        elapsed = time.perf_counter() - t0
    assert words[_lib.STATUS_WORD_BITS] & _lib.DEV_BAD_OFFS
    assert elapsed < 0.5, f"the stream-ordered read waited {elapsed:.2f} s"
    torch.cuda.synchronize()
    assert int(status[0].item()) == 0  # cleared in the same stream order
