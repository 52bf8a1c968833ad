"""Grouped wgrad from pinned host buffers (copies overlapped with the kernel): bit-identical to
the device call."""
import pytest
import torch

from ggemm_asm_b200 import grouped_gemm_fp8_tensorwise_variable_k as wgrad, inputs
from ggemm_asm_b200.host import HostWgrad


@pytest.mark.gpu
@pytest.mark.parametrize("chunks", [1, 3, 8])
@pytest.mark.parametrize("scales", ["tensor", "group"])
def test_host_pipeline_matches_device_call(chunks, scales):
    lens = [700, 0, 256, 1, 3000, 0, 129, 64]
    p = inputs.make_problem("skew" if scales == "group" else "tiny", seed=21, lens=lens,
                            OUT_M=272, OUT_N=384)
    d = p.to("cuda")
    ref = wgrad(d.lhs, d.rhs, d.lhs_scale, d.rhs_scale, d.group_offs)
    h_lhs = p.lhs.pin_memory()
    h_rhs = p.rhs.pin_memory()
    h_out = torch.full((p.G, p.OUT_M, p.OUT_N), 3.0, dtype=torch.bfloat16).pin_memory()
    pipe = HostWgrad(p.M_total, p.G, p.OUT_M, p.OUT_N, chunks=chunks)
    got = pipe(h_lhs, h_rhs, p.lhs_scale, p.rhs_scale, p.offs, h_out)
    torch.cuda.synchronize()
    assert torch.equal(got, ref.cpu())
    with pytest.raises(ValueError, match="pinned"):
        pipe(p.lhs, h_rhs, p.lhs_scale, p.rhs_scale, p.offs, h_out)
