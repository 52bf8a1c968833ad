"""The kernels as torch operators (torch.ops.ggemm.*): fake implementations on the CPU (shapes,
dtypes and devices under FakeTensorMode, including the FP8 MoE layer's forward and backward), and
torch.library.opcheck of the real implementations on the GPU."""
import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

import ggemm_asm_b200  # noqa: F401  (registers the operators)
from ggemm_asm_b200 import (grouped_gemm_fp8_tensorwise, grouped_gemm_fp8_tensorwise_variable_k,
                            inputs, moe, quantize_fp8)

E4M3, E5M2, BF16 = torch.float8_e4m3fn, torch.float8_e5m2, torch.bfloat16


def test_operators_are_registered():
    for name in ("variable_k_wgrad", "grouped_fp8_fwd", "quantize_fp8"):
        assert hasattr(torch.ops.ggemm, name), name


def test_fake_shapes_of_every_operator():
    with FakeTensorMode():
        dev = "cuda"
        lhs = torch.empty(1000, 272, dtype=E4M3, device=dev)
        rhs = torch.empty(1000, 384, dtype=E5M2, device=dev)
        s = torch.empty(1, dtype=torch.float32, device=dev)
        offs = torch.empty(6, dtype=torch.int64, device=dev)
        c = torch.ops.ggemm.variable_k_wgrad(lhs, rhs, s, s, offs)
        assert c.shape == (5, 272, 384) and c.dtype == BF16 and c.device.type == "cuda"
        c2 = grouped_gemm_fp8_tensorwise_variable_k(lhs, rhs, s, s, offs)  # the plain function
        assert c2.shape == (5, 272, 384)
        b = torch.empty(5, 320, 272, dtype=E4M3, device=dev)
        y = torch.ops.ggemm.grouped_fp8_fwd(lhs, b, s, s, offs, True)
        assert y.shape == (1000, 320) and y.dtype == BF16
        bt = torch.empty(5, 272, 320, dtype=E4M3, device=dev)
        assert grouped_gemm_fp8_tensorwise(lhs, bt, s, s, offs, trans_b=False).shape == (1000, 320)
        x = torch.empty(1000, 272, dtype=BF16, device=dev)
        q, sc = torch.ops.ggemm.quantize_fp8(x, offs, "e5m2", True)
        assert q.shape == (1000, 272) and q.dtype == E5M2 and sc.shape == (5,)
        q, sc = quantize_fp8(x, offs, "e4m3", granularity="tensor")
        assert q.dtype == E4M3 and sc.shape == (1,)


class _Ctx:
    """Stand-in for the autograd context (the engine itself needs a device to run a backward)."""

    def save_for_backward(self, *t):
        self.saved_tensors = t

    needs_input_grad = (True, True, False)


def test_fp8_layer_traces_forward_and_backward():
    """The FP8 MoE layer (quantise -> fixed-K GEMM forward; quantise -> dx and dW backward) runs
    on fake tensors: every kernel call in it is a registered operator."""
    with FakeTensorMode():
        x = torch.empty(640, 64, dtype=BF16, device="cuda")
        w = torch.empty(4, 64, 96, dtype=BF16, device="cuda")
        offs = torch.empty(5, dtype=torch.int64, device="cuda")
        ctx = _Ctx()
        y = moe.GroupedLinearFP8Function.forward(ctx, x, w, offs)
        assert y.shape == (640, 96) and y.dtype == BF16
        dx, dw, _ = moe.GroupedLinearFP8Function.backward(ctx, torch.empty_like(y))
        assert dx.shape == x.shape and dx.dtype == BF16
        assert dw.shape == w.shape and dw.dtype == BF16


def test_cpu_tensors_still_raise():
    p = inputs.make_problem("tiny", seed=0)
    with pytest.raises(ValueError, match="CUDA"):
        grouped_gemm_fp8_tensorwise_variable_k(p.lhs, p.rhs, p.lhs_scale, p.rhs_scale,
                                               p.group_offs)


# opcheck's schema test multiplies the inputs, which torch does not implement for fp8 tensors.
CHECKS = ("test_faketensor", "test_autograd_registration")


@pytest.mark.gpu
def test_opcheck_on_the_gpu():
    """The fake implementations agree with the real ones (shapes, dtypes, strides) on real CUDA
    inputs, and no autograd kernel is silently missing."""
    p = inputs.make_problem("tiny", seed=3, lens=[100, 0, 77], OUT_M=64, OUT_N=128).to("cuda")
    torch.library.opcheck(torch.ops.ggemm.variable_k_wgrad,
                          (p.lhs, p.rhs, p.lhs_scale, p.rhs_scale, p.group_offs),
                          test_utils=CHECKS)
    b = torch.randn(3, 96, 64, device="cuda").to(E4M3)
    torch.library.opcheck(torch.ops.ggemm.grouped_fp8_fwd,
                          (p.lhs, b, p.lhs_scale, p.rhs_scale, p.group_offs, True),
                          test_utils=CHECKS)
    x = torch.randn(177, 64, device="cuda").to(BF16)
    torch.library.opcheck(torch.ops.ggemm.quantize_fp8, (x, p.group_offs, "e4m3", True),
                          test_utils=CHECKS)


@pytest.mark.gpu
def test_layer_compiles_through_the_operators():
    """torch.compile (dynamo + AOTAutograd, fullgraph) of the FP8 layer's forward and backward
    traces through the operators' fake implementations and matches eager bit for bit."""
    lens = [300, 0, 77, 160]
    offs = torch.from_numpy(inputs.offsets_from_lens(lens)).cuda()
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(sum(lens), 128, generator=g, device="cuda").to(BF16)
    layer = moe.GroupedLinearFP8(4, 128, 192, device="cuda")

    def fwd(xi):
        return layer(xi, offs)

    xe = x.clone().requires_grad_(True)
    ye = fwd(xe)
    ye.float().square().sum().backward()
    ge, gwe = xe.grad.clone(), layer.weight.grad.clone()
    layer.weight.grad = None
    xc = x.clone().requires_grad_(True)
    # AOTAutograd traces the joint forward + backward graph at compile time.
    yc = torch.compile(fwd, backend="aot_eager", fullgraph=True)(xc)
    yc.float().square().sum().backward()
    torch.cuda.synchronize()
    assert torch.equal(yc, ye) and torch.equal(xc.grad, ge)
    assert torch.equal(layer.weight.grad, gwe)
