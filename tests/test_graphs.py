"""CUDA graphs: the producer step + wgrad chain and a whole FP8 MoE layer training step captured
once and replayed give exactly the eager results (the library's one-time device set-up happens
in a warm-up call before capture, as documented)."""
import pytest
import torch

from ggemm_asm_b200 import grouped_gemm_fp8_tensorwise_variable_k as wgrad, inputs, quantize_fp8
from ggemm_asm_b200.moe import grouped_linear_fp8

pytestmark = pytest.mark.gpu


def test_quantize_and_wgrad_in_a_graph():
    lens = [700, 0, 256, 1301, 64]
    offs = torch.from_numpy(inputs.offsets_from_lens(lens)).cuda()
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(sum(lens), 384, generator=g, device="cuda").to(torch.bfloat16)
    dy = torch.randn(sum(lens), 512, generator=g, device="cuda").to(torch.bfloat16)

    def chain():
        lhs, sl = quantize_fp8(x, offs, "e4m3")
        rhs, sr = quantize_fp8(dy, offs, "e5m2")
        return wgrad(lhs, rhs, sl, sr, offs)

    eager = chain()
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        chain()  # warm-up on the capture stream
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = chain()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    # new inputs in the same buffers: the replay follows them
    x.mul_(0.5)
    graph.replay()
    ref = chain()
    torch.cuda.synchronize()
    assert torch.equal(out, ref)


def test_layer_training_step_in_a_graph():
    E, K, N = 4, 256, 192
    lens = [300, 0, 129, 211]
    offs = torch.from_numpy(inputs.offsets_from_lens(lens)).cuda()
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(sum(lens), K, generator=g, device="cuda").to(torch.bfloat16)
    w = (torch.randn(E, K, N, generator=g, device="cuda") * K ** -0.5).to(torch.bfloat16)
    dy = torch.randn(sum(lens), N, generator=g, device="cuda").to(torch.bfloat16)
    xs = x.clone().requires_grad_(True)
    ws = w.clone().requires_grad_(True)

    def step():
        y = grouped_linear_fp8(xs, ws, offs)
        y.backward(dy)
        return y

    y_eager = step().detach().clone()
    gx, gw = xs.grad.clone(), ws.grad.clone()
    xs.grad = None
    ws.grad = None
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()
    torch.cuda.current_stream().wait_stream(s)
    xs.grad = None
    ws.grad = None
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        y = step()
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(y.detach(), y_eager)
    assert torch.equal(xs.grad, gx) and torch.equal(ws.grad, gw)
