"""FP8 MoE expert linear layer (autograd over the library's kernels): forward and both
gradients against the oracles applied to the same quantised operands, and against unquantised
fp32 math by cosine."""
import pytest
import torch

from ggemm_asm_b200 import inputs
from ggemm_asm_b200.moe import GroupedLinearFP8, grouped_linear_fp8
from oracle import vark_oracle as vo

E4M3, E5M2 = torch.float8_e4m3fn, torch.float8_e5m2


def test_layer_rejects_cpu_tensors():
    w = torch.zeros(2, 32, 16, dtype=torch.bfloat16)
    x = torch.zeros(8, 32, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        grouped_linear_fp8(x, w, torch.tensor([0, 4, 8]))
    with pytest.raises(ValueError, match="x must be"):
        grouped_linear_fp8(torch.zeros(8, 31, dtype=torch.bfloat16), w, torch.tensor([0, 4, 8]))


def _within(got, ref, tol):
    err = (got.detach().float().cpu() - ref).abs()
    return bool((err <= tol).all()), float((err - tol).max())


@pytest.mark.gpu
@pytest.mark.parametrize("lens,K,N", [([300, 0, 129, 77], 256, 384), ([1000, 500], 2880, 576)])
def test_layer_forward_backward(lens, K, N):
    E = len(lens)
    g = torch.Generator().manual_seed(K + N)
    x = torch.randn(sum(lens), K, generator=g).to(torch.bfloat16)
    w = (torch.randn(E, K, N, generator=g) * K ** -0.5).to(torch.bfloat16)
    dy = torch.randn(sum(lens), N, generator=g).to(torch.bfloat16)
    offs = torch.from_numpy(inputs.offsets_from_lens(lens))

    xd = x.cuda().requires_grad_(True)
    wd = w.cuda().requires_grad_(True)
    y = grouped_linear_fp8(xd, wd, offs.cuda())
    y.backward(dy.cuda())
    torch.cuda.synchronize()

    # Oracles on the same quantised operands.
    xq, sx = vo.quantize_fp8_ref(x, offs, "e4m3")
    w_offs = torch.arange(0, (E + 1) * K, K)
    wq, sw = vo.quantize_fp8_ref(w.view(E * K, N), w_offs, "e4m3")
    dyq, sdy = vo.quantize_fp8_ref(dy, offs, "e5m2")
    xq, wq, dyq = xq.view(E4M3), wq.view(E4M3).view(E, K, N), dyq.view(E5M2)

    y_ref = vo.grouped_fwd_f32(xq, wq, sx, sw, offs, trans_b=False)
    ok, ex = _within(y, y_ref, vo.grouped_fwd_tolerance(xq, wq, sx, sw, offs, y_ref, trans_b=False))
    assert ok, f"forward: max excess {ex}"
    dx_ref = vo.grouped_fwd_f32(dyq, wq, sdy, sw, offs, trans_b=True)
    ok, ex = _within(xd.grad, dx_ref, vo.grouped_fwd_tolerance(dyq, wq, sdy, sw, offs, dx_ref))
    assert ok, f"dx: max excess {ex}"
    dw_ref = vo.wgrad_torch_f32(xq, dyq, sx, sdy, offs)
    ok, ex = _within(wd.grad, dw_ref, vo.tolerance(xq, dyq, sx, sdy, offs, dw_ref))
    assert ok, f"dW: max excess {ex}"
    assert wd.grad.dtype == torch.bfloat16 and tuple(wd.grad.shape) == (E, K, N)

    # And against unquantised fp32 math: FP8 rounding only.
    o = offs.tolist()
    y32 = torch.zeros(sum(lens), N)
    dx32 = torch.zeros(sum(lens), K)
    dw32 = torch.zeros(E, K, N)
    for e in range(E):
        xs, ds = x[o[e]:o[e + 1]].float(), dy[o[e]:o[e + 1]].float()
        y32[o[e]:o[e + 1]] = xs @ w[e].float()
        dx32[o[e]:o[e + 1]] = ds @ w[e].float().T
        dw32[e] = xs.T @ ds
    assert vo.cosine(y.float().cpu(), y32) > 0.995
    assert vo.cosine(xd.grad.float().cpu(), dx32) > 0.99
    assert vo.cosine(wd.grad.float().cpu(), dw32) > 0.99


@pytest.mark.gpu
def test_module_trains_a_step():
    torch.manual_seed(0)
    layer = GroupedLinearFP8(4, 128, 64, device="cuda")
    offs = torch.tensor([0, 100, 100, 250, 400], device="cuda")
    x = torch.randn(400, 128, device="cuda").to(torch.bfloat16)
    target = torch.randn(400, 64, device="cuda").to(torch.bfloat16)
    opt = torch.optim.SGD(layer.parameters(), lr=0.5)
    losses = []
    for _ in range(5):
        opt.zero_grad()
        loss = ((layer(x, offs).float() - target.float()) ** 2).mean()
        loss.backward()
        opt.step()
        losses.append(float(loss))
    assert losses[-1] < losses[0]
    assert torch.isfinite(layer.weight).all()
