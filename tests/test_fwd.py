"""The fixed-K grouped FP8 GEMM (forward / data-gradient sites): oracle pins and C-ABI rules on
the CPU, parity with the oracle on the GPU (ragged experts, edge tiles in N, K tails, both A
formats, per-expert scales, rows outside the experts untouched, the harness's full-size sites)."""
import numpy as np
import pytest
import torch

from ggemm_asm_b200 import _lib, grouped_gemm_fp8_tensorwise, inputs
from oracle import vark_oracle as vo

P = 1 << 20  # fake aligned device address: never dereferenced by the CPU tests
E4M3, E5M2 = torch.float8_e4m3fn, torch.float8_e5m2


def make_fwd(lens, N, K, a_dtype=E4M3, seed=0, per_expert_scale=False):
    """Seeded problem: a [M, K] (N(0,1) cast to fp8 as bench.py:221-223 does), b [G, N, K]
    e4m3, scales 0.1 (bench.py:257-258) or per-expert values."""
    g = torch.Generator().manual_seed(seed)
    M, G = int(sum(lens)), len(lens)
    a = torch.randn(M, K, generator=g).to(torch.bfloat16).to(a_dtype)
    b = torch.randn(G, N, K, generator=g).to(torch.bfloat16).to(E4M3)
    if per_expert_scale:
        sa = torch.rand(G, generator=g) * 0.2 + 0.05
        sb = torch.rand(G, generator=g) * 0.2 + 0.05
    else:
        sa, sb = torch.tensor([0.1]), torch.tensor([0.1])
    offs = torch.from_numpy(inputs.offsets_from_lens(lens))
    return a, b, sa.float(), sb.float(), offs


# ------------------------------------------------------------------------------------------------
# CPU
# ------------------------------------------------------------------------------------------------
def test_oracle_matches_float64_restatement():
    a, b, sa, sb, offs = make_fwd([5, 0, 17, 3], N=24, K=40, a_dtype=E5M2, per_expert_scale=True)
    ref = vo.grouped_fwd_f32(a, b, sa, sb, offs)
    ta = vo.fp8_decode_table("e5m2")[a.view(torch.uint8).numpy()]
    tb = vo.fp8_decode_table("e4m3fn")[b.view(torch.uint8).numpy()]
    exact = np.zeros((a.shape[0], 24))
    o = offs.tolist()
    for gi in range(4):
        exact[o[gi]:o[gi + 1]] = ta[o[gi]:o[gi + 1]] @ tb[gi].T * float(sa[gi]) * float(sb[gi])
    tol = vo.grouped_fwd_tolerance(a, b, sa, sb, offs, ref)
    assert (np.abs(ref.numpy() - exact) <= tol.numpy()).all()
    assert float(np.abs(exact).max()) > 0


def test_oracle_row_subset():
    a, b, sa, sb, offs = make_fwd([7, 0, 9], N=16, K=32)
    full = vo.grouped_fwd_f32(a, b, sa, sb, offs)
    rows = torch.tensor([15, 0, 8, 6])
    assert torch.equal(vo.grouped_fwd_f32(a, b, sa, sb, offs, rows), full[rows])


def call_fwd(**kw):
    x = dict(a=P, b=P, c=P, sa=P, sb=P, offs=P, G=4, N=256, K=512, sam=512, sbg=256 * 512,
             sbn=512, scm=256, scn=1, m=1024, fmt=0, ss=0, lay=0, status=None)
    x.update(kw)
    return _lib.lib().ggemm_vark_grouped_fp8_fwd_ex(
        x["a"], x["b"], x["c"], x["sa"], x["sb"], x["offs"], x["G"], x["N"], x["K"], x["sam"],
        x["sbg"], x["sbn"], x["scm"], x["scn"], x["m"], x["fmt"], x["ss"], x["lay"], x["status"],
        0, None)


@pytest.mark.parametrize("kw,code", [
    (dict(sa=None), _lib.EINVAL_PTR), (dict(offs=None), _lib.EINVAL_PTR),
    (dict(a=None), _lib.EINVAL_PTR), (dict(c=None), _lib.EINVAL_PTR),
    (dict(G=-1), _lib.EINVAL_SHAPE), (dict(N=0), _lib.EINVAL_SHAPE), (dict(K=0), _lib.EINVAL_SHAPE),
    (dict(sam=500), _lib.EINVAL_STRIDE), (dict(sbn=100), _lib.EINVAL_STRIDE),
    (dict(sbg=1000), _lib.EINVAL_STRIDE), (dict(scm=100), _lib.EINVAL_STRIDE),
    (dict(scn=0), _lib.EINVAL_STRIDE),
    (dict(fmt=2), _lib.EINVAL_ARG), (dict(ss=2), _lib.EINVAL_ARG), (dict(m=-2), _lib.EINVAL_ARG),
    (dict(status=P + 4), _lib.EINVAL_ARG),
    (dict(a=P + 8), _lib.ELAYOUT), (dict(sam=520), _lib.ELAYOUT), (dict(scn=2), _lib.ELAYOUT),
    (dict(scm=260), _lib.ELAYOUT), (dict(sbn=520, sbg=256 * 520), _lib.ELAYOUT),
    (dict(lay=2), _lib.EINVAL_ARG), (dict(lay=1, sbn=200), _lib.EINVAL_STRIDE),
    (dict(lay=1, sbn=256, sbg=512 * 256 - 1), _lib.EINVAL_STRIDE),
    (dict(lay=1, sbn=264, sbg=512 * 264), _lib.ELAYOUT),
    (dict(G=0), _lib.OK), (dict(m=0, a=None, b=None, c=None), _lib.OK),
])
def test_fwd_argument_checks(kw, code):
    assert call_fwd(**kw) == code


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-device answer")
def test_fwd_without_device():
    assert call_fwd() == _lib.ENO_DEVICE
    assert _lib.lib().ggemm_vark_grouped_fp8_fwd(P, P, P, P, P, P, 4, 256, 512, 512, 256 * 512,
                                                 512, 256, 1, None) == _lib.ENO_DEVICE


def test_torch_fwd_validates_before_launch():
    a, b, sa, sb, offs = make_fwd([4, 4], N=16, K=32)
    with pytest.raises(ValueError, match="CUDA"):
        grouped_gemm_fp8_tensorwise(a, b, sa, sb, offs)
    with pytest.raises(ValueError, match="K="):
        grouped_gemm_fp8_tensorwise(a, b, sa, sb, offs, trans_b=False)
    with pytest.raises(TypeError):
        grouped_gemm_fp8_tensorwise(a, b.view(E5M2), sa, sb, offs)
    with pytest.raises(ValueError, match="G\\+1"):
        grouped_gemm_fp8_tensorwise(a, b, sa, sb, offs[:-1])
    with pytest.raises(ValueError, match="b_scale"):
        grouped_gemm_fp8_tensorwise(a, b, sa, torch.ones(3), offs)
    with pytest.raises(ValueError, match="b_scale"):
        grouped_gemm_fp8_tensorwise(a, b, sa, torch.ones(2), offs)


# ------------------------------------------------------------------------------------------------
# GPU
# ------------------------------------------------------------------------------------------------
def run_gpu(a, b, sa, sb, offs, out=None, status=None, trans_b=True):
    return grouped_gemm_fp8_tensorwise(a.cuda(), b.cuda(), sa.cuda(), sb.cuda(), offs.cuda(),
                                       trans_b=trans_b, out=out, status=status)


def check(a, b, sa, sb, offs, got, rows=None, trans_b=True):
    ref = vo.grouped_fwd_f32(a, b, sa, sb, offs, rows, trans_b)
    tol = vo.grouped_fwd_tolerance(a, b, sa, sb, offs, ref, rows, trans_b)
    g = (got.cpu() if rows is None else got.cpu()[rows]).float()
    err = (g - ref).abs()
    assert bool((err <= tol).all()), f"max excess {float((err - tol).max())}"
    if ref.abs().max() > 0:
        assert vo.cosine(g, ref) >= 0.99999


@pytest.mark.gpu
@pytest.mark.parametrize("a_dtype", [E4M3, E5M2])
@pytest.mark.parametrize("lens,N,K", [
    ([256], 256, 256),                      # one full tile, one full stage
    ([300, 0, 77, 1, 511], 320, 288),       # ragged experts, N edge 64, K tail 32
    ([1000, 24], 48, 96),                   # N < 256, K < 256
    ([129, 700], 2880, 2880),               # the down sites' N and K (tails 64 and 64)
    ([513], 16, 32),                        # smallest N and K
    ([40] * 40, 272, 128),                  # many small experts, N edge 16
])
def test_fwd_matches_oracle(a_dtype, lens, N, K):
    a, b, sa, sb, offs = make_fwd(lens, N, K, a_dtype, seed=N + K)
    got = run_gpu(a, b, sa, sb, offs)
    torch.cuda.synchronize()
    check(a, b, sa, sb, offs, got)


@pytest.mark.gpu
@pytest.mark.parametrize("lens,N,K", [
    ([256], 256, 256), ([300, 0, 77, 1, 511], 320, 288), ([1000, 24], 48, 96),
    ([129, 700], 2880, 2880), ([513], 32, 32), ([40] * 40, 272, 128), ([64, 64], 96, 544),
])
def test_fwd_b_k_by_n_layout(lens, N, K):
    """trans_b=False: b [G, K, N] (N contiguous, MN-major for the MMA); the item's N rounds up
    to 32 so each CTA's column half starts on a 16-byte boundary."""
    a, b, sa, sb, offs = make_fwd(lens, N, K, E5M2, seed=N * 7 + K, per_expert_scale=True)
    bt = b.transpose(1, 2).contiguous()  # [G, K, N]
    got = run_gpu(a, bt, sa, sb, offs, trans_b=False)
    torch.cuda.synchronize()
    check(a, bt, sa, sb, offs, got, trans_b=False)
    same = run_gpu(a, b, sa, sb, offs)  # the same product with b [G, N, K]
    torch.cuda.synchronize()
    check(a, b, sa, sb, offs, same)


@pytest.mark.gpu
def test_fwd_per_expert_scales_and_status():
    a, b, sa, sb, offs = make_fwd([300, 0, 200, 57], 384, 640, E5M2, seed=3, per_expert_scale=True)
    status = torch.zeros(64, dtype=torch.int32, device="cuda")
    got = run_gpu(a, b, sa, sb, offs, status=status)
    torch.cuda.synchronize()
    assert int(status[0]) == 0
    check(a, b, sa, sb, offs, got)


@pytest.mark.gpu
def test_fwd_rows_outside_experts_untouched():
    """offs[0] > 0 and offs[G] < M: only the experts' rows are written (C store clipped per
    expert), so the sentinel survives elsewhere - including right after a partial token tile."""
    a, b, sa, sb, _ = make_fwd([1100], 256, 256, seed=5)
    offs = torch.tensor([50, 300, 300, 1000], dtype=torch.int64)
    b3 = torch.cat([b, b, b])
    out = torch.full((1100, 256), 7.0, dtype=torch.bfloat16, device="cuda")
    run_gpu(a, b3, sa, sb, offs, out=out)
    torch.cuda.synchronize()
    o = out.cpu()
    assert bool((o[:50] == 7).all()) and bool((o[1000:] == 7).all())
    rows = torch.arange(50, 1000)
    check(a, b3, sa, sb, offs, o, rows)


@pytest.mark.gpu
@pytest.mark.parametrize("trans_b", [True, False])
@pytest.mark.parametrize("N", [20, 100])
def test_fwd_ragged_rows_and_columns_stay_inside(trans_b, N):
    """Experts that end inside a 32-row chunk (their last rows are written with plain stores,
    clipped to the expert) and N not a multiple of 8 (the last piece of a row is written element
    by element): results match the oracle, and a sentinel survives in the padding columns of C
    and in the rows outside the experts."""
    lens, K, lead, tail = [45, 0, 290, 7, 131, 1], 160, 3, 5
    a, b, sa, sb, _ = make_fwd(lens, N, K, seed=N + 17, per_expert_scale=True)
    M, G = sum(lens), len(lens)
    a_all = torch.cat([torch.zeros(lead, K), a.float(), torch.zeros(tail, K)]).to(a.dtype)
    offs = torch.from_numpy(inputs.offsets_from_lens(lens)) + lead
    pitch = (N + 7) // 8 * 8 + 8
    out = torch.full((lead + M + tail, pitch), 7.0, dtype=torch.bfloat16, device="cuda")
    if trans_b:
        bl, bd = b, b.cuda()
    else:
        bl = b.transpose(1, 2).contiguous()  # [G, K, N]
        npad = (N + 15) // 16 * 16           # B rows of a [G, K, N] weight: 16-byte pitch
        bd = torch.zeros(G, K, npad, dtype=torch.uint8, device="cuda")
        bd[:, :, :N] = bl.view(torch.uint8).cuda()
        bd = bd.view(E4M3)[:, :, :N]
    grouped_gemm_fp8_tensorwise(a_all.cuda(), bd, sa.cuda(), sb.cuda(), offs.cuda(),
                                trans_b=trans_b, out=out[:, :N])
    torch.cuda.synchronize()
    o = out.cpu()
    assert bool((o[:, N:] == 7).all()), "padding columns written"
    assert bool((o[:lead] == 7).all()) and bool((o[lead + M:] == 7).all()), "rows outside written"
    check(a_all, bl, sa, sb, offs, o[:, :N], torch.arange(lead, lead + M), trans_b)


@pytest.mark.gpu
@pytest.mark.parametrize("trans_b", [True, False])
@pytest.mark.parametrize("K", [20, 100])
def test_fwd_k_padding_is_not_read(trans_b, K):
    """K not a multiple of 16 with padded rows full of large values: the K tail of the last
    stage must read as zero (TMA fill), so the padding never enters the sums."""
    lens, N = [70, 0, 300, 33], 96
    a, b, sa, sb, offs = make_fwd(lens, N, K, seed=K + 31)
    M, G = sum(lens), len(lens)
    junk = 0x7E  # e4m3fn 448: any padding byte read into a sum moves it far out of tolerance
    kp = (K + 15) // 16 * 16 + 16
    ap = torch.full((M, kp), junk, dtype=torch.uint8)
    ap[:, :K] = a.view(torch.uint8)
    ad = ap.cuda().view(E4M3)[:, :K]
    if trans_b:
        bp = torch.full((G, N, kp), junk, dtype=torch.uint8)
        bp[:, :, :K] = b.view(torch.uint8)
        bd, bl = bp.cuda().view(E4M3)[:, :, :K], b
    else:
        bl = b.transpose(1, 2).contiguous()  # [G, K, N]; its rows are whole N, K is the row index
        bd = bl.cuda()
    got = grouped_gemm_fp8_tensorwise(ad, bd, sa.cuda(), sb.cuda(), offs.cuda(), trans_b=trans_b)
    torch.cuda.synchronize()
    check(a, bl, sa, sb, offs, got, trans_b=trans_b)


@pytest.mark.gpu
def test_fwd_padded_strides_and_14_arg_entry():
    lens, N, K = [333, 222], 272, 320
    a, b, sa, sb, offs = make_fwd(lens, N, K, seed=9)
    ap = torch.zeros(a.shape[0], K + 64, dtype=torch.uint8)
    ap[:, :K] = a.view(torch.uint8)
    bp = torch.zeros(2, N + 8, K + 32, dtype=torch.uint8)
    bp[:, :N, :K] = b.view(torch.uint8)
    ad = ap.cuda().view(E4M3)[:, :K]
    bd = bp.cuda().view(E4M3)[:, :N, :K]
    out = torch.zeros(a.shape[0], N + 8, dtype=torch.bfloat16, device="cuda")[:, :N]
    grouped_gemm_fp8_tensorwise(ad, bd, sa.cuda(), sb.cuda(), offs.cuda(), out=out)
    torch.cuda.synchronize()
    check(a, b, sa, sb, offs, out)
    out2 = torch.zeros_like(out)
    sa_d, sb_d, offs_d = sa.cuda(), sb.cuda(), offs.cuda()
    rc = _lib.lib().ggemm_vark_grouped_fp8_fwd(
        ad.data_ptr(), bd.data_ptr(), out2.data_ptr(), sa_d.data_ptr(), sb_d.data_ptr(),
        offs_d.data_ptr(), 2, N, K, ad.stride(0), bd.stride(0), bd.stride(1), out2.stride(0), 1,
        torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.OK
    torch.cuda.synchronize()
    assert torch.equal(out, out2)


@pytest.mark.gpu
def test_fwd_deterministic():
    a, b, sa, sb, offs = make_fwd([900, 5, 400], 512, 512, seed=11)
    x = run_gpu(a, b, sa, sb, offs)
    y = run_gpu(a, b, sa, sb, offs)
    torch.cuda.synchronize()
    assert torch.equal(x, y)


@pytest.mark.gpu
def test_fwd_bad_offsets_reported():
    a, b, sa, sb, offs = make_fwd([100, 100], 64, 64, seed=2)
    bad = torch.tensor([0, 150, 120], dtype=torch.int64)
    status = torch.zeros(64, dtype=torch.int32, device="cuda")
    run_gpu(a, b, sa, sb, bad, status=status)
    torch.cuda.synchronize()
    assert int(status[0]) & _lib.DEV_BAD_OFFS


@pytest.mark.gpu
def test_fwd_expired_wait_is_reported():
    import time

    a, b, sa, sb, offs = make_fwd([600, 300], 512, 512, seed=4)
    status = torch.zeros(64, dtype=torch.int32, device="cuda")
    status[3] = 0x5374616C
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    grouped_gemm_fp8_tensorwise(a.cuda(), b.cuda(), sa.cuda(), sb.cuda(), offs.cuda(),
                                status=status, timeout_ns=20_000_000)
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 5.0
    assert int(status[0]) & _lib.DEV_TIMEOUT
    got = run_gpu(a, b, sa, sb, offs)
    torch.cuda.synchronize()
    check(a, b, sa, sb, offs, got)


SITES = {  # bench.py:154-181 (M_total = 131072, E = 32)
    "gate_up_fwd": (E4M3, 5760, 2880), "down_fwd": (E4M3, 2880, 2880),
    "down_dgrad": (E5M2, 2880, 2880), "gate_up_dgrad": (E5M2, 2880, 5760),
}


@pytest.mark.gpu
@pytest.mark.parametrize("site", sorted(SITES))
def test_fwd_full_size_site(site):
    """Full-size harness site with the reference generator's routing: every row against the CPU
    oracle's per-element bound (four experts at a time), plus a determinism check."""
    a_dtype, N, K = SITES[site]
    lens = inputs.reference_exponential_lens(32, 131072, seed=42)
    offs = torch.from_numpy(inputs.offsets_from_lens(lens))
    g = torch.Generator(device="cuda").manual_seed(N + K)
    a = torch.randn(131072, K, generator=g, device="cuda").to(torch.bfloat16).to(a_dtype)
    b = torch.randn(32, N, K, generator=g, device="cuda").to(torch.bfloat16).to(E4M3)
    sa = torch.tensor([0.1], device="cuda")
    sb = torch.tensor([0.1], device="cuda")
    out = grouped_gemm_fp8_tensorwise(a, b, sa, sb, offs.cuda())
    torch.cuda.synchronize()
    o = offs.tolist()
    ac, bc, sac, sbc, oc = a.cpu(), b.cpu(), sa.cpu(), sb.cpu(), out.cpu()
    for e0 in range(0, 32, 4):
        rows = torch.arange(o[e0], o[min(32, e0 + 4)])
        if rows.numel():
            check(ac, bc, sac, sbc, offs, oc, rows)
    again = grouped_gemm_fp8_tensorwise(a, b, sa, sb, offs.cuda())
    torch.cuda.synchronize()
    assert torch.equal(out, again)
