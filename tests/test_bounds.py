"""The drop-in entry points read no token row at or past group_offs[G].

The reference's kernel arguments (README.md:88-95, bench.py:376-385) carry no M_total: the only
token count a drop-in sees is group_offs[G], and a caller that allocated exactly that many rows
(launcher.cpp:90-91 allocates M_TOTAL x OUT_M bytes) must not have a load run past the end of its
buffer. These tests place the operands at the start of buffers with 256 slack rows after
group_offs[G], fill the slack with NaN bytes, call the entry points without M_total, and check
  * the results against the CPU oracle (a NaN read into any sum would break them), and
  * the status words that record the end of the highest token row any TMA load could read
    (GGEMM_VARK_STATUS_WORD_LHS_ROWS / _RHS_ROWS): exactly group_offs[G] - the last group's
    rows are read, and none past them.
With M_total given the same words never exceed it (the hardware clips boxes at the map's end).
"""
import pytest
import torch

from ggemm_asm_b200 import _lib, inputs, launch_raw
from oracle import vark_oracle as vo

pytestmark = pytest.mark.gpu
NAN = 0x7F  # NaN in both e4m3fn and e5m2
SLACK = 256

LENS = [
    [300, 0, 77, 160, 487],   # last group: two full blocks, 3 whole steps and a 7-token tail
    [64, 200, 384],           # last group ends on a block boundary: no tail
    [1000, 5],                # last group only a tail (moved back over the group before)
    [500, 33, 0, 0],          # trailing empty groups
    [7],                      # one group shorter than a K step: the tail starts at row -25
    [100],                    # one group shorter than a block: the block starts at row -92
    [7] * 300,                # many tails, only the last one crosses
    [3000, 129],              # a last block with 4 whole steps and a 1-token tail
]
SHAPES = [(272, 384), (304, 320), (2880, 128)]  # narrow edges of both operands, 64-row edges


def _slack(t):
    """A device copy of `t` followed by SLACK rows of NaN bytes; returns the view of `t`'s rows."""
    buf = torch.full((t.shape[0] + SLACK, t.shape[1]), NAN, dtype=torch.uint8, device="cuda")
    buf[:t.shape[0]] = t.view(torch.uint8).cuda()
    return buf[:t.shape[0]].view(t.dtype)


def _check(p, out, label):
    ref32 = vo.wgrad_torch_f32(p.lhs, p.rhs, p.lhs_scale, p.rhs_scale, p.group_offs)
    tol = vo.tolerance(p.lhs, p.rhs, p.lhs_scale, p.rhs_scale, p.group_offs, ref32)
    got = out.float().cpu()
    err = (got - ref32.to(torch.bfloat16).float()).abs()
    assert not bool(torch.isnan(got).any()), f"{label}: NaN from the slack rows"
    assert bool((err <= tol).all()), f"{label}: max err {err.max().item()}"
    assert vo.cosine(got, ref32) >= 0.99999, label


def _ex(d, lhs, rhs, out, m_total, path, status):
    return _lib.lib().ggemm_vark_fp8_wgrad_ex(
        lhs.data_ptr(), rhs.data_ptr(), out.data_ptr(), d.lhs_scale.data_ptr(),
        d.rhs_scale.data_ptr(), d.group_offs.data_ptr(), d.G, d.OUT_M, d.OUT_N, lhs.stride(0),
        rhs.stride(0), out.stride(0), out.stride(1), out.stride(2), m_total, 0, path,
        status.data_ptr(), 0, torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("shape", SHAPES, ids=[f"{m}x{n}" for m, n in SHAPES])
@pytest.mark.parametrize("lens", LENS, ids=[str(i) for i in range(len(LENS))])
def test_fourteen_argument_wgrad_stays_inside(lens, shape):
    """ggemm_vark_fp8_wgrad (the pair kernel, reached as the reference harness reaches it)."""
    p = inputs.make_problem("tiny", seed=len(lens) + shape[0], lens=lens, OUT_M=shape[0],
                            OUT_N=shape[1])
    d = p.to("cuda")
    lhs, rhs = _slack(p.lhs), _slack(p.rhs)
    out = torch.full((p.G, p.OUT_M, p.OUT_N), 3.0, dtype=torch.bfloat16, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    _lib.read_status_words(None, 8, clear=True, stream=stream)
    launch_raw(lhs.data_ptr(), rhs.data_ptr(), out.data_ptr(), d.lhs_scale.data_ptr(),
               d.rhs_scale.data_ptr(), d.group_offs.data_ptr(), p.G, p.OUT_M, p.OUT_N,
               lhs.stride(0), rhs.stride(0), out.stride(0), out.stride(1), out.stride(2), stream)
    w = _lib.read_status_words(None, 8, clear=True, stream=stream)
    assert w[_lib.STATUS_WORD_BITS] == 0
    assert w[_lib.STATUS_WORD_LHS_ROWS] == p.M_total, w
    assert w[_lib.STATUS_WORD_RHS_ROWS] == p.M_total, w
    _check(p, out, f"14-arg {lens} {shape}")


@pytest.mark.parametrize("path", ["tcgen05", "tcgen05_1sm", "noalloc"])
@pytest.mark.parametrize("lens", LENS, ids=[str(i) for i in range(len(LENS))])
def test_unknown_m_total_on_every_tensor_core_path(lens, path):
    """m_total = -1 through ggemm_vark_fp8_wgrad_ex (both tensor-core kernels) and the
    allocation-free entry point, with a caller status block; then the same call with m_total
    given, whose recorded rows never exceed it."""
    p = inputs.make_problem("tiny", seed=7 * len(lens), lens=lens, OUT_M=272, OUT_N=384)
    d = p.to("cuda")
    lhs, rhs = _slack(p.lhs), _slack(p.rhs)
    for m_total in (-1, p.M_total):
        status = torch.zeros(64, dtype=torch.int32, device="cuda")
        out = torch.full((p.G, p.OUT_M, p.OUT_N), 3.0, dtype=torch.bfloat16, device="cuda")
        if path == "noalloc":
            rc = _lib.lib().ggemm_vark_fp8_wgrad_noalloc(
                lhs.data_ptr(), rhs.data_ptr(), out.data_ptr(), d.lhs_scale.data_ptr(),
                d.rhs_scale.data_ptr(), d.group_offs.data_ptr(), p.G, p.OUT_M, p.OUT_N,
                lhs.stride(0), rhs.stride(0), out.stride(0), out.stride(1), out.stride(2),
                m_total, 0, status.data_ptr(), torch.cuda.current_stream().cuda_stream)
        else:
            code = _lib.PATH_TCGEN05 if path == "tcgen05" else _lib.PATH_TCGEN05_1SM
            rc = _ex(d, lhs, rhs, out, m_total, code, status)
        assert rc == _lib.OK
        torch.cuda.synchronize()
        s = status.cpu().tolist()
        assert s[_lib.STATUS_WORD_BITS] == 0
        assert s[_lib.STATUS_WORD_LHS_ROWS] == p.M_total, (m_total, s[:8])
        assert s[_lib.STATUS_WORD_RHS_ROWS] == p.M_total, (m_total, s[:8])
        _check(p, out, f"{path} m_total={m_total} {lens}")


def test_offsets_past_the_token_count_are_invalid_without_m_total():
    """Without M_total, group_offs[G] is the token count: a group reaching past it is reported
    and written as zeros, and nothing past group_offs[G] is read."""
    p = inputs.make_problem("tiny", seed=5, lens=[64, 64, 64, 64], OUT_M=256, OUT_N=256)
    d = p.to("cuda")
    lhs, rhs = _slack(p.lhs), _slack(p.rhs)
    d.group_offs = torch.tensor([0, 64, 250, 128, 200], dtype=torch.int64, device="cuda")
    status = torch.zeros(64, dtype=torch.int32, device="cuda")
    out = torch.full((4, 256, 256), 3.0, dtype=torch.bfloat16, device="cuda")
    assert _ex(d, lhs, rhs, out, -1, _lib.PATH_TCGEN05, status) == _lib.OK
    torch.cuda.synchronize()
    s = status.cpu().tolist()
    assert s[0] & _lib.DEV_BAD_OFFS
    assert bool((out[1] == 0).all())  # [64, 250) reaches past group_offs[G] = 200
    assert s[_lib.STATUS_WORD_LHS_ROWS] <= 200 and s[_lib.STATUS_WORD_RHS_ROWS] <= 200


FWD_CASES = [([333, 222], 272, 320), ([300, 0, 77, 1, 511], 320, 288), ([40] * 9, 96, 128),
             ([100], 64, 64), ([256, 256], 256, 256)]


@pytest.mark.parametrize("lens,N,K", FWD_CASES, ids=[str(i) for i in range(len(FWD_CASES))])
def test_fourteen_argument_fwd_stays_inside(lens, N, K):
    """ggemm_vark_grouped_fp8_fwd (14 arguments, no M_total): the A rows its loads can reach end
    at group_offs[G], and C rows past it keep their sentinel; the results match the oracle and
    the m_total-given call bit for bit (moving a box only changes which TMEM lane holds a row)."""
    g = torch.Generator().manual_seed(N + K)
    M, G = sum(lens), len(lens)
    a = torch.randn(M, K, generator=g).to(torch.bfloat16).to(torch.float8_e4m3fn)
    b = torch.randn(G, N, K, generator=g).to(torch.bfloat16).to(torch.float8_e4m3fn)
    sa, sb = torch.tensor([0.1]), torch.tensor([0.1])
    offs = torch.from_numpy(inputs.offsets_from_lens(lens))
    ad = _slack(a)
    bd, sad, sbd, offd = b.cuda(), sa.cuda(), sb.cuda(), offs.cuda()
    cbuf = torch.full((M + SLACK, N), 7.0, dtype=torch.bfloat16, device="cuda")
    out = cbuf[:M]
    stream = torch.cuda.current_stream().cuda_stream
    _lib.read_status_words(None, 8, clear=True, stream=stream)
    rc = _lib.lib().ggemm_vark_grouped_fp8_fwd(
        ad.data_ptr(), bd.data_ptr(), out.data_ptr(), sad.data_ptr(), sbd.data_ptr(),
        offd.data_ptr(), G, N, K, ad.stride(0), bd.stride(0), bd.stride(1), out.stride(0), 1,
        stream)
    assert rc == _lib.OK
    w = _lib.read_status_words(None, 8, clear=True, stream=stream)
    assert w[_lib.STATUS_WORD_BITS] == 0
    assert w[_lib.STATUS_WORD_LHS_ROWS] == M, w
    assert bool((cbuf[M:] == 7.0).all())
    ref = vo.grouped_fwd_f32(a, b, sa, sb, offs)
    tol = vo.grouped_fwd_tolerance(a, b, sa, sb, offs, ref)
    assert bool(((out.float().cpu() - ref).abs() <= tol).all())
    from ggemm_asm_b200 import grouped_gemm_fp8_tensorwise

    known = grouped_gemm_fp8_tensorwise(ad, bd, sad, sbd, offd)
    torch.cuda.synchronize()
    assert torch.equal(known, out)
