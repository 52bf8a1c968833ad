"""The producer step: per-expert amax scaling + fp8 quantisation (ggemm_vark_quantize_fp8).

CPU tests pin the oracle (``quantize_fp8_ref``) against the problem generator and the OCP FP8
code tables, and check the C-ABI argument rules. GPU tests compare the kernel with the oracle
bit for bit (codes and scale bits), on the vector and scalar paths, with empty, ragged,
all-zero, NaN and Inf units, and at the gate_up size.
"""
import numpy as np
import pytest
import torch

from ggemm_asm_b200 import _lib, inputs, quantize_fp8
from oracle import vark_oracle as vo

P = 1 << 20  # fake aligned device address: never dereferenced by the CPU tests


# ------------------------------------------------------------------------------------------------
# CPU: the oracle
# ------------------------------------------------------------------------------------------------
@pytest.mark.parametrize("name,kw", [("tiny", {}),
                                     ("skew", dict(G=8, M_total=20000, OUT_M=32, OUT_N=48)),
                                     ("gate_up", dict(G=5, M_total=9000, OUT_M=24, OUT_N=40))])
def test_oracle_reproduces_the_generator(name, kw):
    p = inputs.make_problem(name, seed=4, **kw)
    per_group = inputs.CONFIGS[name]["scales"] == "group"
    x = inputs.bf16_source(p.M_total, p.OUT_M, 4, 1)
    dy = inputs.bf16_source(p.M_total, p.OUT_N, 4, 2)
    q, s = vo.quantize_fp8_ref(x, p.offs, "e4m3", per_group)
    assert torch.equal(q, p.lhs.view(torch.uint8)) and torch.equal(s, p.lhs_scale)
    q, s = vo.quantize_fp8_ref(dy, p.offs, "e5m2", per_group)
    assert torch.equal(q, p.rhs.view(torch.uint8)) and torch.equal(s, p.rhs_scale)


@pytest.mark.parametrize("fmt", ["e4m3", "e5m2"])
def test_oracle_rounds_to_nearest_even(fmt):
    """Independent of torch's cast: every code is the nearest finite fp8 value to clamp(x/s),
    ties to the even code, checked against the bit-field decode table."""
    _, fmax = vo.FP8_FORMATS[fmt]
    g = torch.Generator().manual_seed(11)
    x = (torch.randn(64, 64, generator=g) * torch.logspace(-6, 0, 64)[None, :]).to(torch.bfloat16)
    q, s = vo.quantize_fp8_ref(x, [0, 64], fmt)
    # the quotient is defined in fp32 (IEEE division); the rounding to fp8 is then exact
    v = np.clip((x.float().numpy() / s.numpy()[0]).astype(np.float64), -fmax, fmax).ravel()
    table = vo.fp8_decode_table({"e4m3": "e4m3fn", "e5m2": "e5m2"}[fmt])
    codes = np.array([c for c in range(256) if np.isfinite(table[c])])
    vals = table[codes]
    got = q.numpy().ravel()
    for vi, ci in zip(v, got):
        d = np.abs(vals - vi)
        best = codes[d == d.min()]
        if best.size > 1:  # tie: the even mantissa (and +0 over -0)
            best = best[(best & 1) == 0]
            if best.size > 1:
                best = best[best < 128] if vi >= 0 else best[best >= 128]
        assert int(ci) == int(best[0]), (vi, ci, best)


def test_oracle_edge_units():
    x = torch.zeros(10, 8, dtype=torch.bfloat16)
    x[4:6] = torch.tensor([1.0, -2.0, 3.0, float("nan"), 0.5, 0.25, 0.125, 4.0]).to(torch.bfloat16)
    x[6:10] = torch.full((4, 8), 3.0).to(torch.bfloat16)
    x[7, 2] = float("inf")
    q, s = vo.quantize_fp8_ref(x, [0, 0, 4, 6, 10], "e4m3")
    assert s[0] == 1.0 and s[1] == 1.0              # empty, all-zero
    assert torch.isnan(s[2]) and torch.isinf(s[3])  # NaN unit, Inf unit
    assert (q[0:4] == 0).all()
    assert (q[6:10].view(torch.float8_e4m3fn).float()[x[6:10].float().isfinite()] == 0).all()


def test_division_free_quotient_is_exact_exhaustively():
    """The kernel replaces x / s by Markstein's correction step (q = x*y, r = fma(-s, q, x),
    q' = fma(r, y, q), y = RN(1/s)). Checked against IEEE division for every bf16 significand and
    every fp32 divisor in [1, 2) - 2^30 pairs, which by exact power-of-two scaling covers all
    normal operands."""
    assert vo.markstein_mismatches() == 0


def test_quotient_checker_detects_a_planted_error(tmp_path):
    """A checker that cannot fail proves nothing: a copy of the C check with the correction step
    removed (q' = q) must report mismatches."""
    import ctypes
    import shutil
    import subprocess

    if shutil.which("gcc") is None:
        pytest.skip("gcc not available")
    src = (vo.HERE / "vark_oracle_c.c").read_text()
    planted = src.replace("const float q2 = __builtin_fmaf(r, y, q);", "const float q2 = q + 0.0f * r;")
    planted = planted.replace("const float q2 = fmaf(r, y, q);", "const float q2 = q + 0.0f * r;")
    assert planted.count("q + 0.0f * r") == 2
    (tmp_path / "planted.c").write_text(planted)
    so = tmp_path / "planted.so"
    subprocess.run(["gcc", "-O2", "-fPIC", "-std=gnu11", "-ffp-contract=off", "-shared", "-o",
                    str(so), str(tmp_path / "planted.c"), "-lm"], check=True)
    f = ctypes.CDLL(str(so)).vark_oracle_markstein_mismatches
    f.restype, f.argtypes = ctypes.c_long, [ctypes.c_uint32, ctypes.c_uint32]
    assert f(0, 1 << 16) > 0


# ------------------------------------------------------------------------------------------------
# CPU: the C ABI
# ------------------------------------------------------------------------------------------------
def call_q(**kw):
    a = dict(x=P, q=P, s=P, offs=P, G=4, F=64, sx=64, sq=64, fmt=0, pg=1, m=1024, ws=P,
             status=None)
    a.update(kw)
    return _lib.lib().ggemm_vark_quantize_fp8(a["x"], a["q"], a["s"], a["offs"], a["G"], a["F"],
                                              a["sx"], a["sq"], a["fmt"], a["pg"], a["m"],
                                              a["ws"], a["status"], 0, None)


@pytest.mark.parametrize("kw,code", [
    (dict(s=None), _lib.EINVAL_PTR), (dict(offs=None), _lib.EINVAL_PTR),
    (dict(ws=None), _lib.EINVAL_PTR), (dict(x=None), _lib.EINVAL_PTR),
    (dict(G=-1), _lib.EINVAL_SHAPE), (dict(F=0), _lib.EINVAL_SHAPE),
    (dict(sx=63), _lib.EINVAL_STRIDE), (dict(sq=10), _lib.EINVAL_STRIDE),
    (dict(fmt=2), _lib.EINVAL_ARG), (dict(pg=2), _lib.EINVAL_ARG), (dict(m=-2), _lib.EINVAL_ARG),
    (dict(ws=P + 8), _lib.EINVAL_ARG), (dict(status=P + 4), _lib.EINVAL_ARG),
    (dict(x=P + 1), _lib.EINVAL_ARG), (dict(G=0), _lib.OK),
])
def test_quantize_argument_checks(kw, code):
    assert call_q(**kw) == code


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-device answer")
def test_quantize_without_device():
    assert call_q() == _lib.ENO_DEVICE


def test_workspace_size():
    f = _lib.lib().ggemm_vark_quantize_workspace_bytes
    assert f(0) == 16 and f(32) == 16 + 8 * 32 and f(1) % 8 == 0


def test_torch_quantize_validates_before_launch():
    x = torch.zeros(8, 16, dtype=torch.bfloat16)
    offs = torch.tensor([0, 8])
    with pytest.raises(ValueError, match="CUDA"):
        quantize_fp8(x, offs)
    with pytest.raises(ValueError, match="fmt"):
        quantize_fp8(x, offs, "e3m4")
    with pytest.raises(ValueError, match="bfloat16"):
        quantize_fp8(x.float(), offs)
    with pytest.raises(ValueError, match="int64"):
        quantize_fp8(x, offs.int())


# ------------------------------------------------------------------------------------------------
# GPU: parity with the oracle
# ------------------------------------------------------------------------------------------------
def _same_codes(got_u8: torch.Tensor, ref_u8: torch.Tensor, fmt: str) -> bool:
    """Bit-equal codes, except that any NaN code matches any NaN code (the sign of a NaN is not
    specified by the op)."""
    dtype, _ = vo.FP8_FORMATS[fmt]
    gn = got_u8.view(dtype).float().isnan()
    rn = ref_u8.view(dtype).float().isnan()
    return bool(torch.equal(gn, rn) and torch.equal(got_u8[~gn], ref_u8[~rn]))


def _same_scales(got: torch.Tensor, ref: torch.Tensor) -> bool:
    gn, rn = got.isnan(), ref.isnan()
    return bool(torch.equal(gn, rn) and torch.equal(got[~gn].view(torch.int32),
                                                     ref[~rn].view(torch.int32)))


def _check(x_cpu, lens, fmt, granularity, pitch=None):
    offs = torch.from_numpy(inputs.offsets_from_lens(lens))
    rows, F = x_cpu.shape
    if pitch is None:
        xd = x_cpu.cuda()
    else:
        base = torch.zeros(rows, pitch, dtype=torch.bfloat16, device="cuda")
        base[:, :F] = x_cpu.cuda()
        xd = base[:, :F]
    status = torch.zeros(64, dtype=torch.int32, device="cuda")
    q, s = quantize_fp8(xd, offs.cuda(), fmt, granularity=granularity, status=status)
    torch.cuda.synchronize()
    assert int(status[0]) == 0
    ref_q, ref_s = vo.quantize_fp8_ref(x_cpu, offs, fmt, granularity == "group")
    units = len(lens) if granularity == "group" else 1
    assert _same_scales(s.cpu()[:units], ref_s)
    lo, hi = int(offs[0]), int(offs[-1])
    assert _same_codes(q.view(torch.uint8).cpu()[lo:hi], ref_q[lo:hi], fmt)


def _randn(rows, F, seed, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(rows, F, generator=g) * scale).to(torch.bfloat16)


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", ["e4m3", "e5m2"])
@pytest.mark.parametrize("granularity", ["group", "tensor"])
@pytest.mark.parametrize("lens,F", [([256, 0, 512, 256], 64), ([300, 0, 77, 1, 160, 487], 2880),
                                    ([5, 0, 1000, 3], 100), ([1], 8), ([0, 0, 64], 24)])
def test_quantize_matches_oracle(fmt, granularity, lens, F):
    x = _randn(sum(lens), F, seed=F + len(lens))
    _check(x, lens, fmt, granularity)


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", ["e4m3", "e5m2"])
@pytest.mark.parametrize("F,pitch", [(64, 72), (64, 67), (2880, 2944), (40, 41)])
def test_quantize_padded_rows(fmt, F, pitch):
    """Row pitch larger than the row: 16-byte multiples take the vector path, others the scalar."""
    lens = [129, 0, 300, 31]
    _check(_randn(sum(lens), F, seed=pitch), lens, fmt, "group", pitch=pitch)


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", ["e4m3", "e5m2"])
def test_quantize_special_units(fmt):
    """All-zero unit (scale 1.0), NaN unit (NaN scale, NaN codes), Inf unit (Inf scale: finite
    values go to 0, the Inf to NaN), tiny values that land on fp8 subnormals, and values at the
    clamp (x = amax exactly, whose quotient may round above FMAX before saturation)."""
    F = 32
    lens = [64, 64, 64, 64, 64]
    x = _randn(sum(lens), F, seed=3)
    x[0:64] = 0
    x[64 + 5, 7] = float("nan")
    x[128 + 9, 1] = float("-inf")
    x[192:256] = (x[192:256].float() * 1e-30).to(torch.bfloat16)
    x[192, 0] = 1.0  # amax of that unit: everything else lands far below, in the subnormals
    x[256 + 3, :] = (x[256:320].float().abs().max()).to(torch.bfloat16)
    _check(x, lens, fmt, "group")


def _all_bf16_up_to(amax: float) -> torch.Tensor:
    """Every finite bf16 value v with |v| <= amax (both signs, zeros included), amax included."""
    bits = torch.arange(0, 0x7f80, dtype=torch.int32).to(torch.int16)
    pos = bits.view(torch.bfloat16)
    pos = pos[pos.float() <= amax]
    vals = torch.cat([pos, -pos, torch.tensor([amax], dtype=torch.bfloat16)])
    pad = (-vals.numel()) % 64
    return torch.cat([vals, torch.zeros(pad, dtype=torch.bfloat16)]).reshape(-1, 64)


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", ["e4m3", "e5m2"])
def test_quantize_every_bf16_value(fmt):
    """Exhaustive over the inputs: each unit holds every finite bf16 value up to its amax, for
    amax values whose scale s = amax/FMAX is not a power of two (the reciprocal-product route
    and its exact fallback both decide) and for powers of two (s exact)."""
    amaxes = [1.0, 3.0, 0.0123, 448.0, 300.0, 57344.0, 1.7e-3, 2.0 ** -20, 6.1e4, 1e30]
    parts = [_all_bf16_up_to(float(torch.tensor(a).to(torch.bfloat16))) for a in amaxes]
    lens = [t.shape[0] for t in parts]
    _check(torch.cat(parts), lens, fmt, "group")


@pytest.mark.gpu
def test_quantize_bad_offsets_reported():
    x = _randn(100, 16, seed=1).cuda()
    offs = torch.tensor([0, 50, 40, 100, 400], dtype=torch.int64, device="cuda")
    status = torch.zeros(64, dtype=torch.int32, device="cuda")
    q = torch.zeros(100, 16, dtype=torch.float8_e4m3fn, device="cuda")
    _, s = quantize_fp8(x, offs, "e4m3", out=q, status=status)
    torch.cuda.synchronize()
    assert int(status[0]) & _lib.DEV_BAD_OFFS
    assert float(s[1]) == 1.0 and float(s[3]) == 1.0           # 50 -> 40 and past m_total
    ref_q, ref_s = vo.quantize_fp8_ref(x.cpu(), [0, 50], "e4m3")
    # rows 40..49 belong to two (overlapping) valid units; rows below 40 to unit 0 alone
    assert torch.equal(q.view(torch.uint8).cpu()[:40], ref_q[:40]) and torch.equal(s[0].cpu(), ref_s[0])


@pytest.mark.gpu
def test_quantize_no_rows():
    offs = torch.zeros(4, dtype=torch.int64, device="cuda")
    x = torch.empty(0, 64, dtype=torch.bfloat16, device="cuda")
    q, s = quantize_fp8(x, offs, "e5m2")
    torch.cuda.synchronize()
    assert q.shape == (0, 64) and torch.equal(s.cpu(), torch.ones(3))


@pytest.mark.gpu
def test_quantize_feeds_the_wgrad():
    """Producer -> wgrad on the device gives exactly the wgrad of the generator's operands."""
    from ggemm_asm_b200 import grouped_gemm_fp8_tensorwise_variable_k as vark

    p = inputs.make_problem("skew", seed=8, G=6, M_total=5000, OUT_M=256, OUT_N=384)
    x = inputs.bf16_source(p.M_total, p.OUT_M, 8, 1).cuda()
    dy = inputs.bf16_source(p.M_total, p.OUT_N, 8, 2).cuda()
    offs = p.group_offs.cuda()
    lhs, sl = quantize_fp8(x, offs, "e4m3")
    rhs, sr = quantize_fp8(dy, offs, "e5m2")
    torch.cuda.synchronize()
    assert torch.equal(lhs.view(torch.uint8).cpu(), p.lhs.view(torch.uint8))
    assert torch.equal(sl.cpu(), p.lhs_scale) and torch.equal(sr.cpu(), p.rhs_scale)
    got = vark(lhs, rhs, sl, sr, offs)
    ref = vark(p.lhs.cuda(), p.rhs.cuda(), p.lhs_scale.cuda(), p.rhs_scale.cuda(), offs)
    assert torch.equal(got, ref)


@pytest.mark.gpu
@pytest.mark.parametrize("fmt,F", [("e4m3", 2880), ("e5m2", 5760)])
def test_quantize_full_size_gate_up(fmt, F):
    """gate_up size (131072 tokens, 32 experts): larger than L2, so the second read of each expert
    is checked where it matters. Three experts against the CPU oracle; every expert against the
    same formula evaluated with torch on the device."""
    lens = inputs.config_lens("gate_up", seed=0)
    offs = torch.from_numpy(inputs.offsets_from_lens(lens))
    g = torch.Generator(device="cuda").manual_seed(F)
    x = torch.randn(int(lens.sum()), F, generator=g, device="cuda").to(torch.bfloat16)
    q, s = quantize_fp8(x, offs.cuda(), fmt)
    torch.cuda.synchronize()
    dtype, fmax = vo.FP8_FORMATS[fmt]
    for e in (0, 17, 31):
        lo, hi = int(offs[e]), int(offs[e + 1])
        rq, rs = vo.quantize_fp8_ref(x[lo:hi].cpu(), [0, hi - lo], fmt)
        assert _same_scales(s[e:e + 1].cpu(), rs)
        assert torch.equal(q[lo:hi].view(torch.uint8).cpu(), rq)
    fm = torch.tensor(fmax, device="cuda")
    for e in range(len(lens)):
        lo, hi = int(offs[e]), int(offs[e + 1])
        se = x[lo:hi].float().abs().amax() / fm
        assert torch.equal(s[e], se)
        ref = (x[lo:hi].float() / se).clamp(-fmax, fmax).to(dtype)
        assert torch.equal(q[lo:hi].view(torch.uint8), ref.view(torch.uint8)), e


@pytest.mark.gpu
@pytest.mark.parametrize("granularity", ["group", "tensor"])
def test_quantize_long_slices(granularity):
    """Units of 50-130 MB: each CTA's slice is cut into many equal bulk-copy chunks whose sizes
    are not a power of two (rows of 2000 bytes, slices of odd vector counts). Every unit against
    the quotient formula evaluated with torch on the device."""
    lens = [40000, 3, 25001]
    F = 1000
    offs = torch.from_numpy(inputs.offsets_from_lens(lens))
    g = torch.Generator(device="cuda").manual_seed(77)
    x = (torch.randn(sum(lens), F, generator=g, device="cuda") * 3.0).to(torch.bfloat16)
    q, s = quantize_fp8(x, offs.cuda(), "e4m3", granularity=granularity)
    torch.cuda.synchronize()
    dtype, fmax = vo.FP8_FORMATS["e4m3"]
    fm = torch.tensor(fmax, device="cuda")
    units = [(0, len(lens))] if granularity == "tensor" else [(e, e + 1) for e in range(len(lens))]
    for u, (a, b) in enumerate(units):
        lo, hi = int(offs[a]), int(offs[b])
        su = x[lo:hi].float().abs().amax() / fm
        assert torch.equal(s[u], su)
        ref = (x[lo:hi].float() / su).clamp(-fmax, fmax).to(dtype)
        assert torch.equal(q[lo:hi].view(torch.uint8), ref.view(torch.uint8)), u


@pytest.mark.gpu
def test_quantize_expired_wait_is_reported():
    """Test hook: CTA 0 withholds its first arrival, so every CTA's wait expires; the call stops
    by itself, reports GGEMM_VARK_DEV_TIMEOUT, and the next call is correct."""
    import time

    lens = [3000, 2000]
    x = _randn(sum(lens), 256, seed=9)
    offs = torch.from_numpy(inputs.offsets_from_lens(lens)).cuda()
    status = torch.zeros(64, dtype=torch.int32, device="cuda")
    status[3] = 0x5374616C
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    quantize_fp8(x.cuda(), offs, "e4m3", status=status, timeout_ns=20_000_000)
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 5.0
    assert int(status[0]) & _lib.DEV_TIMEOUT
    _check(x, lens, "e4m3", "group")
