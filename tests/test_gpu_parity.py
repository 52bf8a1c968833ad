"""GPU parity: the CUDA paths (through the C ABI) against the CPU oracle on identical bytes.

Tolerance (stated by the north star, implemented in oracle.vark_oracle.tolerance):
    |C - oracle| <= 1 ulp_bf16(|oracle_fp32|) + 2 * K_g * 2^-24 * sL*sR * (|LHS_g|^T |RHS_g|)
per element, and cosine(C, oracle) >= 0.99999 over the whole output.
"""
import pytest
import torch

from ggemm_asm_b200 import _lib, grouped_gemm_fp8_tensorwise_variable_k as vark, inputs, launch_raw
from oracle import vark_oracle as vo

pytestmark = pytest.mark.gpu
COS_MIN = 0.99999


def _check(problem, out, groups=None, label=""):
    p = problem
    ref32 = vo.wgrad_torch_f32(p.lhs, p.rhs, p.lhs_scale, p.rhs_scale, p.group_offs, groups)
    tol = vo.tolerance(p.lhs, p.rhs, p.lhs_scale, p.rhs_scale, p.group_offs, ref32, groups)
    got = out.float().cpu()
    if groups is not None:
        got = got[list(groups)]
    ref = ref32.to(torch.bfloat16).float()
    err = (got - ref).abs()
    bad = ~(err <= tol)
    assert not bool(bad.any()), (
        f"{label}: {int(bad.sum())} elements out of tolerance; max err {err.max().item():.4g}, "
        f"first at {tuple(int(i) for i in bad.nonzero()[0])}")
    cos = vo.cosine(got, ref32)
    assert cos >= COS_MIN, f"{label}: cosine {cos}"
    for i, g in enumerate(range(p.G) if groups is None else groups):
        if p.lens[g] == 0:
            assert bool((got[i] == 0).all()), f"{label}: empty group {g} not zero"
    return cos, err.max().item()


def _check_all(problem, out, label, chunk=4):
    """Every expert of a (full-size) problem against the oracle, `chunk` experts at a time so
    that the CPU holds one chunk's fp32 result and bound at once; the cosine is taken over the
    whole output, and empty experts must be exact zeros."""
    p = problem
    dot = na = nb = 0.0
    worst = 0.0
    for g0 in range(0, p.G, chunk):
        gs = list(range(g0, min(p.G, g0 + chunk)))
        ref32 = vo.wgrad_torch_f32(p.lhs, p.rhs, p.lhs_scale, p.rhs_scale, p.group_offs, gs)
        tol = vo.tolerance(p.lhs, p.rhs, p.lhs_scale, p.rhs_scale, p.group_offs, ref32, gs)
        got = out[gs[0]:gs[-1] + 1].float().cpu()
        err = (got - ref32.to(torch.bfloat16).float()).abs()
        bad = ~(err <= tol)
        assert not bool(bad.any()), (
            f"{label}: experts {gs}: {int(bad.sum())} elements out of tolerance; max err "
            f"{err.max().item():.4g}, first at {tuple(int(i) for i in bad.nonzero()[0])}")
        worst = max(worst, float((err / tol.clamp_min(1e-30)).max()))
        a, b = got.double(), ref32.double()
        dot += float((a * b).sum())
        na += float((a * a).sum())
        nb += float((b * b).sum())
        for i, g in enumerate(gs):
            if p.lens[g] == 0:
                assert bool((got[i] == 0).all()), f"{label}: empty group {g} not zero"
    cos = 1.0 if na == 0 and nb == 0 else dot / (na * nb) ** 0.5
    assert cos >= COS_MIN, f"{label}: cosine {cos}"
    return cos, worst


def _run(p, path="auto", out=None):
    d = p.to("cuda")
    o = vark(d.lhs, d.rhs, d.lhs_scale, d.rhs_scale, d.group_offs, out=out, path=path)
    torch.cuda.synchronize()
    assert _lib.read_status(clear=True) == 0
    return o


TC_PATHS = ["tcgen05", "tcgen05_1sm"]
ALL_PATHS = TC_PATHS + ["simt"]


@pytest.mark.parametrize("path", ALL_PATHS)
def test_tiny_config(path):
    p = inputs.make_problem("tiny", seed=0)
    assert p.offs.tolist() == [0, 256, 256, 768, 1024]
    _check(p, _run(p, path), label=f"tiny/{path}")


RAGGED = [
    [1],
    [31, 32, 33],
    [127, 128, 129, 255, 256, 257],
    [5, 0, 0, 1000, 0, 3],
    [300, 0, 77, 160, 487],
    [0, 0, 0],
    [4096],
    # hundreds of groups, so each CTA pair works through many items: every item below 32 tokens
    # is only a ragged tail step, and the tail buffers are reused item after item
    [7] * 300,
    [(i * 37) % 101 for i in range(240)],  # tails only, whole steps only, and mixed
]


@pytest.mark.parametrize("lens", RAGGED, ids=[str(i) for i in range(len(RAGGED))])
@pytest.mark.parametrize("path", ALL_PATHS)
def test_ragged_groups(lens, path):
    p = inputs.make_problem("tiny", seed=3, lens=lens, OUT_M=272, OUT_N=384)
    _check(p, _run(p, path), label=f"ragged{lens}/{path}")


@pytest.mark.parametrize("shape", [(240, 128), (480, 256), (16, 16), (2880, 128), (64, 5760),
                                   (496, 400), (256, 256), (272, 272), (128, 640),
                                   # last column tile widths 64, 96, 224, 32, 192 (transposed
                                   # items; 256 x 192 is the MoE layer test's weight gradient)
                                   (2880, 2880), (112, 96), (304, 480), (48, 224), (512, 32),
                                   (256, 192),
                                   # last row tile of 32 or 64 rows, or OUT_M < 32: B through
                                   # the narrow 32-byte boxes
                                   (288, 256), (320, 384), (16, 304)])
@pytest.mark.parametrize("path", TC_PATHS)
def test_tile_edges(shape, path):
    OUT_M, OUT_N = shape
    p = inputs.make_problem("tiny", seed=5, lens=[200, 57, 0, 301], OUT_M=OUT_M, OUT_N=OUT_N)
    _check(p, _run(p, path), label=f"edges{shape}/{path}")


def test_tc_paths_agree_with_simt():
    p = inputs.make_problem("tiny", seed=7, lens=[700, 1, 300, 2000], OUT_M=480, OUT_N=512)
    a = _run(p, "tcgen05").float()
    b = _run(p, "simt").float()
    c = _run(p, "tcgen05_1sm").float()
    assert vo.cosine(a, b) >= COS_MIN and vo.cosine(c, b) >= COS_MIN


@pytest.mark.parametrize("path", ALL_PATHS)
def test_per_group_scales(path):
    p = inputs.make_problem("skew", seed=11, G=8, M_total=3000, OUT_M=240, OUT_N=256)
    assert p.lhs_scale.numel() == 8
    _check(p, _run(p, path), label=f"per-group/{path}")


@pytest.mark.parametrize("path", TC_PATHS)
def test_launcher_closed_form(path):
    """The reference launcher's workload (launcher.cpp:97-112), shrunk: exact known answer."""
    p = inputs.launcher_problem("gate_up_wgrad", G=8, M_total=8 * 1000 + 5)
    p = inputs.Problem(**{**p.__dict__, "OUT_M": 480, "OUT_N": 256,
                          "lhs": p.lhs[:, :480].contiguous(), "rhs": p.rhs[:, :256].contiguous()})
    out = _run(p, path).float().cpu()
    for g in range(p.G):
        expect = vo.closed_form_launcher_value(int(p.lens[g]))
        assert bool((out[g] == expect).all()), (g, out[g].unique()[:4], expect)


@pytest.mark.parametrize("where", ["middle group", "after the last group"])
@pytest.mark.parametrize("path", TC_PATHS)
def test_neighbour_nan_does_not_leak(path, where):
    """Tokens that are not a group's own never enter its sum, even as NaN or Inf in both
    operands: a group's last token block reaches into the next group's rows (or rows past the
    last group) and the kernel zeroes those rows in both operands before the MMA."""
    p = inputs.make_problem("tiny", seed=13, lens=[100, 50, 200], OUT_M=240, OUT_N=128)
    lhs = p.lhs.view(torch.uint8).clone()
    rhs = p.rhs.view(torch.uint8).clone()
    if where == "middle group":
        lhs[100:150] = 0x7F  # e4m3fn NaN
        rhs[100:150] = 0x7C  # e5m2 +Inf
        clean = [0, 2]
    else:  # 300 poisoned rows after offs[G]; the operands (and m_total) include them
        lhs = torch.cat([lhs, torch.full((300, lhs.shape[1]), 0x7F, dtype=torch.uint8)])
        rhs = torch.cat([rhs, torch.full((300, rhs.shape[1]), 0x7C, dtype=torch.uint8)])
        clean = [0, 1, 2]
    q = inputs.Problem(**{**p.__dict__, "lhs": lhs.view(torch.float8_e4m3fn),
                          "rhs": rhs.view(torch.float8_e5m2)})
    out = _run(q, path)
    if where == "middle group":
        assert bool(torch.isnan(out[1].float()).any() or torch.isinf(out[1].float()).any())
    _check(q, out, groups=clean, label=f"nan-neighbour/{where}")


@pytest.mark.parametrize("path", TC_PATHS)
def test_padded_output_strides(path):
    p = inputs.make_problem("tiny", seed=17, lens=[333, 0, 444], OUT_M=272, OUT_N=384)
    big = torch.full((3, 272 + 8, 384 + 64), 7.0, dtype=torch.bfloat16, device="cuda")
    view = big[:, :272, :384]
    assert _lib.lib().ggemm_vark_tc_supported(1 << 20, 1 << 20, view.data_ptr(), 272, 384, 272,
                                              384, view.stride(0), view.stride(1), 1) == 1
    _run(p, path, out=view)
    _check(p, view, label=f"padded-C/{path}")
    assert bool((big[:, 272:, :] == 7.0).all()) and bool((big[:, :, 384:] == 7.0).all())


def test_unaligned_layout_takes_simt():
    p = inputs.make_problem("tiny", seed=19, lens=[90, 10, 0, 155], OUT_M=100, OUT_N=72)
    d = p.to("cuda")
    wide_l = torch.zeros(255, 101 + 3, dtype=torch.uint8, device="cuda")
    wide_l[:, 3:103] = d.lhs.view(torch.uint8)
    lhs_view = wide_l[:, 3:103].view(torch.float8_e4m3fn)  # odd base offset and row pitch 104
    with pytest.raises(_lib.VarkError) as ei:
        vark(lhs_view, d.rhs, d.lhs_scale, d.rhs_scale, d.group_offs, path="tcgen05")
    assert ei.value.code == _lib.ELAYOUT
    out = vark(lhs_view, d.rhs, d.lhs_scale, d.rhs_scale, d.group_offs)  # auto -> SIMT
    torch.cuda.synchronize()
    _check(p, out, label="unaligned")


def test_ragged_out_n_keeps_padding_columns():
    """OUT_N not a multiple of 8 with a padded C pitch: a TMA store would write the row up to the
    next 16-byte boundary, so the tensor-core paths refuse the layout and auto takes the CUDA-core
    path; the caller's columns past OUT_N keep their contents."""
    p = inputs.make_problem("tiny", seed=29, lens=[200, 0, 77, 300], OUT_M=96, OUT_N=124)
    d = p.to("cuda")
    wide_r = torch.zeros(d.rhs.shape[0], 128, dtype=torch.uint8, device="cuda")
    wide_r[:, :124] = d.rhs.view(torch.uint8)
    rhs = wide_r[:, :124].view(torch.float8_e5m2)  # 16-byte row pitch: only OUT_N is ragged
    big = torch.full((4, 96, 136), 7.0, dtype=torch.bfloat16, device="cuda")
    view = big[:, :, :124]
    for path in TC_PATHS:
        with pytest.raises(_lib.VarkError) as ei:
            vark(d.lhs, rhs, d.lhs_scale, d.rhs_scale, d.group_offs, path=path, out=view)
        assert ei.value.code == _lib.ELAYOUT
    vark(d.lhs, rhs, d.lhs_scale, d.rhs_scale, d.group_offs, out=view)
    torch.cuda.synchronize()
    assert bool((big[:, :, 124:] == 7.0).all())
    _check(p, view, label="ragged OUT_N")


@pytest.mark.parametrize("path", TC_PATHS)
def test_bad_offsets_reported_and_zeroed(path):
    p = inputs.make_problem("tiny", seed=23, lens=[64, 64, 64, 64], OUT_M=240, OUT_N=128)
    d = p.to("cuda")
    bad = torch.tensor([0, 64, 40, 192, 256], dtype=torch.int64, device="cuda")  # 64 -> 40
    out = torch.full((4, 240, 128), 3.0, dtype=torch.bfloat16, device="cuda")
    vark(d.lhs, d.rhs, d.lhs_scale, d.rhs_scale, bad, out=out, path=path)
    assert _lib.read_status(clear=True) & _lib.DEV_BAD_OFFS
    assert bool((out[1] == 0).all())
    past = torch.tensor([0, 64, 128, 192, 257], dtype=torch.int64, device="cuda")  # > m_total
    vark(d.lhs, d.rhs, d.lhs_scale, d.rhs_scale, past, out=out, path=path)
    assert _lib.read_status(clear=True) & _lib.DEV_BAD_OFFS
    assert bool((out[3] == 0).all())


def test_fourteen_argument_entry_point():
    """The drop-in ABI with the reference's argument packing (bench.py:370-385)."""
    p = inputs.make_problem("tiny", seed=29, lens=[500, 0, 524], OUT_M=480, OUT_N=384)
    d = p.to("cuda")
    out = torch.empty(3, 480, 384, dtype=torch.bfloat16, device="cuda")
    launch_raw(d.lhs.data_ptr(), d.rhs.data_ptr(), out.data_ptr(), d.lhs_scale.data_ptr(),
               d.rhs_scale.data_ptr(), d.group_offs.data_ptr(), 3, 480, 384, d.lhs.stride(0),
               d.rhs.stride(0), out.stride(0), out.stride(1), out.stride(2),
               torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    _check(p, out, label="14-arg")


@pytest.mark.parametrize("path", TC_PATHS)
def test_deterministic(path):
    p = inputs.make_problem("tiny", seed=31, lens=[1000, 3000, 17], OUT_M=480, OUT_N=640)
    a = _run(p, path)
    b = _run(p, path)
    assert torch.equal(a, b)


@pytest.fixture(scope="module")
def gate_up_problem():
    return inputs.make_problem("gate_up", seed=0, device="cuda")


def test_gate_up_full_size(gate_up_problem):
    """The gate_up benchmark problem at full size: every expert element by element against the
    oracle's per-element bound, the whole-output cosine, exact scale linearity, and a checksum
    identity."""
    p = gate_up_problem
    out = vark(p.lhs, p.rhs, p.lhs_scale, p.rhs_scale, p.group_offs)
    torch.cuda.synchronize()
    assert _lib.read_status(clear=True) == 0
    _check_all(p.to("cpu"), out, "gate_up")
    # Linearity: doubling a scale doubles every output exactly (power-of-two scaling).
    out2 = vark(p.lhs, p.rhs, p.lhs_scale * 2, p.rhs_scale, p.group_offs)
    torch.cuda.synchronize()
    assert torch.equal(out2.float(), out.float() * 2)
    # Checksum: 1^T C_g 1 = sL sR sum_t (sum_m L[t,m]) (sum_n R[t,n]), per group.
    sl = p.lhs.float().sum(dim=1)
    sr = p.rhs.float().sum(dim=1)
    for g in range(0, p.G, 7):
        lo, hi = int(p.offs[g]), int(p.offs[g + 1])
        expect = float((sl[lo:hi].double() * sr[lo:hi].double()).sum()) * float(p.lhs_scale) * float(p.rhs_scale)
        got = float(out[g].double().sum())
        mag = float((out[g].double().abs()).sum())
        assert abs(got - expect) <= 1e-3 * mag + 1e-6, (g, got, expect)


def _full_size_check(p):
    """Kernel over the whole problem; every expert against the oracle's per-element bound
    (empty experts exact zeros); whole-output determinism."""
    out = vark(p.lhs, p.rhs, p.lhs_scale, p.rhs_scale, p.group_offs)
    torch.cuda.synchronize()
    assert _lib.read_status(clear=True) == 0
    _check_all(p.to("cpu"), out, p.name)
    again = vark(p.lhs, p.rhs, p.lhs_scale, p.rhs_scale, p.group_offs)
    torch.cuda.synchronize()
    assert torch.equal(again, out)
    return out


@pytest.mark.parametrize("name", ["down", "skew"])
def test_baseline_configs_full_size(name):
    """The down_wgrad problem and the skewed-routing stress problem (Zipf routing, 4 empty experts, sizes not multiples
    of 128, per-expert scales) at full size."""
    p = inputs.make_problem(name, seed=0, device="cuda")
    if name == "skew":
        assert p.lhs_scale.numel() == p.G and int((p.lens == 0).sum()) == 4
    _full_size_check(p)


def test_reference_exponential_routing_full_size():
    """The reference harness's own routing (bench.py:205-212, seed 42) at the gate_up shape."""
    lens = inputs.reference_exponential_lens(32, 131072, 42)
    p = inputs.make_problem("gate_up", seed=0, device="cuda", lens=lens)
    _full_size_check(p)


def test_shard120b_on_one_gpu_and_sharded_equivalence():
    """The GPT-OSS-120B-shaped problem (G=128, M_total=1048576, 2880 x 5760) on one GPU, then the same problem
    computed as 4 expert shards (rebased offsets, token-row slices): bit-identical."""
    from ggemm_asm_b200 import sharding

    p = inputs.make_problem("shard120b", seed=0, device="cuda")
    full = _full_size_check(p)
    shards = sharding.partition(p.lens, 4)
    for sh in shards:
        loc = torch.from_numpy(sharding.local_offsets(p.offs, sh)).to("cuda")
        part = vark(p.lhs[sh.t_begin:sh.t_end], p.rhs[sh.t_begin:sh.t_end], p.lhs_scale,
                    p.rhs_scale, loc)
        torch.cuda.synchronize()
        assert torch.equal(part, full[sh.g_begin:sh.g_end]), f"shard {sh.rank} differs"


@pytest.mark.parametrize("site", ["down_wgrad", "gate_up_wgrad"])
def test_harness_wgrad_sites_full_size(site):
    """The reference harness's own correctness problem for the two wgrad sites (bench.py:594-646:
    seed-42 exponential routing, N(0,1) bf16 cast directly to fp8, scales 0.1) at full size,
    every expert against the oracle's per-element bound rather than the harness's cosine rule."""
    from ggemm_asm_b200 import sites

    _, t, _ = sites.make_site(site)
    out = vark(t["lhs"], t["rhs"], t["lhs_scale"], t["rhs_scale"], t["group_offs"])
    torch.cuda.synchronize()
    assert _lib.read_status(clear=True) == 0
    offs = t["group_offs"].cpu()
    lens = (offs[1:] - offs[:-1]).numpy()
    p = inputs.Problem(name=site, G=len(lens), M_total=int(offs[-1]), OUT_M=t["lhs"].shape[1],
                       OUT_N=t["rhs"].shape[1], lens=lens, offs=offs.numpy(),
                       lhs=t["lhs"].cpu(), rhs=t["rhs"].cpu(), lhs_scale=t["lhs_scale"].cpu(),
                       rhs_scale=t["rhs_scale"].cpu(), group_offs=offs)
    _check_all(p, out, site)
