"""CPU tests of the C ABI boundary: the library loads, exports every declared symbol, and
rejects bad arguments before touching a device."""
import ctypes
import re
from pathlib import Path

import pytest
import torch

from ggemm_asm_b200 import _lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "ggemm_vark.h"


def declared_functions():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"GGEMM_VARK_API\s+[\w\s\*]*?\b(ggemm_vark_\w+)\s*\(", text)))


def test_header_declares_the_abi():
    names = declared_functions()
    assert "ggemm_vark_fp8_wgrad" in names and "ggemm_vark_fp8_wgrad_ex" in names
    assert set(names) == set(_lib.SIGNATURES), "ctypes table and header disagree"


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    for name in declared_functions():
        assert hasattr(lib, name), name


def test_codes_match_header():
    text = HEADER.read_text()
    for name in ["OK", "EINVAL_PTR", "EINVAL_SHAPE", "EINVAL_STRIDE", "EINVAL_ARG", "ENO_DEVICE",
                 "ECUDA", "ELAYOUT", "ETOO_LARGE"]:
        m = re.search(rf"#define GGEMM_VARK_{name}\s+(\d+)", text)
        assert m and int(m.group(1)) == getattr(_lib, name), name
    for name in ["DEV_BAD_OFFS", "DEV_TIMEOUT"]:
        m = re.search(rf"#define GGEMM_VARK_{name}\s+(0x[0-9a-fA-F]+)u", text)
        assert m and int(m.group(1), 16) == getattr(_lib, name), name
    for name in ["PATH_AUTO", "PATH_TCGEN05", "PATH_SIMT", "PATH_TCGEN05_1SM"]:
        m = re.search(rf"#define GGEMM_VARK_{name}\s+(\d+)", text)
        assert m and int(m.group(1)) == getattr(_lib, name), name


def test_strerror_and_version():
    assert _lib.strerror(0) == "success"
    assert "NULL" in _lib.strerror(_lib.EINVAL_PTR)
    assert _lib.strerror(999) == "unknown error code"
    assert _lib.lib().ggemm_vark_version() == 0x000100


P = 1 << 20  # fake, 16-byte aligned "device" address: never dereferenced by these tests


def call14(**kw):
    a = dict(lhs=P, rhs=P, c=P, ls=P, rs=P, offs=P, G=4, M=64, N=128, slm=64, srm=128,
             scg=64 * 128, scm=128, scn=1)
    a.update(kw)
    return _lib.lib().ggemm_vark_fp8_wgrad(a["lhs"], a["rhs"], a["c"], a["ls"], a["rs"],
                                           a["offs"], a["G"], a["M"], a["N"], a["slm"],
                                           a["srm"], a["scg"], a["scm"], a["scn"], None)


def call_ex(**kw):
    a = dict(m_total=1024, scale_stride=0, path=0, status=None)
    a.update(kw)
    return _lib.lib().ggemm_vark_fp8_wgrad_ex(P, P, P, P, P, P, 4, 64, 128, 64, 128, 64 * 128,
                                              128, 1, a["m_total"], a["scale_stride"],
                                              a["path"], a["status"], 0, None)


@pytest.mark.parametrize("arg", ["lhs", "rhs", "c", "ls", "rs", "offs"])
def test_null_pointers_rejected(arg):
    assert call14(**{arg: None}) == _lib.EINVAL_PTR


@pytest.mark.parametrize("kw,code", [
    (dict(G=-1), _lib.EINVAL_SHAPE), (dict(M=0), _lib.EINVAL_SHAPE), (dict(N=-5), _lib.EINVAL_SHAPE),
    (dict(slm=63), _lib.EINVAL_STRIDE), (dict(srm=100), _lib.EINVAL_STRIDE),
    (dict(scn=0), _lib.EINVAL_STRIDE), (dict(scm=-1), _lib.EINVAL_STRIDE),
    (dict(scg=0), _lib.EINVAL_STRIDE),
])
def test_bad_shapes_and_strides_rejected(kw, code):
    assert call14(**kw) == code


@pytest.mark.parametrize("kw", [dict(scale_stride=2), dict(scale_stride=-1), dict(path=4),
                                dict(path=-1), dict(m_total=-2), dict(status=P + 8)])
def test_bad_extended_args_rejected(kw):
    assert call_ex(**kw) == _lib.EINVAL_ARG


def test_zero_groups_is_a_no_op():
    assert call14(G=0) == _lib.OK


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-device answer")
def test_valid_call_without_device_reports_no_device():
    assert call14() == _lib.ENO_DEVICE


@pytest.mark.parametrize("kw,expect", [
    (dict(), 1),
    (dict(lhs=P + 1), 0), (dict(c=P + 8), 0), (dict(slm=72), 0), (dict(srm=136), 0), (dict(srm=144), 1),
    (dict(scn=2), 0), (dict(scm=132), 0), (dict(scm=136), 1), (dict(scg=64 * 128 + 4), 0),
    # a TMA store writes C rows in 16-byte pieces: OUT_N must be a multiple of 8 elements
    (dict(N=124), 0), (dict(N=120), 1), (dict(N=4), 0),
])
def test_tensor_core_layout_rules(kw, expect):
    a = dict(lhs=P, rhs=P, c=P, M=64, N=128, slm=64, srm=128, scg=64 * 128, scm=128, scn=1)
    a.update(kw)
    got = _lib.lib().ggemm_vark_tc_supported(a["lhs"], a["rhs"], a["c"], a["M"], a["N"], a["slm"],
                                             a["srm"], a["scg"], a["scm"], a["scn"])
    assert got == expect


def test_torch_api_validates_before_launch():
    from ggemm_asm_b200 import grouped_gemm_fp8_tensorwise_variable_k as vark

    lhs = torch.zeros(8, 16, dtype=torch.float8_e4m3fn)
    rhs = torch.zeros(8, 16, dtype=torch.float8_e5m2)
    s = torch.ones(1)
    offs = torch.tensor([0, 8])
    with pytest.raises(ValueError, match="CUDA"):
        vark(lhs, rhs, s, s, offs)
    with pytest.raises(TypeError):
        vark(lhs.view(torch.float8_e5m2), rhs, s, s, offs)
    with pytest.raises(ValueError, match="token counts"):
        vark(lhs, rhs[:4], s, s, offs)
    with pytest.raises(ValueError, match="int64"):
        vark(lhs, rhs, s, s, offs.int())
    with pytest.raises(ValueError, match="G=1"):
        vark(lhs, rhs, torch.ones(3), torch.ones(3), offs)


def test_ctypes_signatures_are_complete():
    for name, (res, args) in _lib.SIGNATURES.items():
        fn = getattr(_lib.lib(), name)
        assert fn.restype == res and list(fn.argtypes) == args
    assert _lib.SIGNATURES["ggemm_vark_fp8_wgrad"][1].count(ctypes.c_int32) == 8


def call_noalloc(**kw):
    a = dict(lhs=P, rhs=P, c=P, ls=P, rs=P, offs=P, G=4, M=64, N=128, slm=64, srm=128,
             scg=64 * 128, scm=128, scn=1, m_total=1024, scale_stride=0, status=None)
    a.update(kw)
    return _lib.lib().ggemm_vark_fp8_wgrad_noalloc(
        a["lhs"], a["rhs"], a["c"], a["ls"], a["rs"], a["offs"], a["G"], a["M"], a["N"],
        a["slm"], a["srm"], a["scg"], a["scm"], a["scn"], a["m_total"], a["scale_stride"],
        a["status"], None)


@pytest.mark.parametrize("kw,code", [
    (dict(lhs=None), _lib.EINVAL_PTR), (dict(offs=None), _lib.EINVAL_PTR),
    (dict(G=-1), _lib.EINVAL_SHAPE), (dict(slm=32), _lib.EINVAL_STRIDE),
    (dict(scale_stride=3), _lib.EINVAL_ARG), (dict(status=P + 4), _lib.EINVAL_ARG),
    (dict(slm=72), _lib.ELAYOUT), (dict(c=P + 2), _lib.ELAYOUT), (dict(scn=2), _lib.ELAYOUT),
    (dict(G=0), _lib.OK),
])
def test_noalloc_argument_checks(kw, code):
    assert call_noalloc(**kw) == code


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-device answer")
def test_noalloc_without_device():
    assert call_noalloc() == _lib.ENO_DEVICE
