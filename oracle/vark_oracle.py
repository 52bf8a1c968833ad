"""TEST INFRASTRUCTURE ONLY - the checker for the variable-K grouped FP8 wgrad, never the product.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference legs import this
module. The product path (ggemm_asm_b200) never does.

Reference semantics restated (ggemm-asm):
  * README.md:5,45-48 and bench.py:182-193: per expert g, dW_g = lhs_g^T @ rhs_g with
    lhs = x (e4m3) and rhs = dy (e5m2), token ranges given by group_offs (bench.py:215-218);
  * bench.py:266-268: tensorwise fp32 scales, out [G, OUT_M, OUT_N] bf16;
  * the Triton kernel it is checked against (primus_turbo, not vendored) dequantises with the
    scales and accumulates in fp32.

The producer step (per-expert amax scaling and fp8 quantisation of x and dy) is restated by
``quantize_fp8_ref``; the reference harness does this on the host (bench.py:221-223, 266-267).

Three restatements of the wgrad live here:
  ``wgrad_torch``      torch CPU fp32: dequantise each group's slice (fp8 -> fp32, x scale),
                       fp32 matmul, round to bf16 (RNE). This is the parity oracle and the timed
                       CPU baseline.
  ``wgrad_c_f64``      the plain-C restatement (oracle/vark_oracle_c.c): bit-field fp8 decode,
                       exact products, double accumulation, scale last. Pins ``wgrad_torch``.
  ``fp8_decode_table`` numpy bit-field decoders for all 256 codes of each format (OCP FP8).

Parity is pinned against: the OCP FP8 code tables (all 256 codes, cross-checked with torch's
casts), the reference launcher's closed-form workload (launcher.cpp:97-112), the reference
harness's own group-size generator (bench.py:205-212, imported to make tests/golden fixtures)
and the C restatement. The reference kernel itself cannot run here (AMD gfx950 binary; its
Triton oracle primus_turbo is absent), so end-to-end parity against the reference's own
outputs is not available.
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
C_LIB = HERE / "_build" / "libvark_oracle.so"


# ----------------------------------------------------------------------------------------------
# fp8 code tables (OCP 8-bit floating point specification)
# ----------------------------------------------------------------------------------------------
def fp8_decode_table(fmt: str) -> np.ndarray:
    """float64 value of each of the 256 codes of 'e4m3fn' or 'e5m2' (NaN/Inf as IEEE)."""
    codes = np.arange(256, dtype=np.int64)
    sign = np.where(codes >> 7, -1.0, 1.0)
    if fmt == "e4m3fn":
        exp, man = (codes >> 3) & 0xF, codes & 0x7
        mag = np.where(exp == 0, man / 8.0 * 2.0 ** -6, (1 + man / 8.0) * 2.0 ** (exp - 7.0))
        mag = np.where((exp == 0xF) & (man == 0x7), np.nan, mag)
    elif fmt == "e5m2":
        exp, man = (codes >> 2) & 0x1F, codes & 0x3
        mag = np.where(exp == 0, man / 4.0 * 2.0 ** -14, (1 + man / 4.0) * 2.0 ** (exp - 15.0))
        mag = np.where(exp == 0x1F, np.where(man == 0, np.inf, np.nan), mag)
    else:
        raise ValueError(fmt)
    return sign * mag


def bf16_ulp(x: torch.Tensor) -> torch.Tensor:
    """Spacing of bf16 numbers at |x| (fp32 tensor in, fp32 out); 2^-133 floor near zero."""
    ax = x.abs().float().clamp_min(2.0 ** -126)
    e = torch.floor(torch.log2(ax))
    return torch.pow(2.0, e - 7.0)


# ----------------------------------------------------------------------------------------------
# torch CPU fp32 oracle
# ----------------------------------------------------------------------------------------------
def _scale_of(scale: torch.Tensor, g: int) -> torch.Tensor:
    s = scale.reshape(-1)
    return s[0] if s.numel() == 1 else s[g]


def wgrad_torch_f32(lhs, rhs, lhs_scale, rhs_scale, group_offs, groups=None) -> torch.Tensor:
    """fp32 [G, OUT_M, OUT_N] (or [len(groups), ...]) before the bf16 rounding, on the CPU."""
    lhs, rhs = lhs.cpu(), rhs.cpu()
    ls, rs = lhs_scale.cpu().float(), rhs_scale.cpu().float()
    offs = group_offs.cpu().tolist()
    G = len(offs) - 1
    gs = list(range(G)) if groups is None else list(groups)
    out = torch.zeros(len(gs), lhs.shape[1], rhs.shape[1], dtype=torch.float32)
    for i, g in enumerate(gs):
        lo, hi = int(offs[g]), int(offs[g + 1])
        if hi <= lo:
            continue
        a = lhs[lo:hi].float() * _scale_of(ls, g)
        b = rhs[lo:hi].float() * _scale_of(rs, g)
        torch.matmul(a.t(), b, out=out[i])
    return out


def wgrad_torch(lhs, rhs, lhs_scale, rhs_scale, group_offs, groups=None) -> torch.Tensor:
    """The oracle: bf16 [G, OUT_M, OUT_N] (bench.py:268 output contract), computed on the CPU."""
    return wgrad_torch_f32(lhs, rhs, lhs_scale, rhs_scale, group_offs, groups).to(torch.bfloat16)


def abs_product_sum(lhs, rhs, lhs_scale, rhs_scale, group_offs, groups=None) -> torch.Tensor:
    """sL*sR * |LHS_g|^T |RHS_g| (fp32, CPU): the magnitude that bounds reassociation error."""
    return wgrad_torch_f32(_abs_fp8(lhs), _abs_fp8(rhs), lhs_scale.abs(), rhs_scale.abs(),
                           group_offs, groups)


def _abs_fp8(t: torch.Tensor) -> torch.Tensor:
    # Clearing the sign bit of an fp8 code gives |value| exactly.
    return (t.cpu().view(torch.uint8) & 0x7F).view(t.dtype)


def tolerance(lhs, rhs, lhs_scale, rhs_scale, group_offs, ref_f32: torch.Tensor,
              groups=None, ulps: float = 1.0, gamma_factor: float = 2.0) -> torch.Tensor:
    """Per-element bound  ulps * ulp_bf16(|ref|) + gamma_factor * K_g * 2^-24 * sL*sR*|L_g|^T|R_g|.

    The first term allows the two fp32 sums to round to neighbouring bf16 values; the second
    is the fp32 reassociation bound (each of the oracle and the kernel sums K_g products in a
    different order; each ordering is within K_g * 2^-24 * sum|p| of the exact sum)."""
    offs = group_offs.cpu().tolist()
    G = len(offs) - 1
    gs = list(range(G)) if groups is None else list(groups)
    k = torch.tensor([max(int(offs[g + 1]) - int(offs[g]), 0) for g in gs], dtype=torch.float32)
    mag = abs_product_sum(lhs, rhs, lhs_scale, rhs_scale, group_offs, groups)
    return ulps * bf16_ulp(ref_f32) + gamma_factor * (k * 2.0 ** -24)[:, None, None] * mag


def cosine(a: torch.Tensor, b: torch.Tensor) -> float:
    """Cosine similarity of two tensors (float64), the reference's check (bench.py:641-645)."""
    a = a.double().flatten()
    b = b.double().flatten()
    na, nb = a.norm().item(), b.norm().item()
    if na == 0.0 and nb == 0.0:
        return 1.0
    return float(torch.dot(a, b).item() / (na * nb + 1e-300))


# ----------------------------------------------------------------------------------------------
# plain-C restatement
# ----------------------------------------------------------------------------------------------
_c = None


def build_c(force: bool = False) -> Path:
    if force or not C_LIB.exists() or C_LIB.stat().st_mtime < (HERE / "vark_oracle_c.c").stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return C_LIB


def c_lib():
    global _c
    if _c is None:
        build_c()
        lib = ctypes.CDLL(str(C_LIB))
        lib.vark_oracle_e4m3fn_to_f64.restype = ctypes.c_double
        lib.vark_oracle_e4m3fn_to_f64.argtypes = [ctypes.c_uint8]
        lib.vark_oracle_e5m2_to_f64.restype = ctypes.c_double
        lib.vark_oracle_e5m2_to_f64.argtypes = [ctypes.c_uint8]
        lib.vark_oracle_f32_to_bf16_rne.restype = ctypes.c_uint16
        lib.vark_oracle_f32_to_bf16_rne.argtypes = [ctypes.c_float]
        vp = ctypes.c_void_p
        lib.vark_oracle_wgrad_f64.restype = ctypes.c_int
        lib.vark_oracle_wgrad_f64.argtypes = [vp, vp, vp, vp, ctypes.c_int, vp, ctypes.c_int,
                                              ctypes.c_int, ctypes.c_int, ctypes.c_int64,
                                              ctypes.c_int64, vp]
        lib.vark_oracle_markstein_mismatches.restype = ctypes.c_long
        lib.vark_oracle_markstein_mismatches.argtypes = [ctypes.c_uint32, ctypes.c_uint32]
        _c = lib
    return _c


def markstein_mismatches(lo: int = 0, hi: int = 1 << 23) -> int:
    """Pairs (bf16 significand a, fp32 divisor b in [1, 2) with bit offsets [lo, hi)) for which
    the quantiser's division-free quotient differs from IEEE division (plain-C exhaustive check,
    oracle/vark_oracle_c.c)."""
    return int(c_lib().vark_oracle_markstein_mismatches(lo, hi))


def wgrad_c_f64(lhs, rhs, lhs_scale, rhs_scale, group_offs) -> np.ndarray:
    """float64 [G, OUT_M, OUT_N] from the plain-C restatement (small problems only)."""
    lhs_u8 = np.ascontiguousarray(lhs.cpu().view(torch.uint8).numpy())
    rhs_u8 = np.ascontiguousarray(rhs.cpu().view(torch.uint8).numpy())
    ls = np.ascontiguousarray(lhs_scale.cpu().float().reshape(-1).numpy())
    rs = np.ascontiguousarray(rhs_scale.cpu().float().reshape(-1).numpy())
    offs = np.ascontiguousarray(group_offs.cpu().numpy().astype(np.int64))
    G = offs.size - 1
    out = np.zeros((G, lhs_u8.shape[1], rhs_u8.shape[1]), dtype=np.float64)
    rc = c_lib().vark_oracle_wgrad_f64(
        lhs_u8.ctypes.data, rhs_u8.ctypes.data, ls.ctypes.data, rs.ctypes.data,
        0 if ls.size == 1 else 1, offs.ctypes.data, G, lhs_u8.shape[1], rhs_u8.shape[1],
        lhs_u8.shape[1], rhs_u8.shape[1], out.ctypes.data)
    if rc != 0:
        raise ValueError("group_offs is not monotone / non-negative")
    return out


def f32_to_bf16_bits_c(x: float) -> int:
    return int(c_lib().vark_oracle_f32_to_bf16_rne(float(x)))


def closed_form_launcher_value(K: int, scale: float = 0.1) -> float:
    """Every output of the reference launcher's workload (launcher.cpp:97-112) for a group of K
    tokens: bf16(fp32(0.1) * fp32(0.1) * K * 1.0 * 0.5) with e4m3fn 0x38 = 1.0, e5m2 0x38 = 0.5."""
    s = np.float32(scale) * np.float32(scale)
    acc = np.float32(K * 0.5)
    v = np.float32(acc * s)
    return float(torch.tensor(float(v), dtype=torch.float32).to(torch.bfloat16).float())


FP8_FORMATS = {"e4m3": (torch.float8_e4m3fn, 448.0), "e5m2": (torch.float8_e5m2, 57344.0)}


def quantize_fp8_ref(x: torch.Tensor, group_offs, fmt: str, per_group: bool = True):
    """CPU restatement of the producer step: per unit (expert, or all rows), s = amax|x| / FMAX
    in fp32 (1.0 for an empty unit or amax 0; NaN when the unit holds a NaN), q = fp8(x / s)
    with the division in fp32, clamped to +-FMAX, cast round-to-nearest-even.

    Follows the operand construction of the wgrad configurations (amax scaling of N(0,1) bf16,
    the per-expert variant from the expert's own token slice) and the fp8 cast of the reference
    harness (bench.py:221-223). Returns (q as uint8 codes [rows, F], rows outside every unit 0;
    scales fp32 [units]).
    """
    dtype, fmax = FP8_FORMATS[fmt]
    offs = [int(v) for v in (group_offs.tolist() if hasattr(group_offs, "tolist") else group_offs)]
    units = list(zip(offs[:-1], offs[1:])) if per_group else [(offs[0], offs[-1])]
    xf = x.float()
    q = torch.zeros(x.shape, dtype=torch.uint8)
    scales = torch.ones(len(units), dtype=torch.float32)
    fmax_t = torch.tensor(fmax, dtype=torch.float32)
    for u, (lo, hi) in enumerate(units):
        if hi <= lo:
            continue
        amax = xf[lo:hi].abs().amax()
        s = torch.tensor(1.0) if bool(amax == 0) else amax / fmax_t
        scales[u] = s
        q[lo:hi] = (xf[lo:hi] / s).clamp(-fmax, fmax).to(dtype).view(torch.uint8)
    return q, scales


def grouped_fwd_f32(a: torch.Tensor, b: torch.Tensor, a_scale, b_scale, group_offs,
                    rows=None, trans_b: bool = True) -> torch.Tensor:
    """CPU restatement of the fixed-K grouped GEMM (the harness's persistent sites, bench.py:
    154-181, checked there against Primus-Turbo's grouped_gemm_fp8_tensorwise_triton_kernel,
    bench.py:260): per expert g, out[off_g:off_{g+1}] = sA_g * sB_g * a_g @ B_g, fp8 decoded to
    fp32, fp32 matmul. b is [G, N, K] (trans_b: B_g = b[g]^T) or [G, K, N] (B_g = b[g]); the
    scales hold 1 or G values. Returns fp32 [M, N]; `rows` (optional index tensor) restricts the
    output to those token rows (returned in that order)."""
    offs = [int(v) for v in (group_offs.tolist() if hasattr(group_offs, "tolist") else group_offs)]
    if not trans_b:
        b = b.transpose(1, 2)
    G, N, _ = b.shape
    sa = a_scale.reshape(-1).float()
    sb = b_scale.reshape(-1).float()
    which = torch.arange(a.shape[0]) if rows is None else torch.as_tensor(rows)
    out = torch.zeros(which.numel(), N, dtype=torch.float32)
    starts = torch.tensor(offs[:-1])
    ends = torch.tensor(offs[1:])
    gid = torch.searchsorted(torch.tensor(offs[1:]), which, right=True)
    for g in range(G):
        sel = ((gid == g) & (which >= starts[g]) & (which < ends[g])).nonzero().flatten()
        if sel.numel() == 0:
            continue
        ag = a[which[sel]].float()
        bg = b[g].float()
        s = float(sa[g] if sa.numel() > 1 else sa[0]) * float(sb[g] if sb.numel() > 1 else sb[0])
        out[sel] = (ag @ bg.T) * s
    return out


def grouped_fwd_tolerance(a, b, a_scale, b_scale, group_offs, ref: torch.Tensor, rows=None,
                          trans_b: bool = True):
    """|C - ref| bound: one bf16 ulp of |ref| plus fp32 reassociation over K terms,
    K * 2^-24 * sA * sB * (|a| @ |B|) (the same form as the wgrad's)."""
    K = a.shape[1]
    absd = grouped_fwd_f32(_abs_fp8(a), _abs_fp8(b), a_scale.abs(), b_scale.abs(), group_offs,
                           rows, trans_b)
    return bf16_ulp(ref.abs()) + K * 2.0 ** -24 * absd
