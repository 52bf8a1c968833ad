"""The six MoE call sites of the ggemm-asm harness, as a command line over this library's kernels.

    python -m ggemm_asm_b200.sites --correctness [--site all|all_fwd|all_wgrad|<site>]
    python -m ggemm_asm_b200.sites --bench [--site ...] [--warmup 20] [--iters 100]

Mirrors the harness's correctness and benchmark modes (ggemm-asm bench.py:592-640 and
bench.py:690-): the same sites and shapes (bench.py:147-200), the same inputs (N(0,1) bf16 cast
directly to fp8, scales 0.1, bench.py:221-223,257-258, exponential routing, bench.py:205-212),
the same pass rule (cosine >= 0.999 against a reference, bench.py:636-638) and TFLOPS =
2*M*N*K / time (2*M*OUT_M*OUT_N for the wgrad sites). The harness's reference is Primus-Turbo's
Triton kernels, which are absent here; the check uses an fp32 torch computation of the same
products on the device, and the benchmark times torch._scaled_mm per expert (cuBLAS) beside ours.
"""
from __future__ import annotations

import argparse
import sys

import torch

E, M_TOTAL, F_DIM, F2_DIM = 32, 131072, 2880, 5760
E4M3, E5M2 = torch.float8_e4m3fn, torch.float8_e5m2

# name: (kind, A dtype, B dtype, M-or-OUT_M dims)
SITES = {
    "gate_up_fwd": ("persistent", E4M3, E4M3, dict(K=F_DIM, N=F2_DIM)),    # x @ W_gu
    "down_fwd": ("persistent", E4M3, E4M3, dict(K=F_DIM, N=F_DIM)),        # swiglu @ W_d
    "down_dgrad": ("persistent", E5M2, E4M3, dict(K=F_DIM, N=F_DIM)),      # dy_d @ W_d^T
    "gate_up_dgrad": ("persistent", E5M2, E4M3, dict(K=F2_DIM, N=F_DIM)),  # dy_gu @ W_gu^T
    "down_wgrad": ("variable_k", E4M3, E5M2, dict(OUT_M=F_DIM, OUT_N=F_DIM)),    # swiglu^T dy_d
    "gate_up_wgrad": ("variable_k", E4M3, E5M2, dict(OUT_M=F_DIM, OUT_N=F2_DIM)),  # x^T dy_gu
}
GROUPS = {"all": list(SITES), "all_fwd": [s for s in SITES if SITES[s][0] == "persistent"],
          "all_wgrad": [s for s in SITES if SITES[s][0] == "variable_k"]}


def _fp8(shape, dtype, gen, device):
    return torch.randn(shape, generator=gen, device=device, dtype=torch.float32).to(
        torch.bfloat16).to(dtype)


def make_site(name: str, M: int = M_TOTAL, device="cuda", seed: int = 42):
    from . import inputs

    kind, adt, bdt, dims = SITES[name]
    lens = inputs.reference_exponential_lens(E, M, seed=seed)
    offs = torch.from_numpy(inputs.offsets_from_lens(lens)).to(device)
    gen = torch.Generator(device=device).manual_seed(seed)
    s = torch.tensor([0.1], dtype=torch.float32, device=device)
    if kind == "persistent":
        a = _fp8((M, dims["K"]), adt, gen, device)
        b = _fp8((E, dims["N"], dims["K"]), bdt, gen, device)
        return kind, dict(a=a, b=b, a_scale=s, b_scale=s.clone(), group_offs=offs), dims
    lhs = _fp8((M, dims["OUT_M"]), adt, gen, device)
    rhs = _fp8((M, dims["OUT_N"]), bdt, gen, device)
    return kind, dict(lhs=lhs, rhs=rhs, lhs_scale=s, rhs_scale=s.clone(), group_offs=offs), dims


def run_ours(kind, t):
    from .grouped_fwd import grouped_gemm_fp8_tensorwise
    from .grouped_gemm import grouped_gemm_fp8_tensorwise_variable_k

    if kind == "persistent":
        return grouped_gemm_fp8_tensorwise(t["a"], t["b"], t["a_scale"], t["b_scale"],
                                           t["group_offs"], trans_b=True)
    return grouped_gemm_fp8_tensorwise_variable_k(t["lhs"], t["rhs"], t["lhs_scale"],
                                                  t["rhs_scale"], t["group_offs"])


def reference_fp32(kind, t):
    """fp32 torch products on the device (the check the harness makes against Triton)."""
    offs = t["group_offs"].tolist()
    if kind == "persistent":
        a, b = t["a"], t["b"]
        out = torch.zeros(a.shape[0], b.shape[1], device=a.device)
        s = float(t["a_scale"]) * float(t["b_scale"])
        for g in range(b.shape[0]):
            if offs[g + 1] > offs[g]:
                out[offs[g]:offs[g + 1]] = (a[offs[g]:offs[g + 1]].float() @ b[g].float().T) * s
        return out
    lhs, rhs = t["lhs"], t["rhs"]
    out = torch.zeros(len(offs) - 1, lhs.shape[1], rhs.shape[1], device=lhs.device)
    s = float(t["lhs_scale"]) * float(t["rhs_scale"])
    for g in range(len(offs) - 1):
        if offs[g + 1] > offs[g]:
            out[g] = (lhs[offs[g]:offs[g + 1]].float().T @ rhs[offs[g]:offs[g + 1]].float()) * s
    return out


def run_cublas(kind, t):
    """torch._scaled_mm per expert (cuBLAS) on the same fp8 data."""
    offs = t["group_offs"].tolist()
    if kind == "persistent":
        a, b = t["a"], t["b"]
        for g in range(b.shape[0]):
            if offs[g + 1] > offs[g]:
                torch._scaled_mm(a[offs[g]:offs[g + 1]], b[g].t(), scale_a=t["a_scale"],
                                 scale_b=t["b_scale"], out_dtype=torch.bfloat16)
        return
    # wgrad: lhs_g^T (col-major view of token-major data) x rhs_g; cuBLAS fp8 wants A row-major
    # and B column-major, so the token-major operands are transposed into place per expert.
    lhs, rhs = t["lhs"], t["rhs"]
    for g in range(len(offs) - 1):
        if offs[g + 1] > offs[g]:
            lt = lhs[offs[g]:offs[g + 1]].t().contiguous()
            rt = rhs[offs[g]:offs[g + 1]].t().contiguous()
            torch._scaled_mm(lt, rt.t(), scale_a=t["lhs_scale"], scale_b=t["rhs_scale"],
                             out_dtype=torch.bfloat16)


def flops(kind, t, dims):
    M = t["a"].shape[0] if kind == "persistent" else t["lhs"].shape[0]
    if kind == "persistent":
        return 2.0 * M * dims["N"] * dims["K"]
    return 2.0 * M * dims["OUT_M"] * dims["OUT_N"]


def time_ms(fn, warmup: int, iters: int) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters


def correctness(names, M=M_TOTAL) -> bool:
    print("=" * 80)
    print("CORRECTNESS - ggemm_asm_b200 kernels vs fp32 torch reference (pass: cos >= 0.999)")
    print("=" * 80)
    ok = True
    for name in names:
        kind, t, dims = make_site(name, M)
        got = run_ours(kind, t).float()
        ref = reference_fp32(kind, t)
        cos = float(torch.nn.functional.cosine_similarity(got.flatten(), ref.flatten(), dim=0))
        diff = float((got - ref).abs().max())
        passed = cos >= 0.999
        ok &= passed
        print(f"  [{'PASS' if passed else 'FAIL'}] {name:14s} cos={cos:.6f}  max_diff={diff:.6f}")
        del t, got, ref
        torch.cuda.empty_cache()
    return ok


def benchmark(names, warmup=20, iters=100, cublas=True, M=M_TOTAL):
    print("=" * 80)
    print(f"BENCHMARK - {torch.cuda.get_device_name(0)}  E={E} M_total={M} F={F_DIM} 2F={F2_DIM}")
    print(f"Warmup: {warmup}, Iters: {iters}")
    print("=" * 80)
    print(f"  {'site':14s} {'ours ms':>9s} {'TFLOPS':>8s} {'cuBLAS ms':>10s} {'TFLOPS':>8s} {'x':>6s}")
    rows = []
    for name in names:
        kind, t, dims = make_site(name, M)
        f = flops(kind, t, dims)
        ms = time_ms(lambda: run_ours(kind, t), warmup, iters)
        cms = float("nan")
        if cublas:
            try:
                cms = time_ms(lambda: run_cublas(kind, t), max(2, warmup // 4), max(3, iters // 10))
            except RuntimeError:  # e.g. an expert size cuBLAS fp8 does not accept
                pass
        rows.append((name, ms, f / ms / 1e9, cms, f / cms / 1e9))
        print(f"  {name:14s} {ms:9.3f} {f / ms / 1e9:8.1f} {cms:10.3f} {f / cms / 1e9:8.1f} "
              f"{cms / ms:6.2f}")
        del t
        torch.cuda.empty_cache()
    return rows


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--site", default="all", help="site name, all, all_fwd or all_wgrad")
    ap.add_argument("--correctness", action="store_true")
    ap.add_argument("--bench", action="store_true")
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--iters", type=int, default=100)
    ap.add_argument("--no-cublas", action="store_true")
    ap.add_argument("--tokens", type=int, default=M_TOTAL, help="M_total (default 131072)")
    args = ap.parse_args(argv)
    names = GROUPS.get(args.site, [args.site])
    unknown = [n for n in names if n not in SITES]
    if unknown:
        ap.error(f"unknown site(s) {unknown}; choose from {sorted(SITES) + sorted(GROUPS)}")
    if not (args.correctness or args.bench):
        args.correctness = args.bench = True
    ok = True
    if args.correctness:
        ok = correctness(names, args.tokens)
    if args.bench:
        benchmark(names, args.warmup, args.iters, not args.no_cublas, args.tokens)
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
