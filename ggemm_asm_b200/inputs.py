"""Seeded synthetic problems for the variable-K grouped FP8 wgrad.

Shapes and value distributions follow the reference's call sites (ggemm-asm bench.py:146-223,
launcher.cpp:64-112) and the five benchmark configurations of this project:

  tiny      G=4, M_total=1024, OUT_M=64, OUT_N=128, group sizes [256, 0, 512, 256]
  gate_up   G=32, M_total=131072, 2880 x 5760, multinomial(uniform) routing  (GPT-OSS-20B)
  down      as gate_up with OUT_N=2880
  skew      gate_up shape, Zipf(1.2) routing, 4 empty experts, no size a multiple of 128,
            per-expert scales
  shard120b G=128, M_total=1048576, 2880 x 5760, multinomial routing (GPT-OSS-120B)

plus the reference's own schemes: ``reference_exponential_lens`` (bench.py:205-212, seed 42)
and ``launcher_problem`` (launcher.cpp:97-112: uniform split, every fp8 byte 0x38,
scales 0.1). No public dataset is involved; all data is generated here.

Values: N(0,1) drawn in fp32, rounded to bf16 (the reference draws bf16 randn,
bench.py:221-223), then quantized with an amax scale (e4m3: amax/448, e5m2: amax/57344),
per tensor or per group. Generation is chunked by absolute token row with a per-chunk seed, so
any row range can be produced on any device without materialising the rest.
"""
from __future__ import annotations

import dataclasses

import numpy as np
import torch

E4M3_MAX = 448.0
E5M2_MAX = 57344.0
LHS_DTYPE = torch.float8_e4m3fn
RHS_DTYPE = torch.float8_e5m2
CHUNK_ROWS = 8192

CONFIGS = {
    "tiny": dict(G=4, M_total=1024, OUT_M=64, OUT_N=128, routing="fixed",
                 lens=[256, 0, 512, 256], scales="tensor"),
    "gate_up": dict(G=32, M_total=131072, OUT_M=2880, OUT_N=5760, routing="multinomial",
                    scales="tensor"),
    "down": dict(G=32, M_total=131072, OUT_M=2880, OUT_N=2880, routing="multinomial",
                 scales="tensor"),
    "skew": dict(G=32, M_total=131072, OUT_M=2880, OUT_N=5760, routing="zipf",
                 scales="group"),
    "shard120b": dict(G=128, M_total=1048576, OUT_M=2880, OUT_N=5760, routing="multinomial",
                      scales="tensor"),
}


# ----------------------------------------------------------------------------------------------
# Group sizes
# ----------------------------------------------------------------------------------------------
def multinomial_lens(G: int, M_total: int, seed: int) -> np.ndarray:
    """Token counts from a seeded multinomial(M_total, uniform over G experts)."""
    rng = np.random.default_rng(seed)
    return rng.multinomial(M_total, [1.0 / G] * G).astype(np.int64)


def zipf_lens(G: int, M_total: int, seed: int, s: float = 1.2, n_empty: int = 4,
              align: int = 128) -> np.ndarray:
    """Zipf(s) allocation over G - n_empty experts (seeded rank order), n_empty experts forced
    empty at seeded positions, and no non-empty size a multiple of `align`."""
    rng = np.random.default_rng(seed)
    live = G - n_empty
    ranks = rng.permutation(live) + 1
    w = ranks.astype(np.float64) ** (-s)
    w /= w.sum()
    sizes = np.maximum(np.floor(w * M_total).astype(np.int64), 1)
    sizes[np.argmax(sizes)] += M_total - sizes.sum()
    for _ in range(10 * live):
        bad = np.nonzero(sizes % align == 0)[0]
        if bad.size == 0:
            break
        i = int(bad[0])
        j = int(np.argmax(sizes)) if int(np.argmax(sizes)) != i else (i + 1) % live
        sizes[i] += 1
        sizes[j] -= 1
    assert sizes.sum() == M_total and (sizes > 0).all() and (sizes % align != 0).all()
    empty = np.sort(rng.choice(G, size=n_empty, replace=False))
    lens = np.zeros(G, dtype=np.int64)
    lens[np.setdiff1d(np.arange(G), empty)] = sizes
    return lens


def reference_exponential_lens(G: int, M_total: int, seed: int = 42) -> np.ndarray:
    """The reference harness's group sizes (bench.py:205-212): seeded Exp(1) draws on the CPU
    generator, normalised to M_total, truncated, remainder given to the last group."""
    gen = torch.Generator().manual_seed(seed)
    raw = torch.empty(G).exponential_(generator=gen)
    raw = raw / raw.sum() * M_total
    lens = raw.long()
    lens[-1] = M_total - lens[:-1].sum()
    assert int(lens.sum()) == M_total and bool((lens > 0).all())
    return lens.numpy().astype(np.int64)


def uniform_split_lens(G: int, M_total: int) -> np.ndarray:
    """launcher.cpp:99-102: offs[i] = M_total * i / G (integer division)."""
    offs = np.array([(M_total * i) // G for i in range(G + 1)], dtype=np.int64)
    return np.diff(offs)


def offsets_from_lens(lens) -> np.ndarray:
    lens = np.asarray(lens, dtype=np.int64)
    offs = np.zeros(lens.size + 1, dtype=np.int64)
    offs[1:] = np.cumsum(lens)
    return offs


def config_lens(name: str, seed: int = 0) -> np.ndarray:
    cfg = CONFIGS[name]
    if cfg["routing"] == "fixed":
        return np.asarray(cfg["lens"], dtype=np.int64)
    if cfg["routing"] == "multinomial":
        return multinomial_lens(cfg["G"], cfg["M_total"], seed)
    if cfg["routing"] == "zipf":
        return zipf_lens(cfg["G"], cfg["M_total"], seed)
    raise ValueError(cfg["routing"])


# ----------------------------------------------------------------------------------------------
# Operands
# ----------------------------------------------------------------------------------------------
@dataclasses.dataclass
class Problem:
    name: str
    G: int
    M_total: int
    OUT_M: int
    OUT_N: int
    lens: np.ndarray            # host int64 [G]
    offs: np.ndarray            # host int64 [G+1]
    lhs: torch.Tensor           # [rows, OUT_M] e4m3fn (rows = materialised token range)
    rhs: torch.Tensor           # [rows, OUT_N] e5m2
    lhs_scale: torch.Tensor     # fp32 [1] or [G]
    rhs_scale: torch.Tensor
    group_offs: torch.Tensor    # int64 [G+1] (same device as lhs)
    row0: int = 0               # first materialised token row

    @property
    def flops(self) -> float:
        return 2.0 * float(self.lens.sum()) * self.OUT_M * self.OUT_N

    def to(self, device) -> "Problem":
        return dataclasses.replace(
            self, lhs=self.lhs.to(device), rhs=self.rhs.to(device),
            lhs_scale=self.lhs_scale.to(device), rhs_scale=self.rhs_scale.to(device),
            group_offs=self.group_offs.to(device))


def _chunk_normal(rows: int, cols: int, seed: int, chunk: int, which: int, device) -> torch.Tensor:
    gen = torch.Generator(device=device)
    gen.manual_seed((seed * 1_000_003 + chunk * 7919 + which * 104_729) % (2**62))
    x = torch.randn(rows, cols, generator=gen, device=device, dtype=torch.float32)
    return x.to(torch.bfloat16)


def bf16_source(M_total: int, cols: int, seed: int, which: int, device="cpu") -> torch.Tensor:
    """The bf16 [M_total, cols] values a problem's operand is quantised from (which: 1 = LHS / x,
    2 = RHS / dy), generated chunk by chunk exactly as make_problem does."""
    parts = [_chunk_normal(min(CHUNK_ROWS, M_total - c0), cols, seed, c0 // CHUNK_ROWS, which,
                           device) for c0 in range(0, M_total, CHUNK_ROWS)]
    return torch.cat(parts) if parts else torch.empty(0, cols, dtype=torch.bfloat16, device=device)


def _row_scale(scales: torch.Tensor, offs: np.ndarray, r0: int, r1: int) -> torch.Tensor:
    """fp32 [r1-r0] scale of each token row."""
    if scales.numel() == 1:
        return scales.expand(r1 - r0)
    lens_local = []
    for g in range(len(offs) - 1):
        lo, hi = max(int(offs[g]), r0), min(int(offs[g + 1]), r1)
        lens_local.append(max(hi - lo, 0))
    return torch.repeat_interleave(scales, torch.tensor(lens_local, device=scales.device))


def _quantize_operand(M_total: int, cols: int, offs: np.ndarray, seed: int, which: int,
                      dtype, fmax: float, per_group: bool, r0: int, r1: int, device):
    G = len(offs) - 1
    # Pass 1: amax (per tensor, or per group) over ALL rows, chunk by chunk.
    amax_rows = []
    for c0 in range(0, M_total, CHUNK_ROWS):
        rows = min(CHUNK_ROWS, M_total - c0)
        x = _chunk_normal(rows, cols, seed, c0 // CHUNK_ROWS, which, device)
        amax_rows.append(x.abs().amax(dim=1).float())
    amax_rows = torch.cat(amax_rows) if amax_rows else torch.zeros(0, device=device)
    if per_group:
        scales = torch.ones(G, dtype=torch.float32, device=device)  # empty groups: 1.0
        for g in range(G):
            lo, hi = int(offs[g]), int(offs[g + 1])
            if hi > lo:
                scales[g] = amax_rows[lo:hi].max() / fmax
    else:
        scales = (amax_rows.max() / fmax).reshape(1) if M_total > 0 else torch.ones(1, device=device)
    scales = scales.to(torch.float32)
    # Pass 2: quantize the requested row range.
    out = torch.empty(r1 - r0, cols, dtype=dtype, device=device)
    for c0 in range((r0 // CHUNK_ROWS) * CHUNK_ROWS, r1, CHUNK_ROWS):
        rows = min(CHUNK_ROWS, M_total - c0)
        x = _chunk_normal(rows, cols, seed, c0 // CHUNK_ROWS, which, device)
        lo, hi = max(c0, r0), min(c0 + rows, r1)
        if hi <= lo:
            continue
        rs = _row_scale(scales, offs, lo, hi)
        q = (x[lo - c0:hi - c0].float() / rs[:, None]).clamp_(-fmax, fmax).to(dtype)
        out[lo - r0:hi - r0] = q
    return out, scales


def make_problem(name: str = "gate_up", *, seed: int = 0, device="cpu", lens=None,
                 G=None, M_total=None, OUT_M=None, OUT_N=None, scales=None,
                 rows: tuple[int, int] | None = None) -> Problem:
    """Build a seeded problem. `name` picks a config from CONFIGS; any field can be overridden
    (lens overrides routing). `rows` materialises only token rows [r0, r1) of LHS/RHS (the
    scales still cover every row), which is how expert-sharded ranks build their slice."""
    cfg = dict(CONFIGS.get(name, CONFIGS["gate_up"]))
    if lens is not None:
        lens = np.asarray(lens, dtype=np.int64)
        cfg["G"], cfg["M_total"] = int(lens.size), int(lens.sum())
    for k, v in (("G", G), ("M_total", M_total), ("OUT_M", OUT_M), ("OUT_N", OUT_N),
                 ("scales", scales)):
        if v is not None:
            cfg[k] = v
    if lens is None:
        if name in CONFIGS and G is None and M_total is None:
            lens = config_lens(name, seed)
        elif cfg["routing"] == "zipf":
            lens = zipf_lens(cfg["G"], cfg["M_total"], seed)
        else:
            lens = multinomial_lens(cfg["G"], cfg["M_total"], seed)
    offs = offsets_from_lens(lens)
    M = int(offs[-1])
    r0, r1 = rows if rows is not None else (0, M)
    per_group = cfg["scales"] == "group"
    lhs, sl = _quantize_operand(M, cfg["OUT_M"], offs, seed, 1, LHS_DTYPE, E4M3_MAX, per_group,
                                r0, r1, device)
    rhs, sr = _quantize_operand(M, cfg["OUT_N"], offs, seed, 2, RHS_DTYPE, E5M2_MAX, per_group,
                                r0, r1, device)
    return Problem(name=name, G=int(lens.size), M_total=M, OUT_M=cfg["OUT_M"],
                   OUT_N=cfg["OUT_N"], lens=lens, offs=offs, lhs=lhs, rhs=rhs,
                   lhs_scale=sl, rhs_scale=sr,
                   group_offs=torch.from_numpy(offs.copy()).to(device), row0=r0)


def launcher_problem(site: str = "gate_up_wgrad", device="cpu", G: int = 32,
                     M_total: int = 131072) -> Problem:
    """The reference C launcher's timing workload (launcher.cpp:64-112): uniform split, every
    LHS/RHS byte 0x38, scales 0.1. The launcher's comment calls 0x38 "0.5 in e4m3", which holds
    for the fnuz variant (bias 8); in the OCP e4m3fn format used here (and by bench.py's
    torch.float8_e4m3fn inputs) 0x38 is 1.0, while in e5m2 it is 0.5. Every output of a group
    with K tokens is therefore bf16(0.1f*0.1f * K * 0.5)."""
    OUT_M, OUT_N = {"gate_up_wgrad": (2880, 5760), "down_wgrad": (2880, 2880)}[site]
    lens = uniform_split_lens(G, M_total)
    offs = offsets_from_lens(lens)
    lhs = torch.full((M_total, OUT_M), 0x38, dtype=torch.uint8, device=device).view(LHS_DTYPE)
    rhs = torch.full((M_total, OUT_N), 0x38, dtype=torch.uint8, device=device).view(RHS_DTYPE)
    s = torch.tensor([0.1], dtype=torch.float32, device=device)
    return Problem(name=f"launcher_{site}", G=G, M_total=M_total, OUT_M=OUT_M, OUT_N=OUT_N,
                   lens=lens, offs=offs, lhs=lhs, rhs=rhs, lhs_scale=s, rhs_scale=s.clone(),
                   group_offs=torch.from_numpy(offs.copy()).to(device))
