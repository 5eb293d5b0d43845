"""Config 2: isolated fused-GEMM microbenchmark on one B200 (plus the memory-bound passes).

    python microbench.py [--m 32760] [--only ffn1,ffn2,...] [--iters 20] [--model 1.3b|14b]

Each kernel is timed alone with CUDA events (median of --iters launches after warm-up; the
operands exceed the 126 MB L2 at the default M, so launches do not hit in L2 from the
previous one). Reported per kernel: ms, TFLOP/s (2*M*N*K) or GB/s (algorithmic bytes), the
fraction of the measured burst peak (MEASURED_PEAKS.json: timed alone), and the same-shape
torch.matmul (cuBLAS, bf16) time for context.

Shapes (Wan2.1-1.3B, batch 1, N = 32760 tokens):
  ffn1   [M x 1536] . [1536 x 8960]  LayerNorm folded + shift term + bias + tanh-GELU -> bf16
  ffn2   [M x 8960] . [8960 x 1536]  (acc + b) * gate + residual -> fp32, + bf16 copy + LN stats
  qkv    [M x 1536] . [1536 x 4608]  LN folded, full-width q/k RMSNorm, 3D RoPE -> bf16 (one launch;
                                     qkv_split: GEMM + partials, then the RMSNorm / RoPE pass)
  self_o [M x 1536] . [1536 x 1536]  gate + residual (+ bf16 copy + stats)
  cross_q[M x 1536] . [1536 x 1536]  norm3 folded + RMSNorm (cross_q_split: two launches)
  cross_o[M x 1536] . [1536 x 1536]  bias + residual (+ bf16 copy + stats)
  stats  LayerNorm statistics pass over fp32 [M x 1536]   (reads 4 B, writes 8 B per row... HBM)
  fold   per-step weight fold of the FFN1 weight [8960 x 1536] (reads 2 B + writes 2 B / weight)
(`--model 14b`: the same kernels at the Wan2.1-14B shapes, dim 5120 and ffn 13824.)
"""
from __future__ import annotations

import argparse
import json
import statistics
import sys
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent


def _pkg():
    sys.path.insert(0, str(ROOT))
    from __graft_entry__ import load_package

    return load_package()


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["bf16_tflops"], d["hbm_gbs"], "measured"
    return 1590.0, 6650.0, "fallback"


def _time(fn, iters: int, warmup: int = 3) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    out = []
    for _ in range(iters):
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        b.synchronize()
        out.append(a.elapsed_time(b))
    return statistics.median(out)


SHAPES = {"1.3b": (1536, 8960), "14b": (5120, 13824)}  # (dim, ffn_dim)


def run(M: int = 32760, only: set[str] | None = None, iters: int = 20, cublas: bool = True,
        model: str = "1.3b") -> list[dict]:
    pkg = _pkg()
    ops = pkg.ops
    dev = torch.device("cuda")
    D, F = SHAPES[model]
    g = torch.Generator(device="cpu").manual_seed(0)

    def rnd(shape, scale=1.0, dtype=torch.bfloat16):
        return (scale * torch.randn(shape, generator=g)).to(dtype).to(dev)

    peak_tf, peak_bw, src = _peaks()
    x32 = rnd((M, D), 1.0, torch.float32)
    xb = x32.to(torch.bfloat16)
    stats = ops.ln_stats(x32)
    res = []

    def add(name, ms, flops=None, nbytes=None, cublas_ms=None):
        row = {"kernel": name, "model": model, "M": M, "ms": ms}
        if flops:
            row["tflops"] = flops / (ms * 1e-3) / 1e12
            row["frac_of_peak"] = row["tflops"] / peak_tf
        if nbytes:
            row["gbs"] = nbytes / (ms * 1e-3) / 1e9
            row["frac_of_hbm"] = row["gbs"] / peak_bw
        if cublas_ms:
            row["cublas_ms"] = cublas_ms
        row["peak_source"] = src
        res.append(row)
        print(json.dumps(row), flush=True)

    def want(n):
        return only is None or n in only

    def cub(a, w):
        if not cublas:
            return None
        return _time(lambda: torch.matmul(a, w.t()), iters)

    if want("ffn1"):
        w = rnd((F, D), 0.02)
        s = rnd((D,), 0.1, torch.float32)
        sh = rnd((D,), 0.1, torch.float32)
        b = rnd((F,), 0.01, torch.float32)
        wf, cs, vec = ops.fold_weight(w, mult_c=1.0, mult_a=s, shift_a=sh, bias=b)
        h = torch.empty((M, F), dtype=torch.bfloat16, device=dev)
        ln = ops.LnFold(cs, stats, 1e-6)
        ms = _time(lambda: ops.gemm_act(xb, wf, vec=vec, act="gelu_tanh", ln=ln, out=h), iters)
        add("ffn1", ms, 2.0 * M * F * D, cublas_ms=cub(xb, wf))
    if want("fold"):
        w = rnd((F, D), 0.02)
        s = rnd((D,), 0.1, torch.float32)
        outs = (torch.empty_like(w), torch.empty(F, device=dev), torch.empty(F, device=dev))
        ms = _time(lambda: ops.fold_weight(w, mult_c=1.0, mult_a=s, shift_a=s, w_out=outs[0], csum_out=outs[1],
                                           vec_out=outs[2]), iters)
        add("fold", ms, nbytes=4.0 * F * D)
    if want("stats"):
        st = torch.empty_like(stats)
        ms = _time(lambda: ops.ln_stats(x32, stats_out=st), iters)
        add("stats", ms, nbytes=4.0 * M * D + 8.0 * M * (D // 256))
    if want("ffn2"):
        h = rnd((M, F))
        w = rnd((D, F), 0.02)
        c = x32.clone()
        gate = rnd((D,), 0.1, torch.float32)
        b = rnd((D,), 0.01, torch.float32)
        xo = torch.empty((M, D), dtype=torch.bfloat16, device=dev)
        so = torch.empty_like(stats)
        ms = _time(lambda: ops.gemm_residual(h, w, c, out=c, bias=b, gate_a=gate, x_bf16_out=xo, stats_out=so),
                   iters)
        add("ffn2", ms, 2.0 * M * D * F, cublas_ms=cub(h, w))
    for name, fused in (("qkv", True), ("qkv_split", False)):
        if not want(name):
            continue
        w = rnd((3 * D, D), 0.02)
        s = rnd((D,), 0.1, torch.float32)
        wf, cs, vec = ops.fold_weight(w, mult_c=1.0, mult_a=s, shift_a=s)
        ang = rnd((M, 64), 3.0, torch.float32)
        cos, sin = torch.cos(ang), torch.sin(ang)  # token-major [M, 64]
        nw = 1.0 + rnd((D,), 0.1, torch.float32)
        out = torch.empty((M, 3 * D), dtype=torch.bfloat16, device=dev)
        ln = ops.LnFold(cs, stats, 1e-6)
        ws = ops.Workspace()
        ms = _time(lambda: ops.gemm_norm(xb, wf, vec=vec, ln=ln, norm_groups=2, norm_width=D, norm_w=(nw, nw),
                                         rope_groups=2, rope_cos=cos, rope_sin=sin, rows_per_batch=M, out=out,
                                         workspace=ws, fused=fused), iters)
        add(name, ms, 2.0 * M * 3 * D * D, cublas_ms=cub(xb, wf))
    for name, gate in (("self_o", True), ("cross_o", False)):
        if want(name):
            a = rnd((M, D))
            w = rnd((D, D), 0.02)
            c = x32.clone()
            gt = rnd((D,), 0.1, torch.float32) if gate else None
            b = rnd((D,), 0.01, torch.float32)
            xo = torch.empty((M, D), dtype=torch.bfloat16, device=dev)
            so = torch.empty_like(stats)
            ms = _time(lambda: ops.gemm_residual(a, w, c, out=c, bias=b, gate_a=gt, x_bf16_out=xo, stats_out=so),
                       iters)
            add(name, ms, 2.0 * M * D * D, cublas_ms=cub(a, w))
    for name, fused in (("cross_q", True), ("cross_q_split", False)):
        if not want(name):
            continue
        w = rnd((D, D), 0.02)
        gm = 1.0 + rnd((D,), 0.1, torch.float32)
        wf, cs, vec = ops.fold_weight(w, mult_c=0.0, mult_a=gm, shift_a=gm)
        nw = 1.0 + rnd((D,), 0.1, torch.float32)
        out = torch.empty((M, D), dtype=torch.bfloat16, device=dev)
        ln = ops.LnFold(cs, stats, 1e-6)
        ws = ops.Workspace()
        ms = _time(lambda: ops.gemm_norm(xb, wf, vec=vec, ln=ln, norm_groups=1, norm_width=D, norm_w=(nw, None),
                                         out=out, workspace=ws, fused=fused), iters)
        add(name, ms, 2.0 * M * D * D, cublas_ms=cub(xb, wf))
    pkg._lib.raise_on_device_error()
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--m", type=int, default=32760)
    ap.add_argument("--only", type=str, default="")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--no-cublas", action="store_true")
    ap.add_argument("--pair", type=int, default=1, help="CTA pairs for the tensor-bound GEMMs (1) or not (0)")
    ap.add_argument("--model", choices=tuple(SHAPES), default="1.3b",
                    help="layer shapes: Wan2.1-1.3B (dim 1536, ffn 8960) or 14B (dim 5120, ffn 13824)")
    a = ap.parse_args()
    only = set(a.only.split(",")) if a.only else None
    _pkg()._lib.load().wdit_set_cta_pair(a.pair)
    run(a.m, only, a.iters, not a.no_cublas, a.model)


if __name__ == "__main__":
    main()
