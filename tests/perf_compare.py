"""Reference-path comparison on one B200 (not collected by pytest; run directly):

    python tests/perf_compare.py [--layers 30] [--iters 5] [--compile-mode max-autotune]

Times, on the same random-init weights and seeded inputs:
  * the stock-Wan eager forward (the oracle in the stock bf16 mixed precision), the path
    the reference measures as "eager" (coda_wan/run_wan_coda.py:248-252, 278-282);
  * the same under torch.compile (the reference's strong baseline, mode max-autotune,
    coda_wan/run_wan_coda.py:280);
  * the fused forward of this repository (FusedWanModel);
for config 3 (30-layer DiT, CFG batch 2, N = 32760) and config 1 (one block, N = 32760),
and reports the 30-layer parity of the fused output against eager (relative L2, max-abs,
the reference's allclose(2e-2) and latent PSNR, coda_wan/run_wan_coda.py:219-234).
Prints one JSON object per measurement. Lives under tests/ because it runs the oracle.
"""
from __future__ import annotations

import argparse
import json
import statistics
import sys
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

from oracle import wan_ref  # noqa: E402

LATENT = (16, 21, 60, 104)


def timeit(fn, iters):
    fn()
    torch.cuda.synchronize()
    out = []
    for _ in range(iters):
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        out.append(a.elapsed_time(b))
    return statistics.median(out)


def numerical(got, ref):
    got, ref = got.float(), ref.float()
    diff = (got - ref).abs()
    mse = (got - ref).square().mean()
    return {
        "rel_l2": ((got - ref).norm() / ref.norm()).item(),
        "max_abs": diff.max().item(),
        "mean_abs": diff.mean().item(),
        "allclose_rtol_2e-2_atol_2e-2": bool(torch.allclose(got, ref, rtol=2e-2, atol=2e-2)),
        "latent_psnr_db": float(20 * torch.log10((ref.max() - ref.min()) / torch.sqrt(mse))),
    }


def stock_model(cfg, layers, seed, dev):
    ref = wan_ref.init_weights_(wan_ref.WanModelRef(cfg, torch.bfloat16, num_layers=layers), seed=seed)
    ref = ref.to(dev)
    state = ref.state_dict()
    ref = ref.to(torch.bfloat16)
    ref.freqs = wan_ref.rope_freqs(1024, cfg.head_dim).to(dev)
    ref.time_embedding.float()
    ref.time_projection.float()
    for b in ref.blocks:
        b.modulation.data = b.modulation.data.float()
    ref.head.modulation.data = ref.head.modulation.data.float()
    return ref.eval(), state


def fused_model(pkg, state, layers, dev):
    params = pkg.build_wan(pkg.WAN_1_3B, seed=0, device=dev, num_layers=layers)
    params.load_state_dict(state, strict=True)
    params.to(torch.bfloat16)
    params.time_embedding.float()
    params.time_projection.float()
    for b in params.blocks:
        b.modulation.data = b.modulation.data.float()
    params.head.modulation.data = params.head.modulation.data.float()
    return pkg.FusedWanModel(params)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=30)
    ap.add_argument("--iters", type=int, default=5)
    ap.add_argument("--compile-mode", default="max-autotune")
    ap.add_argument("--skip-compile", action="store_true")
    a = ap.parse_args()
    from __graft_entry__ import load_package

    pkg = load_package()
    dev = torch.device("cuda")
    cfg = wan_ref.WAN_1_3B
    ref, state = stock_model(cfg, a.layers, seed=20260715, dev=dev)
    fused = fused_model(pkg, state, a.layers, dev)
    inp = wan_ref.model_inputs(cfg, LATENT[1:], 2, seed=20260716, device=dev)
    xs = [u.to(torch.bfloat16) for u in inp["x"]]
    ctx = [u.to(torch.bfloat16) for u in inp["context"]]
    args = (xs, inp["t"], ctx, inp["seq_len"])
    info = {"gpu": torch.cuda.get_device_name(), "torch": torch.__version__, "layers": a.layers,
            "workload": "cfg3: CFG batch 2, N=32760/sample, random init, bf16"}
    print(json.dumps(info), flush=True)
    with torch.no_grad():
        want = ref(*args)
        got = fused(*args)
        print(json.dumps({"parity_fused_vs_stock_eager": numerical(torch.stack(got), torch.stack(want))}), flush=True)
        del want, got
        t_ours = timeit(lambda: fused(*args), a.iters)
        print(json.dumps({"cfg3_fused_ms": t_ours}), flush=True)
        t_eager = timeit(lambda: ref(*args), a.iters)
        print(json.dumps({"cfg3_stock_eager_ms": t_eager, "speedup_vs_eager": t_eager / t_ours}), flush=True)
        # config 1: one block, batch 1, N = 32760
        blk_inp = wan_ref.block_inputs(cfg, (21, 30, 52), 1, seed=14, device=dev)
        x1 = blk_inp["x"].to(torch.bfloat16)
        ctx1 = blk_inp["context"].to(torch.bfloat16)
        freqs = fused.freqs
        b_ref = ref.blocks[0]
        b_fused = fused.model.blocks[0]
        bargs = (blk_inp["seq_lens"], blk_inp["grid_sizes"], freqs, ctx1, blk_inp["context_lens"])
        t_b_eager = timeit(lambda: b_ref(x1, blk_inp["e"], *bargs), a.iters)
        t_b_ours = timeit(lambda: b_fused(x1, blk_inp["e"], *bargs), a.iters)
        print(json.dumps({"cfg1_block_stock_eager_ms": t_b_eager, "cfg1_block_fused_ms": t_b_ours}), flush=True)
        if not a.skip_compile:
            t0 = time.time()
            cref = torch.compile(ref, mode=a.compile_mode, fullgraph=False)
            cref(*args)
            torch.cuda.synchronize()
            compile_s = time.time() - t0
            t_comp = timeit(lambda: cref(*args), a.iters)
            print(json.dumps({"cfg3_stock_compile_ms": t_comp, "compile_mode": a.compile_mode,
                              "compile_seconds": compile_s, "speedup_vs_compile": t_comp / t_ours}), flush=True)
            cblk = torch.compile(b_ref, mode=a.compile_mode, fullgraph=False)
            t_b_comp = timeit(lambda: cblk(x1, blk_inp["e"], *bargs), a.iters)
            print(json.dumps({"cfg1_block_stock_compile_ms": t_b_comp}), flush=True)
    pkg._lib.raise_on_device_error()


if __name__ == "__main__":
    main()
