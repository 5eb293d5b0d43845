#!/usr/bin/env python3
"""Wan2.1 DiT forward benchmark. Default workload (config 3): Wan2.1-1.3B, 30 layers, CFG
batch 2, N = 32760 tokens per sample (latent [16, 21, 60, 104], patch (1, 2, 2)), text context
[512, 4096] per sample, t = 500, bf16, random-init weights, seeded synthetic inputs.
`--workload cfg4`: the Wan2.1-14B shape (dim 5120, 40 heads, ffn 13824, 40 layers) at 720p
(latent [16, 21, 90, 160], N = 75600), CFG batch 2.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload cfg3|cfg4]
    torchrun --nproc-per-node N bench.py --gpus N ...   (token-sharded, Ulysses all-to-all)

One "step" is one DiT forward of the CFG batch (one denoising step). Prints one JSON line.
  value        device time per step (CUDA events, inputs resident in HBM; max over ranks)
  e2e          the same forward through the public API with host (pinned) buffers, the H2D
               copy of the inputs and the D2H copy of the output inside the timed region
  roofline     FFN1 fused GEMM (the largest kernel): algorithmic FLOPs per launch / its
               CUDA-event duration inside the timed region, vs the measured bf16 peak
  oracle_*     (N = 1, cfg3) the stock-Wan forward restated in eager PyTorch, bf16 mixed
               precision, with the same weights and inputs on the same GPU: eager and
               torch.compile(mode="max-autotune"), the reference's two baselines
               (coda_wan/run_wan_coda.py:248-252, 278-282); reported beside `value`, never in it
  cpu_baseline the eager fp32 stock-Wan block on the host cores, timed on one exact unit of the
               forward (one block, one CFG sample, all N tokens) and multiplied by the
               layers x samples of the forward
Activations (> 1 GB per step) exceed the 126 MB L2, so no explicit flush is needed.
"""
from __future__ import annotations

import argparse
import contextlib
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

WORKLOADS = {
    "cfg3": {"metric": "Wan-1.3B DiT step ms (CFG b2, N=32760) @1/2/4/8 B200; fused-GEMM % bf16 peak",
             "name": "cfg3: Wan2.1-1.3B 30-layer DiT forward, CFG batch 2, N=32760/sample",
             "shape": "WAN_1_3B", "latent": (16, 21, 60, 104), "dim": 1536, "ffn": 8960, "heads": 12, "layers": 30},
    "cfg4": {"metric": "Wan-14B-shaped DiT step ms (CFG b2, N=75600) @1/2/4/8 B200; fused-GEMM % bf16 peak",
             "name": "cfg4: Wan2.1-14B-shaped 40-layer DiT forward (720p), CFG batch 2, N=75600/sample",
             "shape": "WAN_14B", "latent": (16, 21, 90, 160), "dim": 5120, "ffn": 13824, "heads": 40, "layers": 40},
}
PATCH = (1, 2, 2)
TEXT = (512, 4096)
BATCH = 2
T_STEP = 500.0
SEED = 20260715


def seq_len(w: dict) -> int:
    f, h, wd = w["latent"][1:]
    return f * (h // PATCH[1]) * (wd // PATCH[2])


def block_flops(B: int, L: int, D: int, F: int, Lc: int = 512) -> dict:
    M = B * L
    gemm = 2 * M * D * (3 * D + D + D + D + 2 * F) + 2 * B * Lc * D * 2 * D
    attn = 4 * B * L * L * D + 4 * B * L * Lc * D
    return {"gemm": gemm, "attn": attn, "total": gemm + attn}


def forward_flops(w: dict, layers: int) -> dict:
    f = block_flops(BATCH, seq_len(w), w["dim"], w["ffn"])
    return {k: v * layers for k, v in f.items()}


def load_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16": d["bf16_tflops"], "bf16_sustained": d["bf16_tflops_sustained"],
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16": 1590.0, "bf16_sustained": 1400.0, "source": "fallback"}


def traffic_from_profiles(kernel: str) -> float | None:
    """Per-launch DRAM bytes of `kernel` from the committed ncu summary (scaled to the bench
    shape there), or None when no capture exists."""
    p = ROOT / "profiles" / "traffic_per_launch.txt"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        parts = line.split()
        if len(parts) >= 2 and parts[0] == kernel:
            return float(parts[1])
    return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 50 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = None
        self.skip = 0

    def _lines(self) -> list[str]:
        try:
            return [ln for ln in Path(self.path).read_text().splitlines() if ln.count(",") >= 8]
        except OSError:
            return []

    def start(self):
        """Start sampling every 50 ms; returns once sampling is live, so that only samples taken
        after this call (inside the timed region that follows) are kept."""
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
            return
        t0 = time.time()
        while time.time() - t0 < 10.0 and not self._lines():
            time.sleep(0.02)
        self.skip = len(self._lines())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        for line in self._lines()[self.skip:]:
            f = [x.strip() for x in line.split(",")]
            if len(f) >= 9:
                rows.append(f)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def cpu_block_unit(w: dict, repeats: int = 1) -> dict:
    """The eager fp32 stock-Wan block (the oracle) on all host cores, timed on one exact unit
    of the forward: one block, one CFG sample, all N tokens of the workload (every block and
    sample of the forward has the same shapes and work; the non-block parts (patch / text /
    time embeddings, head) are < 0.5% of the forward and not timed). Returns the unit time."""
    from oracle import wan_ref

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    cfg = wan_ref.WAN_1_3B if w["shape"] == "WAN_1_3B" else wan_ref.WAN_14B
    blk = wan_ref.init_weights_(wan_ref.WanBlockRef(cfg, torch.float32), seed=SEED).eval()
    f, h, wd = w["latent"][1:]
    grid = (f, h // PATCH[1], wd // PATCH[2])
    inp = wan_ref.block_inputs(cfg, grid, 1, seed=SEED)
    freqs = wan_ref.rope_freqs(1024, cfg.head_dim)
    times = []
    with torch.no_grad():
        for _ in range(repeats):
            t0 = time.perf_counter()
            blk(inp["x"].clone(), inp["e"], inp["seq_lens"], inp["grid_sizes"], freqs, inp["context"],
                inp["context_lens"])
            times.append(time.perf_counter() - t0)
    return {"unit_s": statistics.median(times), "threads": threads, "runs": len(times)}


def cpu_baseline_line(w: dict, layers: int) -> dict:
    r = cpu_block_unit(w, repeats=1)
    units = layers * BATCH
    return {"value": r["unit_s"] * 1e3 * units, "unit": "ms", "cores": r["threads"], "kind": "port",
            "sample": f"1 stock-Wan block (fp32 eager oracle) on 1 sample at the workload's N={seq_len(w)} "
                      f"tokens: {r['unit_s'] * 1e3:.0f} ms; x {units} = {layers} layers x {BATCH} CFG samples "
                      f"(identical units; embeddings and head not timed)",
            "cpu_model": _cpu_model()}


def _cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except Exception:
        pass
    return "unknown"


def run_reference(args) -> None:
    """The reference arm: the reference has no CPU implementation of this path (its kernels are
    CUDA / Triton / CuTeDSL on an absent Hopper GEMM package), so its stock eager block is timed
    through the fp32 oracle restatement on the host cores. One step = one exact unit of the
    forward (one block on one CFG sample at the full N); the forward is layers x samples units.
    The CPU needs no long warm-up: at most one untimed unit runs first."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    w = WORKLOADS[args.workload]
    layers = args.layers or w["layers"]
    units = layers * BATCH
    if args.warmup > 0:
        cpu_block_unit(w, repeats=1)
    r = cpu_block_unit(w, repeats=args.steps)
    v = r["unit_s"] * 1e3 * units
    base = {"value": v, "unit": "ms", "cores": r["threads"], "kind": "port",
            "sample": f"per step: 1 stock-Wan block (fp32 eager oracle) on 1 CFG sample at N={seq_len(w)}; "
                      f"median of {r['runs']} steps = {r['unit_s'] * 1e3:.0f} ms, x {units} "
                      f"({layers} layers x {BATCH} samples, identical units)",
            "cpu_model": _cpu_model()}
    line = {
        "metric": w["metric"], "impl": "reference", "value": v, "unit": "ms", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": min(args.warmup, 1), "ms_per_step": v, "higher_is_better": False,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded randn inputs, random-init weights)",
        "config": {"workload": w["name"], "weights": "random init", "layers": layers, "global_batch": BATCH,
                   "seq_len": seq_len(w), "latent": list(w["latent"]), "context": list(TEXT), "t": T_STEP,
                   "parallelism": "host cores (rank 0 only)"},
        "cpu_baseline": base,
        "e2e": {"value": v, "unit": "ms", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "The reference's fused path needs coda-kernels (rapier, unpinned, not installable offline) and "
                "Hopper; its stock eager block runs here as the build's fp32 oracle restatement on the host CPU.",
    }
    print(json.dumps(line), flush=True)


@contextlib.contextmanager
def stdout_to_stderr():
    """Send everything written to file descriptor 1 meanwhile to stderr. torch.compile's
    max-autotune prints its tuning tables, JSON-formatted lines among them, to stdout; the
    benchmark's stdout must carry only its own result line."""
    sys.stdout.flush()
    saved = os.dup(1)
    try:
        os.dup2(2, 1)
        yield
    finally:
        sys.stdout.flush()
        os.dup2(saved, 1)
        os.close(saved)


def oracle_gpu_baselines(pkg, w: dict, state: dict, layers: int, args_fwd, iters: int, warmup: int,
                         compile_mode: str | None) -> dict:
    """The reference's two GPU baselines on this GPU with this run's weights and inputs: the
    stock-Wan forward (oracle restatement) in eager bf16 mixed precision, and the same under
    torch.compile. Median of `iters` CUDA-event-timed forwards after `warmup` untimed ones."""
    from oracle import wan_ref

    cfg = wan_ref.WAN_1_3B if w["shape"] == "WAN_1_3B" else wan_ref.WAN_14B
    dev = torch.device("cuda", torch.cuda.current_device())
    stock = wan_ref.stock_bf16_model(cfg, state, dev, num_layers=layers)

    def median_ms(fn):
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
            torch.cuda.synchronize()
            out.append(a.elapsed_time(b))
        return statistics.median(out)

    res = {"what": "stock-Wan forward restated in eager PyTorch (oracle), bf16 mixed precision, same weights "
                   "and inputs, same GPU", "iters": iters, "warmup": warmup}
    with torch.no_grad(), stdout_to_stderr():
        res["eager_ms"] = median_ms(lambda: stock(*args_fwd))
        if compile_mode:
            # a compiler failure must not cost the benchmark line: it is reported instead
            try:
                t0 = time.time()
                comp = torch.compile(stock, mode=compile_mode)
                comp(*args_fwd)
                torch.cuda.synchronize()
                res["compile_s"] = time.time() - t0
                res["compile_mode"] = compile_mode
                res["compile_ms"] = median_ms(lambda: comp(*args_fwd))
                del comp
            except Exception as exc:  # noqa: BLE001
                res["compile_error"] = f"{type(exc).__name__}: {str(exc)[:300]}"
    del stock
    torch.cuda.empty_cache()
    return res


def run_ours(args) -> None:
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(minutes=5))
    from __graft_entry__ import load_package

    pkg = load_package()
    w = WORKLOADS[args.workload]
    layers = args.layers or w["layers"]
    latent = w["latent"]
    L = seq_len(w)
    sp = None
    if world > 1:
        sp = pkg.SeqParallel(dist.group.WORLD, world, rank, (latent[1], latent[2] // 2, latent[3] // 2), L,
                             transport=args.transport, gemm_exchange=args.gemm_exchange)
    torch.manual_seed(SEED)
    params = pkg.build_wan(getattr(pkg, w["shape"]), seed=SEED, device=dev, num_layers=layers)
    # The weights as built (before the fused blocks re-point the parameters at packed storage),
    # for the stock-Wan comparison forwards after the timed regions.
    want_oracle = world == 1 and not args.no_oracle and (args.workload == "cfg3" or args.oracle)
    state = dict(params.state_dict()) if want_oracle else None
    model = pkg.FusedWanModel(params, sp)

    g = torch.Generator().manual_seed(SEED + 1)
    host_x = [torch.randn(*latent, generator=g).to(torch.bfloat16).pin_memory() for _ in range(BATCH)]
    host_c = [torch.randn(*TEXT, generator=g).to(torch.bfloat16).pin_memory() for _ in range(BATCH)]
    t = torch.full((BATCH,), T_STEP)
    dev_x = [h.to(dev) for h in host_x]
    dev_c = [h.to(dev) for h in host_c]

    def forward_resident():
        return model(dev_x, t, dev_c, L)

    out_shape = forward_resident()
    out_host = [torch.empty(o.shape, dtype=o.dtype, pin_memory=True) for o in
                (out_shape if isinstance(out_shape, list) else [out_shape])]
    h2d = sum(h.numel() * h.element_size() for h in host_x + host_c)
    d2h = sum(o.numel() * o.element_size() for o in out_host)

    def forward_e2e():
        xs = [h.to(dev, non_blocking=True) for h in host_x]
        cs = [h.to(dev, non_blocking=True) for h in host_c]
        out = model(xs, t, cs, L)
        outs = out if isinstance(out, list) else [out]
        for o, hbuf in zip(outs, out_host):
            hbuf.copy_(o, non_blocking=True)
        return out

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def timed(fn, k, tag):
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        torch.cuda.nvtx.range_push(tag)
        e0.record()
        for _ in range(k):
            fn()
        e1.record()
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        ms = torch.tensor([e0.elapsed_time(e1) / k], device=dev)
        if world > 1:
            dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        barrier()
        return float(ms.item())

    with torch.no_grad():
        for _ in range(args.warmup):
            forward_resident()
        for _ in range(max(1, args.warmup // 2)):
            forward_e2e()
        pkg._lib.raise_on_device_error()

        # Timed region 1: resident inputs, with per-launch events around the FFN1 GEMMs.
        timer = []
        for blk in model.model.blocks:
            blk.kernel_timer = timer
        clocks = ClockSampler(local)
        clocks.start()
        n0 = pkg._lib.launch_counter["n"]
        ms = timed(forward_resident, args.steps, "timed_resident")
        launches = pkg._lib.launch_counter["n"] - n0
        clk = clocks.stop()
        if world > 1:
            # every rank sampled its own GPU: gather the medians (clock-normalized comparison across N)
            mine = torch.tensor([float(clk.get("sm_mhz") or 0.0)], device=dev)
            every = [torch.zeros_like(mine) for _ in range(world)]
            dist.all_gather(every, mine)
            clk["per_rank_sm_mhz"] = [float(t.item()) for t in every]
        for blk in model.model.blocks:
            blk.kernel_timer = None
        k_ms = [a.elapsed_time(b) for a, b, _ in timer]
        k_flops = timer[0][2] if timer else 0.0
        # Timed region 2: end to end from host buffers.
        ms_e2e = timed(forward_e2e, args.steps, "timed_e2e")
        pkg._lib.raise_on_device_error()

    peaks = load_peaks()
    ffn1_ms = statistics.mean(k_ms) if k_ms else float("nan")
    ach = k_flops / (ffn1_ms * 1e-3) / 1e12 if k_ms else None
    fl = forward_flops(w, layers)
    result = None
    if rank == 0:
        sm_mhz = clk.get("sm_mhz")
        result = {
            "metric": w["metric"],
            "value": ms,
            "unit": "ms",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms,
            "higher_is_better": False,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded randn latents/contexts, random-init weights; no checkpoint)",
            "config": {"workload": w["name"],
                       "weights": "random init", "layers": layers, "global_batch": BATCH,
                       "seq_len": L, "latent": list(latent), "context": list(TEXT), "t": T_STEP,
                       "parallelism": (f"sp{world} (token-sharded, Ulysses all-to-all over {args.transport}"
                                       + (", sent by the QKV GEMM" if sp is not None and sp.gemm_exchange else "")
                                       + ")" if world > 1 else "single GPU"),
                       "attention": "torch SDPA (out of scope)", "l2": "activations > L2 (no flush needed)"},
            "tflops": fl["total"] / (ms * 1e-3) / 1e12,
            "gemm_tflop_per_step": fl["gemm"] / 1e12,
            # step time x median SM clock (GHz): clock-independent work measure for comparing N
            "ms_x_sm_ghz": ms * sm_mhz / 1e3 if sm_mhz else None,
            "e2e": {"value": ms_e2e, "unit": "ms", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "roofline": {
                "kernel": f"wdit gemm_kernel<kEpiAct> (FFN1 {w['dim']}->{w['ffn']}, LN folded, bias+tanh-GELU "
                          f"epilogue)",
                "bound": "tensor",
                "achieved": ach,
                "peak": peaks["bf16_sustained"],
                "unit": "TFLOP/s",
                "frac": (ach / peaks["bf16_sustained"]) if ach else None,
                "frac_of_burst_peak": (ach / peaks["bf16"]) if ach else None,
                "peak_source": f"{peaks['source']} bf16_tflops_sustained (kernel timed inside the long step)",
                "launch_ms": ffn1_ms,
                "flops_per_launch": k_flops,
                # one ncu capture of the FFN1 launch at M = 65520 (1 GPU), scaled by the rows of
                # this launch (A and the GELU output scale with the rows; the 27.5 MB weight does not)
                "traffic": (traffic_from_profiles("ffn1_gemm") * (timer[0][2] / (2.0 * 65520 * w["ffn"] * w["dim"]))
                            if args.workload == "cfg3" and timer and traffic_from_profiles("ffn1_gemm") else None),
            },
            "clocks": clk,
            "gpu_launches": launches,
        }
    if want_oracle:
        # The reference's GPU baselines, after (never inside) the timed regions.
        del model
        torch.cuda.empty_cache()
        try:
            ob = oracle_gpu_baselines(pkg, w, state, layers, (dev_x, t, dev_c, L), iters=args.oracle_iters,
                                      warmup=3, compile_mode=None if args.no_compile else "max-autotune")
        except Exception as exc:  # noqa: BLE001  (the baselines are reported, never required)
            ob = {"error": f"{type(exc).__name__}: {str(exc)[:300]}"}
        del state
        if "eager_ms" in ob:
            result["oracle_eager_ms"] = ob["eager_ms"]
            result["speedup_vs_eager"] = ob["eager_ms"] / ms
        if "compile_ms" in ob:
            result["oracle_compile_ms"] = ob["compile_ms"]
            result["oracle_compile_s"] = ob["compile_s"]
            result["speedup_vs_compile"] = ob["compile_ms"] / ms
        result["oracle_gpu"] = ob
    if rank == 0 and not args.no_cpu_baseline and world == 1:
        result["cpu_baseline"] = cpu_baseline_line(w, layers)
    if world > 1:
        sp.close()
        dist.barrier()
        dist.destroy_process_group()
    if result is not None:
        print(json.dumps(result), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", choices=tuple(WORKLOADS), default="cfg3")
    ap.add_argument("--layers", type=int, default=0, help="layers of the forward (default: the workload's)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-oracle", action="store_true",
                    help="skip the stock-Wan eager / torch.compile forwards on the GPU (N = 1, cfg3)")
    ap.add_argument("--oracle", action="store_true",
                    help="also run the stock-Wan eager / torch.compile forwards for workloads other than cfg3")
    ap.add_argument("--no-compile", action="store_true", help="skip only the torch.compile forward")
    ap.add_argument("--oracle-iters", type=int, default=5)
    ap.add_argument("--transport", choices=("p2p", "nccl"), default="p2p",
                    help="Ulysses all-to-all: NVLink peer stores (p2p) or NCCL all_to_all_single")
    ap.add_argument("--gemm-exchange", action="store_true",
                    help="p2p: the QKV GEMM stores q / k / v into the peers itself instead of a separate "
                         "exchange kernel after it (0.5%% slower on B200 at 2 GPUs, kept as an option)")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
