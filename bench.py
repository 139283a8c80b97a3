"""Benchmark of the exact base/residual split FFN path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload c2]

Workload (default): the Llama-7B-shape FFN stack — 32 layers, d_model 4096,
d_ff 11008, Q4 codes with a radix-4 split (r = 2: base = high 2 bits from the host,
residual = low 2 bits on the GPU), decode batches of 1, 8 and 64 tokens. One step
runs the three batches back to back through all 32 layers (73 tokens). Every
layer has its own seeded synthetic weights, activations and host base sums.
The stack's weights (~4 GB) exceed L2 (126 MB), so no layer's weights are L2
resident when it runs again; no explicit flush is needed.

* ``value``  — tokens/s with inputs (activations, base sums) resident in HBM.
* ``e2e``    — the same through the public host API: per layer, pinned host
  activations and base sums are copied in (base sums on a side stream,
  overlapped with the residual contraction) and y is copied back.
* N > 1 ranks (torchrun): d_ff sharded, row-parallel down, one NCCL allreduce of
  the fp32 partial per layer; value = all tokens / max-over-ranks time.
* ``--impl reference``: the reference's own AVX2 CPU implementation of the path
  (direct_q4 gate/up from src/radix_cpu_kernels.h, built from its source into
  oracle/_ref) plus the SwiGLU/down step, timed on this host's cores over a
  bounded sample (one layer per step, scaled to the 32-layer stack).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from ffn_residual_mesh_b200 import synth  # noqa: E402

METRIC = "FFN tokens/s"
UNIT = "tokens/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", default="c2", choices=("c2",))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--eager", action="store_true", help="time eager calls instead of CUDA-graph replays")
    ap.add_argument("--layers", type=int, default=None, help="override the stack depth (profiling cases)")
    ap.add_argument("--tokens", type=str, default=None, help="override the decode batches, e.g. 64 or 1,8")
    return ap.parse_args()


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def config_block(cfg, world):
    return {"workload": cfg.workload, "layers": cfg.layers, "d_model": cfg.d_model, "d_ff": cfg.d_ff,
            "residual_bits": cfg.residual_bits, "decode_tokens": list(cfg.tokens),
            "tokens_per_step": sum(cfg.tokens), "base_tile_rows": cfg.base_tile_rows,
            "parallelism": f"d_ff-shard{world}" if world > 1 else "single-gpu",
            "l2": "working set (stack weights) larger than L2; no flush"}


# ---------------------------------------------------------------------------
# clocks
# ---------------------------------------------------------------------------
class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index, self.proc, self.lines = index, None, []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                                          "-i", str(self.index), "-lms", "200"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "samples": len(sm), "reasons": sorted(reasons)}


# ---------------------------------------------------------------------------
# reference CPU arm (oracle/_ref = the reference's AVX2 evaluator)
# ---------------------------------------------------------------------------
class CpuReference:
    """The reference's CPU path on ``layers_sample`` layers of the workload."""

    def __init__(self, cfg, layers_sample: int = 1):
        from oracle import refcpu
        if not refcpu.available():
            subprocess.run(["make", "-C", str(ROOT / "oracle")], check=True, capture_output=True)
        self.cfg, self.threads = cfg, os.cpu_count() or 1
        self.models, self.acts = [], []
        for l in range(layers_sample):
            L = synth.make_layer(1000 + l, cfg.d_ff, cfg.d_model)
            self.models.append(refcpu.RefFfn(L.gate_codes, L.up_codes, L.gate_alpha, L.up_alpha, L.gate_beta,
                                             L.up_beta, L.down, threads=self.threads))
            self.acts.append([synth.make_activations(7000 + 100 * l + T, T, cfg.d_model)[1:] for T in cfg.tokens])
        self.models[0].forward(*self.acts[0][0])  # warm the pool and pages

    def step_seconds(self) -> float:
        """One bounded sample: every sampled layer x every batch, scaled to the stack."""
        t0 = time.perf_counter()
        for m, acts in zip(self.models, self.acts):
            for z, s in acts:
                m.forward(z, s)
        return (time.perf_counter() - t0) / len(self.models) * self.cfg.layers

    def info(self):
        return {"cores": self.threads, "kind": "reference",
                "sample": f"{len(self.models)} of {self.cfg.layers} layers x batches {list(self.cfg.tokens)} at full "
                          f"d_ff={self.cfg.d_ff}, d_model={self.cfg.d_model}: reference direct_q4 AVX2 gate/up per "
                          "token (src/radix_cpu_kernels.h:228-248) + SwiGLU + fp16 down, time scaled to all layers"}

    def close(self):
        for m in self.models:
            m.close()


def run_reference(args, cfg, rank, world):
    if rank != 0:
        return
    ref = CpuReference(cfg, layers_sample=1)
    secs = [ref.step_seconds() for _ in range(args.warmup + args.steps)][args.warmup:]
    sec = statistics.median(secs)
    v = sum(cfg.tokens) / sec
    info = ref.info()
    info.update(value=v, unit=UNIT)
    ref.close()
    print(json.dumps({"impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": world,
                      "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True,
                      "scaling": "strong", "vs_baseline": None, "dtype": "int8 x u4 -> int32 (AVX2), fp32 down",
                      "data": "synthetic", "config": config_block(cfg, 1), "cpu_baseline": info,
                      "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
def run_ours(args, cfg, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    from ffn_residual_mesh_b200.engine import LayerSpec
    from ffn_residual_mesh_b200.graphs import StepGraph
    from ffn_residual_mesh_b200.shard import ShardedFfnStack

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    stack = ShardedFfnStack(cfg.d_model, cfg.d_ff, cfg.residual_bits, cfg.layers, max(cfg.tokens),
                            cfg.base_tile_rows, rank=rank, world=world, device=local_rank)
    F = stack.d_ff
    mesh = stack.mesh
    t_setup = time.perf_counter()
    for l in range(cfg.layers):
        L = synth.make_layer_device(1000 + l, cfg.d_ff, cfg.d_model, rows=stack.rows, device=dev)
        mesh.load_layer(l, LayerSpec(L.gate_codes, L.up_codes, L.gate_alpha, L.up_alpha, L.down,
                                     L.gate_beta, L.up_beta, keep_fallback=True))
    # Per (batch, layer) inputs. The host base sums are the exact unsplit projection
    # (fallback path, all tiles flagged) minus the residual: g_base + g_res = g.
    n_tiles = -(-F // cfg.base_tile_rows)
    all_tiles = torch.ones(n_tiles, dtype=torch.uint8, device=dev)
    inputs = {}
    for T in cfg.tokens:
        for l in range(cfg.layers):
            _, z, s = synth.make_activations(7000 + 100 * l + T, T, cfg.d_model)
            zd, sd = torch.from_numpy(z).to(dev), torch.from_numpy(s).to(dev)
            full_g, full_u = torch.empty(T, F, device=dev), torch.empty(T, F, device=dev)
            res_g, res_u = torch.empty_like(full_g), torch.empty_like(full_g)
            mesh.residual(l, zd, sd, full_g, full_u, fallback_tiles=all_tiles)
            mesh.residual(l, zd, sd, res_g, res_u)
            gb, ub = full_g - res_g, full_u - res_u
            host = {k: v.cpu().pin_memory() for k, v in (("z", zd), ("s", sd), ("gb", gb), ("ub", ub))}
            host["y16"] = torch.empty(T, cfg.d_model, dtype=torch.float16).pin_memory()
            inputs[(T, l)] = {"z": zd, "s": sd, "gb": gb, "ub": ub,
                              "y16": torch.empty(T, cfg.d_model, dtype=torch.float16, device=dev), "host": host}
    torch.cuda.synchronize()
    setup_s = time.perf_counter() - t_setup
    staging = stack.staging(dev) if world > 1 else None

    def step_device():
        for T in cfg.tokens:
            for l in range(cfg.layers):
                b = inputs[(T, l)]
                stack.forward(l, b["z"], b["s"], b["gb"], b["ub"], b["y16"])

    def step_e2e():
        for T in cfg.tokens:
            for l in range(cfg.layers):
                h = inputs[(T, l)]["host"]
                stack.forward_host(l, h["z"], h["s"], h["gb"], h["ub"], h["y16"], staging=staging)

    def timed(fn, steps):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(steps):
            fn()
        stop.record()
        torch.cuda.synchronize()
        ms = start.elapsed_time(stop)
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
            dist.barrier()
        return ms

    # NCCL collectives are captured with the kernels (all ranks capture the same calls, after
    # an eager warm-up has created the communicators); graphs are released before the process
    # group is destroyed.
    use_graphs = not args.eager
    launches0 = mesh.launches
    step_device()
    torch.cuda.synchronize()
    launches_per_step = mesh.launches - launches0
    if use_graphs:
        g_dev, g_e2e = StepGraph(step_device), StepGraph(step_e2e)
        run_dev, run_e2e = g_dev.replay, g_e2e.replay
    else:
        run_dev, run_e2e = step_device, step_e2e

    clocks = ClockSampler(local_rank)
    clocks.start()
    dev_ms = timed(run_dev, args.steps)
    clock_info = clocks.stop()
    e2e_ms = timed(run_e2e, args.steps)
    eager_ms = timed(step_device, args.steps) if use_graphs else dev_ms
    eager_e2e_ms = timed(step_e2e, args.steps) if use_graphs else e2e_ms

    # Per-kernel device time over K steps: CUDA events recorded around each launch on the
    # launching stream (captured as graph nodes when graphs are used).
    mesh.profile(True)
    prof = {"residual": [0.0, 0], "down": [0.0, 0]}
    if use_graphs:
        g_prof = StepGraph(step_device, warmup=0)
        for _ in range(args.steps):
            g_prof.replay()
            for k, (ms, n) in mesh.profile_read().items():
                if k in prof:
                    prof[k][0] += ms
                    prof[k][1] += n
        g_prof.close()
    else:
        for _ in range(args.steps):
            step_device()
        for k, (ms, n) in mesh.profile_read().items():
            if k in prof:
                prof[k] = [ms, n]
    mesh.profile(False)
    launches = launches_per_step * args.steps

    res_bytes_layer, down_bytes_layer = mesh.layer_bytes(0)
    D, G = cfg.d_model, cfg.d_model // 32
    tfile = ROOT / "profiles" / "traffic.json"
    traffic_table = json.loads(tfile.read_text()) if tfile.exists() else {}
    pfile = ROOT / "MEASURED_PEAKS.json"
    peaks_all = json.loads(pfile.read_text()) if pfile.exists() else {}

    def alg_bytes(T):
        # residual: codes + alpha, activations and scales, both base sums in, h (fp16 hi + lo) out;
        # down: fp16 down weight, h (hi + lo) in, y (fp16) out
        return {"residual": res_bytes_layer + T * D + T * G * 4 + 2 * T * F * 4 + T * F * 4,
                "down": down_bytes_layer + T * F * 4 + T * D * 2}

    per_batch = {}
    for T in cfg.tokens:
        def one_batch(T=T):
            for l in range(cfg.layers):
                b = inputs[(T, l)]
                stack.forward(l, b["z"], b["s"], b["gb"], b["ub"], b["y16"])
        runner = StepGraph(one_batch) if use_graphs else None
        ms_b = timed(runner.replay if runner else one_batch, args.steps)
        per_batch[str(T)] = {"ms_per_stack": ms_b / args.steps, "tokens_per_s": T * args.steps / (ms_b / 1e3),
                             "us_per_layer": 1e3 * ms_b / args.steps / cfg.layers}
        if runner:
            runner.close()

        def one_batch_e2e(T=T):
            for l in range(cfg.layers):
                h = inputs[(T, l)]["host"]
                stack.forward_host(l, h["z"], h["s"], h["gb"], h["ub"], h["y16"], staging=staging)
        runner = StepGraph(one_batch_e2e) if use_graphs else None
        ms_e = timed(runner.replay if runner else one_batch_e2e, args.steps)
        per_batch[str(T)]["e2e_us_per_layer"] = 1e3 * ms_e / args.steps / cfg.layers
        if runner:
            runner.close()
        # per-kernel device time for this batch size alone
        mesh.profile(True)
        pk = {"residual": [0.0, 0], "down": [0.0, 0]}
        g_b = StepGraph(one_batch, warmup=0) if use_graphs else None
        for _ in range(args.steps):
            g_b.replay() if g_b else one_batch()
            if g_b:
                for k, (ms, n) in mesh.profile_read().items():
                    if k in pk:
                        pk[k][0] += ms
                        pk[k][1] += n
        if not g_b:
            for k, (ms, n) in mesh.profile_read().items():
                if k in pk:
                    pk[k] = [ms, n]
        else:
            g_b.close()
        mesh.profile(False)
        ab = alg_bytes(T)
        for k, (ms, n) in pk.items():
            if n:
                us = 1e3 * ms / n
                e = {"us_per_launch": us, "achieved_gbs": ab[k] / (us * 1e-6) / 1e9,
                     "dram_bytes_per_launch": traffic_table.get(f"{k}:{cfg.key}:T{T}")}
                if k == "residual" and T > 4:
                    # int8 tensor-core work of the exact group dots: 2 x (2 F) x D x T ops
                    ops = 2.0 * 2 * F * D * T
                    e["int8_tops"] = ops / (us * 1e-6) / 1e12
                    e["int8_frac_of_2x_measured_bf16"] = e["int8_tops"] / (2 * peaks_all.get("bf16_tflops", 1590.0))
                per_batch[str(T)][k] = e
    if use_graphs:
        g_dev.close()
        g_e2e.close()
    mesh.check_device_error()

    tokens_step = sum(cfg.tokens)
    value = tokens_step * args.steps / (dev_ms / 1e3)
    e2e_value = tokens_step * args.steps / (e2e_ms / 1e3)

    # roofline: algorithmic bytes per launch / live CUDA-event time per launch
    alg = {"residual": 0, "down": 0}
    for T in cfg.tokens:
        for k, v in alg_bytes(T).items():
            alg[k] += cfg.layers * v
    alg = {k: v * args.steps for k, v in alg.items()}
    peak, peak_kind = peaks()
    kern = {}
    for k, (ms, n) in prof.items():
        if n:
            kern[k] = {"ms_total": ms, "launches": n, "achieved_gbs": alg[k] / (ms / 1e3) / 1e9 if ms else None,
                       "us_per_launch": 1e3 * ms / n}
    dom = max(kern, key=lambda k: kern[k]["ms_total"])
    # DRAM bytes per launch of the dominant kernel, averaged over the step's batch sizes
    # (each batch size launches it once per layer) from the per-batch ncu captures
    per_t = [traffic_table.get(f"{dom}:{cfg.key}:T{T}") for T in cfg.tokens]
    traffic = sum(per_t) / len(per_t) if all(v is not None for v in per_t) else None
    achieved = kern[dom]["achieved_gbs"]
    roofline = {"bound": "hbm", "kernel": dom, "achieved": achieved, "peak": peak, "unit": "GB/s",
                "frac": achieved / peak, "peak_source": peak_kind, "traffic": traffic,
                "bytes_per_launch": alg[dom] / kern[dom]["launches"],
                "ms_per_launch": kern[dom]["ms_total"] / kern[dom]["launches"]}
    residual_kernel = None
    if "residual" in kern:
        residual_kernel = {"achieved_gbs": kern["residual"]["achieved_gbs"], "peak_gbs": peak,
                           "frac": kern["residual"]["achieved_gbs"] / peak,
                           "ms_per_launch": kern["residual"]["ms_total"] / kern["residual"]["launches"]}


    h2d = sum(cfg.layers * (T * D + T * G * 4 + 2 * T * F * 4) for T in cfg.tokens)
    d2h = sum(cfg.layers * T * D * 2 for T in cfg.tokens)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            ref = CpuReference(cfg, layers_sample=2)
            sec = min(ref.step_seconds() for _ in range(3))
            cpu = ref.info()
            cpu.update(value=tokens_step / sec, unit=UNIT)
            ref.close()
        except Exception as exc:  # the baseline is reported, never required
            cpu = {"value": None, "unit": UNIT, "error": str(exc)[:200]}
    if rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": dev_ms / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None,
            "dtype": "int8 x u2 -> int32 residual, fp16 x fp32 down", "data": "synthetic",
            "config": config_block(cfg, world),
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d * world,
                    "d2h_bytes_per_step": d2h * world, "ms_per_step": e2e_ms / args.steps,
                    "path": "ShardedFfnStack.forward_host -> ffnrm_ffn_forward_host"
                            + (" (CUDA graph replay)" if use_graphs else ""),
                    "eager_value": tokens_step * args.steps / (eager_e2e_ms / 1e3)},
            "eager_value": tokens_step * args.steps / (eager_ms / 1e3), "cuda_graphs": use_graphs,
            "roofline": roofline, "residual_kernel": residual_kernel, "kernels": kern, "per_batch": per_batch,
            "cpu_baseline": cpu, "gpu_launches": launches, "clocks": clock_info,
            "setup_s": round(setup_s, 1),
        }))
    stack.close()


def main():
    args = parse()
    cfg = synth.CONFIGS[args.workload]
    if args.layers or args.tokens:
        import dataclasses
        cfg = dataclasses.replace(cfg, layers=args.layers or cfg.layers,
                                  tokens=tuple(int(t) for t in args.tokens.split(",")) if args.tokens else cfg.tokens)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.gpus != world and world != 1:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    if args.impl == "reference":
        run_reference(args, cfg, rank, world)
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    try:
        run_ours(args, cfg, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
