#!/usr/bin/env python
"""pi0.5 engine benchmark (one JSON line on rank 0).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--workload bs64|bs1|denoise|sweep] [--impl ours|reference]

Workloads (seeded synthetic weights and inputs; the reference measured on its own robot data, which is
not available, so random tensors of the same shapes stand in):
  bs64     batched inference of 64 independent environments (64/N per GPU, no collective): chunks/s.
           Also reports the bs1 chunk latency p50 (ms) at N=1.  This is the default.
  bs1      full inference of one chunk (SigLIP, Gemma-2B prefill, 10-step denoise): p50 latency (ms)
  denoise  expert-only 10-step denoise over a 968-token N(0,1) bf16 prefix cache: p50 latency (ms)
  sweep    hot-operator sweep (GEMM shapes x M, attention); prints one line per operator

A step is one call of the engine's public entry point over one batch: pi05_infer (prefill + denoise)
for bs64/bs1, pi05_denoise for the expert-only workload.  `value` uses inputs already resident in
HBM; `e2e` makes the same call with pinned host buffers (host->device copies of images, tokens and
noise and the device->host read of the actions inside the timed region).
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "behavior-2026_b200"))

METRIC = "pi0.5 p50 chunk latency (bs1, ms); action chunks/s at bs64 on 1/2/4/8 B200"
MODEL = "pi0.5: SigLIP So400m/14 (27 layers) + Gemma-2B prefix (18 layers) + Gemma-300M action expert (18 layers)"


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d.get("hbm_gbs", 6650.0), d.get("bf16_tflops", 1590.0), d.get("bf16_tflops_sustained", 1400.0), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


def profiled_traffic(key):
    """DRAM bytes per launch from a committed ncu summary (profiles/roofline_traffic.txt: `key bytes`)."""
    p = os.path.join(ROOT, "profiles", "roofline_traffic.txt")
    if not os.path.exists(p):
        return None
    for line in open(p):
        f = line.split()
        if len(f) >= 2 and f[0] == key:
            try:
                return float(f[1])
            except ValueError:
                return None
    return None


class ClockSampler:
    """nvidia-smi samples (SM clock, throttle reasons) of one GPU during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu):
        self.gpu = gpu
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(2)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def dist_setup(n_gpus):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(local)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x, world):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def timed(eng, fn, steps):
    """Run fn() `steps` times between CUDA events on the engine stream; returns (total_ms, per-step ms)."""
    import torch
    s = torch.cuda.ExternalStream(eng.stream)
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    evs[0].record(s)
    for i in range(steps):
        fn()
        evs[i + 1].record(s)
    torch.cuda.synchronize()
    per = [evs[i].elapsed_time(evs[i + 1]) for i in range(steps)]
    return evs[0].elapsed_time(evs[-1]), per


# ---------------------------------------------------------------- CPU baseline (the oracle, rank 0 only)
def cpu_chunk_seconds(depth_full=True):
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    O.build()
    cfg = O.Config.make() if depth_full else O.Config.make(siglip_layers=1, gemma_layers=1, num_steps=1)
    img, tok, noise = O.gen_images(0, 0), O.gen_tokens(0, 0), O.gen_noise(0, 0)
    t = time.perf_counter()
    O.infer(cfg, 0, img, tok, noise)
    return time.perf_counter() - t, O.lib().p5o_threads()


def cpu_denoise_seconds():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    O.build()
    cfg = O.Config.make()
    k, v = O.gen_kv_cache(0, 0, 18, 968)
    noise = O.gen_noise(0, 0)
    t = time.perf_counter()
    O.denoise(cfg, 0, k, v, noise)
    return time.perf_counter() - t, O.lib().p5o_threads()


def run_reference(args, world, rank):
    """The CPU implementation of the path (the oracle, all host threads) on the same workload."""
    if rank != 0:
        return 0
    steps = min(args.steps, 5)  # one full-depth chunk per step (tens of seconds each)
    warm = 1 if args.warmup > 0 else 0
    if args.workload == "lora":
        steps = min(args.steps, 2)
        ts, cores = [], 1
        for _ in range(steps):
            t, cores = cpu_lora_sample_seconds()
            ts.append(t)
        v = 1.0 / statistics.median(ts)
        line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "samples/s", "n_gpus": args.gpus,
                "steps": steps, "steps_requested": args.steps, "warmup": 0, "ms_per_step": statistics.median(ts) * 1e3,
                "higher_is_better": True, "dtype": "f32", "data": "synthetic", "config": config_for(args, world),
                "cpu_baseline": {"value": v, "unit": "samples/s", "cores": cores, "kind": "port",
                                 "sample": "one full-depth sample per step: fp32 torch-CPU loss + autograd"},
                "e2e": {"value": v, "unit": "samples/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return 0
    if args.workload == "denoise":
        fn, unit = cpu_denoise_seconds, "ms"
    else:
        fn, unit = cpu_chunk_seconds, ("ms" if args.workload == "bs1" else "chunks/s")
    for _ in range(warm):
        fn() if args.workload == "denoise" else cpu_chunk_seconds(depth_full=False)
    ts, cores = [], 1
    for _ in range(steps):
        t, cores = fn()
        ts.append(t)
    p50 = statistics.median(ts)
    if unit == "ms":
        value, hib = p50 * 1e3, False
    else:
        value, hib = 1.0 / p50, True
    sample = ("one full-depth chunk per step (SigLIP 27 + Gemma 18 + 10-step denoise), bs1"
              if args.workload != "denoise" else "one 10-step expert denoise per step")
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": unit, "n_gpus": args.gpus,
            "steps": steps, "steps_requested": args.steps, "warmup": warm, "ms_per_step": p50 * 1e3,
            "higher_is_better": hib, "dtype": "f32", "data": "synthetic",
            "config": config_for(args, world),
            "cpu_baseline": {"value": value, "unit": unit, "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "fp32 C++ oracle of the same network (OpenMP); the reference engine's own code was deleted"}
    print(json.dumps(line), flush=True)
    return 0


def config_for(args, world):
    if args.workload == "lora":
        return {"workload": f"LoRA step: {args.lora_batch} samples per GPU", "model": MODEL,
                "global_batch": args.lora_batch * world, "parallelism": f"dp{world}"}
    if args.workload == "bs64":
        return {"workload": f"batched pi0.5 inference: {args.batch} independent environments "
                            f"({args.batch // world} per GPU), 3x224^2 images + 200 tokens -> 50x32 chunk, 10 steps",
                "model": MODEL, "global_batch": args.batch, "per_gpu_batch": args.batch // world,
                "prefix_tokens": 968, "action_chunk": [50, 32], "denoise_steps": 10, "parallelism": f"dp{world}",
                "l2": "no flush: every step streams 6.7 GB of weights and GBs of activations (> 126 MB L2)"}
    if args.workload == "bs1":
        return {"workload": "full pi0.5 inference bs1: 3x224^2 images + 200 tokens -> 50x32 chunk, 10 steps",
                "model": MODEL, "global_batch": 1, "prefix_tokens": 968, "parallelism": "replicas",
                "l2": "no flush: every step streams 6.7 GB of weights (> 126 MB L2)"}
    return {"workload": "action-expert denoise bs1: 18 layers, 10 Euler steps, 968-token N(0,1) bf16 prefix cache",
            "model": "Gemma-300M action expert (width 1024, MLP 4096, 8 heads / 1 KV head of 256)",
            "global_batch": 1, "parallelism": "replicas",
            "l2": "no flush: each step streams 623 MB of expert weights + 17.8 MB KV (> 126 MB L2)"}


# ---------------------------------------------------------------- our engine
# algorithmic bytes of one 10-step expert denoise: 311.4 M linear weights (bf16) + the 18-layer K/V cache
# of 968 tokens x 256 (bf16), read once per step
DENOISE_BYTES = 10 * (311.4e6 * 2 + 2 * 18 * 968 * 256 * 2)


def make_inputs(pn, n, first, seed=0):
    import numpy as np
    imgs = np.stack([pn.synth_images(seed, first + i) for i in range(n)])
    toks = np.stack([pn.synth_tokens(seed, first + i) for i in range(n)])
    noise = np.stack([pn.synth_noise(seed, first + i) for i in range(n)])
    return imgs, toks, noise


def gemm_roofline(pn, eng, M, N, K, epi, reps=5):
    """Time the dominant GEMM alone (CUDA events on the engine stream) at the workload's shape."""
    import torch
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.02).bfloat16()
    out = torch.empty(M, N // 2 if epi == "geglu" else N, device="cuda", dtype=torch.bfloat16)
    res = torch.randn(M, N, device="cuda", generator=g).bfloat16() if epi in ("resid", "gated") else None
    gate = torch.randn(N, device="cuda", generator=g).bfloat16() if epi == "gated" else None
    torch.cuda.synchronize()
    for _ in range(2):
        eng.op_linear(x, w, out, epi, res=res, gate=gate)
    total, per = timed(eng, lambda: eng.op_linear(x, w, out, epi, res=res, gate=gate), reps)
    ms = total / reps
    del x, w, out, res, gate
    torch.cuda.empty_cache()
    return ms


def run_ours(args, world, rank, local):
    import numpy as np
    import torch
    import pi05native as pn

    hbm, tf_burst, tf_sus, peak_src = peaks()
    if args.workload in ("bs64", "bs1"):
        nb = args.batch // world if args.workload == "bs64" else 1
        if args.workload == "bs64" and args.batch % world:
            raise SystemExit("batch must divide by the number of GPUs")
        eng = pn.Engine(pn.Config.make(), device=local, max_batch=nb)
        eng.init_random_weights(args.seed)
        imgs, toks, noise = make_inputs(pn, nb, rank * nb, args.seed)
        d_imgs = torch.from_numpy(imgs).cuda()
        d_toks = torch.from_numpy(toks).cuda()
        d_noise = torch.from_numpy(noise).cuda()
        d_out = torch.empty_like(d_noise)
        h_imgs = torch.from_numpy(imgs).pin_memory()
        h_toks = torch.from_numpy(toks).pin_memory()
        h_noise = torch.from_numpy(noise).pin_memory()
        h_out = torch.empty(noise.shape, dtype=torch.float32).pin_memory()
        step = lambda: eng.infer(d_imgs, d_toks, d_noise, out=d_out)
        step_e2e = lambda: eng.infer(h_imgs, h_toks, h_noise, out=h_out)
        h2d = imgs.nbytes + toks.nbytes + noise.nbytes
        d2h = noise.nbytes
        units = nb
    else:
        eng = pn.Engine(pn.Config.make(), device=local, max_batch=1)
        eng.init_random_weights(args.seed)
        eng.synth_prefix_cache(1, args.seed)
        noise = pn.synth_noise(args.seed, 0)[None]
        d_noise = torch.from_numpy(noise).cuda()
        d_out = torch.empty_like(d_noise)
        h_noise = torch.from_numpy(noise).pin_memory()
        h_out = torch.empty(noise.shape, dtype=torch.float32).pin_memory()
        step = lambda: eng.denoise(d_noise, out=d_out)
        step_e2e = lambda: eng.denoise(h_noise, out=h_out)
        h2d, d2h, units = noise.nbytes, noise.nbytes, 1

    for _ in range(args.warmup):
        step()
    for _ in range(max(1, args.warmup // 2)):
        step_e2e()
    eng.sync()
    launches = (max(0, eng.graph_launches("prefill", units)) if args.workload != "denoise" else 0) + \
        max(0, eng.graph_launches("denoise", units))

    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        total_ms, per = timed(eng, step, args.steps)
    barrier(world)
    total_ms = max_over_ranks(total_ms, world)
    torch.cuda.synchronize()
    total_e2e, per_e2e = timed(eng, step_e2e, args.steps)
    barrier(world)
    total_e2e = max_over_ranks(total_e2e, world)
    chunk = d_out.cpu().numpy()
    assert np.isfinite(chunk).all(), "non-finite actions"

    line = {"metric": METRIC, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": total_ms / args.steps, "dtype": "bf16", "data": "synthetic",
            "vs_baseline": None, "config": config_for(args, world), "gpu_launches": launches * args.steps,
            "kernels_per_step": launches, "clocks": clk.summary()}
    if args.workload == "bs64":
        all_units = units * world
        line.update({"value": all_units * args.steps / (total_ms / 1e3), "unit": "chunks/s",
                     "higher_is_better": True, "scaling": "strong",
                     "e2e": {"value": all_units * args.steps / (total_e2e / 1e3), "unit": "chunks/s",
                             "h2d_bytes_per_step": h2d * world, "d2h_bytes_per_step": d2h * world}})
    else:
        line.update({"value": statistics.median(per), "unit": "ms", "higher_is_better": False,
                     "scaling": "replicas",
                     "e2e": {"value": statistics.median(per_e2e), "unit": "ms", "h2d_bytes_per_step": h2d,
                             "d2h_bytes_per_step": d2h}})

    # bs1 latency beside the bs64 throughput (rank 0, single GPU run)
    if args.workload == "bs64" and world == 1 and not args.no_bs1:
        e1 = pn.Engine(pn.Config.make(), device=local, max_batch=1)
        e1.init_random_weights(args.seed)
        i1 = torch.from_numpy(imgs[:1].copy()).cuda()
        t1 = torch.from_numpy(toks[:1].copy()).cuda()
        n1 = torch.from_numpy(noise[:1].copy()).cuda()
        o1 = torch.empty_like(n1)
        for _ in range(args.warmup):
            e1.infer(i1, t1, n1, out=o1)
        e1.sync()
        _, per1 = timed(e1, lambda: e1.infer(i1, t1, n1, out=o1), max(args.steps, 5))
        line["bs1_p50_ms"] = statistics.median(per1)
        # the expert-only 10-step denoise (18 layers over a N(0,1) 968-token cache) and its HBM fraction
        e1.synth_prefix_cache(1, args.seed)
        for _ in range(args.warmup):
            e1.denoise(n1, out=o1)
        e1.sync()
        _, perd = timed(e1, lambda: e1.denoise(n1, out=o1), max(args.steps, 5))
        dms = statistics.median(perd)
        line["denoise_p50_ms"] = dms
        line["denoise_hbm_frac"] = DENOISE_BYTES / (dms / 1e3) / 1e9 / hbm
        e1.close()

    # roofline of the dominant kernel
    if args.workload in ("bs64", "bs1"):
        M = units * 968
        ms = gemm_roofline(pn, eng, M, 32768, 2048, "geglu")
        fl = 2.0 * M * 32768 * 2048
        ach = fl / (ms / 1e3) / 1e12
        tr = profiled_traffic(f"gemma_gate_up_M{M}")
        line["roofline"] = {"kernel": "gemm_pair_kernel<EPI_GEGLU> Gemma-2B gate/up + GeGLU epilogue (CTA pairs, cta_group::2)",
                            "shape": [M, 32768, 2048], "bound": "tensor", "achieved": ach, "peak": tf_burst,
                            "unit": "TFLOP/s", "frac": ach / tf_burst, "peak_source": f"{peak_src} bf16 burst",
                            "ms_per_launch": ms, "algorithmic_flops": fl, "traffic": tr}
    else:
        # the denoise is weight streaming: algorithmic bytes per 10-step call over its duration
        algo = DENOISE_BYTES
        ach = algo / (statistics.median(per) / 1e3) / 1e9
        line["roofline"] = {"kernel": "whole 10-step denoise (weight streaming)", "bound": "hbm", "achieved": ach,
                            "peak": hbm, "unit": "GB/s", "frac": ach / hbm, "peak_source": f"{peak_src} hbm",
                            "algorithmic_bytes": algo, "traffic": profiled_traffic("denoise_step")}

    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        if args.workload == "denoise":
            t, cores = cpu_denoise_seconds()
            line["cpu_baseline"] = {"value": t * 1e3, "unit": "ms", "cores": cores, "kind": "port",
                                    "sample": "one 10-step expert denoise (full depth), fp32 oracle"}
        else:
            t, cores = cpu_chunk_seconds()
            v = 1.0 / t if args.workload == "bs64" else t * 1e3
            line["cpu_baseline"] = {"value": v, "unit": "chunks/s" if args.workload == "bs64" else "ms",
                                    "cores": cores, "kind": "port",
                                    "sample": "one full-depth chunk (bs1), fp32 oracle; chunks/s = 1/time"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    eng.close()
    return 0


def run_sweep(args, local):
    """Config 5: skinny/large GEMMs and the 50-query attention, each against its roofline."""
    import torch
    import pi05native as pn
    hbm, tf_burst, _, src = peaks()
    eng = pn.Engine(pn.Config.make(siglip_layers=0, gemma_layers=1, num_steps=1), device=local, max_batch=1)
    shapes = [(1024, 4096), (4096, 1024), (1024, 2304), (2048, 16384), (16384, 2048)]
    for (K, N) in shapes:
        for M in (50, 100, 800, 3200):
            ms = eng.op_bench_linear(M, N, K, "store", reps=60) / 1e3  # graph-timed device time
            fl = 2.0 * M * N * K
            by = 2.0 * (K * N + M * K + M * N)
            if M <= 100:
                ach, peak, unit, bound = by / (ms / 1e3) / 1e9, hbm, "GB/s", "hbm"
            else:
                ach, peak, unit, bound = fl / (ms / 1e3) / 1e12, tf_burst, "TFLOP/s", "tensor"
            print(json.dumps({"op": "linear", "M": M, "K": K, "N": N, "ms": ms, "bound": bound, "achieved": ach,
                              "unit": unit, "peak": peak, "frac": ach / peak, "peak_source": src}), flush=True)
    for S in (968, 1536, 2048):
        q = (torch.randn(1, 50, 2560, device="cuda") * 0.1).bfloat16()
        k = torch.randn(1, S, 256, device="cuda").bfloat16()
        v = torch.randn(1, S, 256, device="cuda").bfloat16()
        o = torch.empty(1, 50, 2048, device="cuda", dtype=torch.bfloat16)
        for _ in range(3):
            eng.op_attention(q, k, v, o, 8)
        total, _ = timed(eng, lambda: eng.op_attention(q, k, v, o, 8), 50)
        ms = total / 50
        by = 2.0 * (2 * S * 256 + 50 * 2560 + 50 * 2048)
        print(json.dumps({"op": "attention_mqa_50q", "S": S, "ms": ms, "bound": "hbm",
                          "achieved": by / (ms / 1e3) / 1e9, "unit": "GB/s", "peak": hbm,
                          "frac": by / (ms / 1e3) / 1e9 / hbm, "flops": 4.0 * 50 * 8 * 256 * S}), flush=True)
    eng.close()
    return 0


def run_sigattn(args, local):
    """SigLIP attention by image count on both kernels (tcgen05 and mma.sync, PI05_ATTN_TC): the measurement
    behind the engine's choice of kernel per image count.  Device time per launch over 20 launches."""
    import torch
    import pi05native as pn
    for tc in ("1", "0"):
        os.environ["PI05_ATTN_TC"] = tc  # read when the engine is created
        eng = pn.Engine(pn.Config.make(siglip_layers=1, gemma_layers=1, num_steps=1), device=local, max_batch=1)
        for images in (3, 6, 12, 24, 48, 96, 192):
            qkv = torch.randn(images * 256, 3456, device="cuda").bfloat16()
            out = torch.empty(images * 256, 1152, device="cuda", dtype=torch.bfloat16)
            torch.cuda.synchronize()
            for _ in range(3):
                eng.op_siglip_attention(qkv, out)
            total, _ = timed(eng, lambda: eng.op_siglip_attention(qkv, out), 20)
            fl = 4.0 * images * 16 * 256 * 256 * 72
            print(json.dumps({"op": "siglip_attention", "kernel": "tcgen05" if tc == "1" else "mma.sync",
                              "images": images, "us": total / 20 * 1e3,
                              "tflops": fl / (total / 20 / 1e3) / 1e12}), flush=True)
        eng.close()
    os.environ.pop("PI05_ATTN_TC", None)
    return 0


# ---------------------------------------------------------------- LoRA train step (config 4)
LORA_TFLOP_PER_SAMPLE = None  # filled by lora_flops_per_sample()


def lora_flops_per_sample(P=968, H=50, L=18):
    """Algorithmic FLOPs of one sample of the LoRA step: SigLIP forward, Gemma/expert forward, the
    dX backward through the frozen linears (no frozen dW), attention forward + backward (the backward
    recomputes S in each of its three kernels: 8 matmuls), LoRA projections and gradients."""
    gem = 2048 * 2560 + 2048 * 2048 + 2048 * 32768 + 16384 * 2048
    exp = 1024 * 2560 + 2048 * 1024 + 1024 * 8192 + 4096 * 1024
    sig_lin = 27 * (1152 * 3456 + 1152 * 1152 + 2 * 1152 * 4304) * 768 * 2 + 768 * (588 * 1152 + 1152 * 2048) * 2
    sig_att = 27 * 3 * 4 * 256 * 256 * 1152
    gem_fwd = 2 * P * (gem * (L - 1) + 2048 * 2560)
    exp_fwd = 2 * H * exp * L
    att = (L - 1) * 4 * P * P * 256 * 8 + L * 4 * H * (P + H) * 256 * 8
    lora_cols = 16 * 2 * (L * (3 * 2048 + 2048 + 2 * 2048 + 16384) * P + L * (3 * 1024 + 2048 + 2 * 1024 + 4096) * H)
    return sig_lin + sig_att + 2 * (gem_fwd + exp_fwd) + att * (1 + 4) + 3 * lora_cols


def lora_inputs(pn, nb, first, seed):
    import numpy as np
    imgs = np.stack([pn.synth_images(seed, first + i) for i in range(nb)])
    toks = np.stack([pn.synth_tokens(seed, first + i) for i in range(nb)])
    acts = np.stack([pn.synth_noise(seed + 101, first + i) for i in range(nb)])
    noise = np.stack([pn.synth_noise(seed + 202, first + i) for i in range(nb)])
    rng = np.random.default_rng(seed * 7919 + first)
    t = (rng.beta(1.5, 1.0, nb) * 0.999 + 0.001).astype(np.float32)
    return imgs, toks, acts, noise, t


def cpu_lora_sample_seconds():
    """fp32 torch-CPU autograd of the full-depth loss for one sample (the oracle of the LoRA step)"""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import numpy as np
    import oracle as O
    import lora_ref
    import pi05native as pn
    O.build()
    cfg = O.Config.make()
    imgs, toks, acts, noise, t = lora_inputs(pn, 1, 0, 0)
    n = sum(a * b for _, (a, b) in lora_ref.lora_layout(cfg.gemma_layers))
    p0 = O.gen_normal(5, 80, 0, (n,), 0.01, True)
    import torch
    t0 = time.perf_counter()
    emb = O.prefix_embed(cfg, 0, imgs[0], toks[0])[None]  # frozen SigLIP forward: part of the work
    t1 = time.perf_counter()
    ref = lora_ref.LoraRef(cfg, 0, p0)  # generating the frozen weights is set-up, not work
    t2 = time.perf_counter()
    ref.loss(emb, acts, noise, t).backward()
    t3 = time.perf_counter()
    return (t1 - t0) + (t3 - t2), torch.get_num_threads()


def run_lora(args, world, rank, local):
    import numpy as np
    import torch
    import dp
    import pi05native as pn

    hbm, tf_burst, tf_sus, peak_src = peaks()
    nb = args.lora_batch
    mb = min(args.micro_batch, nb)  # no larger than the per-GPU batch
    eng = pn.Engine(pn.Config.make(), device=local, max_batch=mb)
    eng.init_random_weights(args.seed)
    eng.lora_init(seed=args.seed + 1, micro_batch=mb)
    dp.attach_nccl(eng, rank, world)  # the engine's own communicator: per-layer averages during backward
    first, _ = dp.shard(nb * world, world, rank)
    imgs, toks, acts, noise, t = lora_inputs(pn, nb, first, args.seed)
    dev = [torch.from_numpy(a).cuda() for a in (imgs, toks, acts, noise, t)]
    host = [torch.from_numpy(a).pin_memory() for a in (imgs, toks, acts, noise, t)]

    def step(bufs):
        # zero + forward/backward (each finished layer's gradients averaged over the ranks on the engine's
        # communication stream) + clip/AdamW; the loss is read back to the host
        return eng.lora_step(*bufs)

    for _ in range(args.warmup):
        step(dev)
    eng.sync()
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        total_ms, per = timed(eng, lambda: step(dev), args.steps)
    barrier(world)
    total_ms = max_over_ranks(total_ms, world)
    total_e2e, _ = timed(eng, lambda: step(host), args.steps)
    barrier(world)
    total_e2e = max_over_ranks(total_e2e, world)
    loss = step(dev)
    assert np.isfinite(loss)
    samples = nb * world
    fl = lora_flops_per_sample() * nb
    ach = fl / (total_ms / args.steps / 1e3) / 1e12
    line = {"metric": METRIC, "value": samples * args.steps / (total_ms / 1e3), "unit": "samples/s",
            "higher_is_better": True, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": total_ms / args.steps, "lora_steps_per_s": args.steps / (total_ms / 1e3),
            "scaling": "weak", "dtype": "bf16", "data": "synthetic", "vs_baseline": None, "loss": loss,
            "config": {"workload": f"LoRA step (rank 16, alpha 32, q/k/v/o/gate/up/down of Gemma-2B and the expert): "
                                   f"{nb} samples per GPU, micro-batch {mb}, flow-matching loss, "
                                   f"AdamW lr 1e-4" + (", NCCL gradient average per layer, overlapped with the "
                                                       f"backward pass" if world > 1 else ""),
                       "model": MODEL, "global_batch": samples, "per_gpu_batch": nb, "parallelism": f"dp{world}",
                       "l2": "no flush: every step streams GBs of weights and saved activations (> 126 MB L2)"},
            "e2e": {"value": samples * args.steps / (total_e2e / 1e3), "unit": "samples/s",
                    "h2d_bytes_per_step": sum(a.nbytes for a in (imgs, toks, acts, noise, t)), "d2h_bytes_per_step": 4},
            "roofline": {"kernel": "whole LoRA step (tcgen05 GEMMs + attention fwd/bwd)", "bound": "tensor",
                         "achieved": ach, "peak": tf_sus, "unit": "TFLOP/s", "frac": ach / tf_sus,
                         "peak_source": f"{peak_src} bf16 sustained", "algorithmic_flops_per_step": fl,
                         "traffic": None},
            "clocks": clk.summary()}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        ts, th = cpu_lora_sample_seconds()
        line["cpu_baseline"] = {"value": 1.0 / ts, "unit": "samples/s", "cores": th, "kind": "port",
                                "sample": "one full-depth sample: fp32 torch-CPU forward + autograd backward of the loss"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    eng.close()
    return 0


def run_gemm(args, local):
    """One linear layer M x N x K (`--gemm M,N,K`, epilogue `--epi`), timed with CUDA events: the small,
    self-contained case the kernel profiles are captured on."""
    import pi05native as pn
    M, N, K = (int(v) for v in args.gemm.split(","))
    hbm, tf_burst, _, src = peaks()
    eng = pn.Engine(pn.Config.make(siglip_layers=0, gemma_layers=1, num_steps=1), device=local, max_batch=1)
    ms = gemm_roofline(pn, eng, M, N, K, args.epi, reps=max(1, args.steps))
    fl = 2.0 * M * N * K
    print(json.dumps({"op": "linear", "epi": args.epi, "M": M, "N": N, "K": K, "ms": ms,
                      "tflops": fl / (ms / 1e3) / 1e12, "frac": fl / (ms / 1e3) / 1e12 / tf_burst,
                      "peak": tf_burst, "peak_source": src}), flush=True)
    eng.close()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="bs64", choices=["bs64", "bs1", "denoise", "sweep", "gemm", "lora", "sigattn"])
    ap.add_argument("--lora-batch", type=int, default=32, help="samples per GPU per LoRA step")
    ap.add_argument("--micro-batch", type=int, default=32,
                    help="samples per LoRA forward/backward pass (measured on B200: one 32-sample pass 86.0 "
                         "samples/s, four 8-sample passes 76.3)")
    ap.add_argument("--gemm", default="7744,32768,2048", help="M,N,K for --workload gemm")
    ap.add_argument("--epi", default="geglu", help="epilogue for --workload gemm")
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-bs1", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3) if args.impl == "ours" else args.warmup
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, world, rank)
    world, rank, local = dist_setup(args.gpus)
    try:
        if args.workload == "sweep":
            return run_sweep(args, local) if rank == 0 else 0
        if args.workload == "gemm":
            return run_gemm(args, local) if rank == 0 else 0
        if args.workload == "sigattn":
            return run_sigattn(args, local) if rank == 0 else 0
        if args.workload == "lora":
            return run_lora(args, world, rank, local)
        return run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
