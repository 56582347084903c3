#!/usr/bin/env python
"""Benchmark of the denoise-step hot path on B200.

Workload: image DiT at 1024x1024, 4096 image + 512 text tokens, hidden 3072,
24 x 128 heads, 8 double-stream + 24 single-stream blocks, GELU-tanh MLP x4, flow-matching
Euler with sigmas linearly spaced 1 -> 0 over 4 steps, bf16, random-init weights (seed 42),
N(0, 1) latents (seed 43) and text (seed 44). A "step" is one transformer evaluation plus the
Euler update (fused into the last projection). Weights (9.4 GB) stream through HBM every step,
far more than the 126 MB L2, so no explicit L2 flush is needed between timed steps.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl kino|reference]

--impl reference times the reference's CPU path for the same workload: the reference (MLX,
Python >= 3.15) cannot run on this box, so that arm times the CPU restatement of its formulas
(oracle/) on all host cores, one double + one single block per step, extrapolated x8 / x24.
With N > 1 (torchrun) the same step runs with Ulysses sequence parallelism: each rank holds
1/N of the text and image tokens; the q/k/v projection epilogues store each head group straight
into its owner GPU's buffer over NVLink and the attention stores its rows straight back (device
barriers between; strong scaling); the step time is the max over ranks.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

METRIC = "DiT denoise-step latency (ms)"
UNIT = "ms/step"
WORKLOAD = (
    "image DiT 1024x1024 (BASELINE config 2): 4096 image + 512 text tokens, hidden 3072, "
    "24x128 heads, 8 double + 24 single blocks, GELU-tanh MLP x4, 2D axial RoPE theta 10000, "
    "4-step linear-sigma flow-matching Euler, batch 1, no CFG"
)
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def log(msg: str) -> None:
    print(msg, file=sys.stderr, flush=True)


_RESULT_OUT = sys.stdout


def reserve_stdout() -> None:
    """Keep the process's stdout for the result line alone: file descriptor 1 and sys.stdout are
    pointed at stderr (libraries that print at the C level, NCCL's banner among them, land
    there), and the original stdout is kept for emit()."""
    global _RESULT_OUT
    sys.stdout.flush()
    saved = os.dup(1)
    os.dup2(2, 1)
    _RESULT_OUT = os.fdopen(saved, "w")
    sys.stdout = sys.stderr


def emit(obj: dict) -> None:
    """The one JSON result line."""
    _RESULT_OUT.write(json.dumps(obj) + "\n")
    _RESULT_OUT.flush()


def peaks() -> tuple[dict, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        return json.loads(path.read_text()), "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def step_flops(dim=3072, heads=24, nt=512, ni=4096, mlp=12288, double=8, single=24, cin=64):
    """Algorithmic FLOPs of one transformer evaluation (projections + attention)."""
    n = nt + ni
    d = dim
    dbl = 2 * n * (3 * d * d + d * d + 2 * d * mlp) + 4 * n * n * d
    sgl = 2 * n * (3 * d * d + d * mlp) + 2 * n * (d + mlp) * d + 4 * n * n * d
    io = 2 * ni * cin * d + 2 * ni * d * cin
    return double * dbl + single * sgl + io


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = (
        "index,clocks.sm,clocks.max.sm,utilization.gpu,power.draw,"
        "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
        "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"
    )

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.proc = None
        self.path = None

    def start(self) -> None:
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.gpu_index), "-f", self.path],
                stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL,
            )
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.3)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None

        loaded = [r for r in rows if (num(r[3]) or 0) >= 50] or rows
        sm = [num(r[1]) for r in loaded if num(r[1]) is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[j] for r in loaded for j in range(4) if r[5 + j] == "Active"})
        power = [num(r[4]) for r in loaded if num(r[4]) is not None]
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": num(rows[0][2]),
            "reasons": reasons,
            "samples": len(rows),
            "samples_under_load": len(loaded),
            "power_w_max": max(power) if power else None,
        }


# ----------------------------------------------------------------------------- distributed
def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world: int) -> None:
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(value: float, world: int) -> float:
    if world == 1:
        return value
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def physical_gpu(local: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [x for x in vis.split(",") if x.strip()]
        if local < len(ids) and ids[local].strip().isdigit():
            return int(ids[local])
    return local


# ----------------------------------------------------------------------------- CPU oracle sample
def config_dict() -> dict:
    """The workload description both arms print (the same keys and values)."""
    return {
        "workload": WORKLOAD,
        "l2": "no flush: 9.4 GB of weights stream per step, inputs exceed the 126 MB L2",
        "step_gflop": round(step_flops() / 1e9, 1),
    }


def cpu_sample_ms(threads: int) -> tuple[float, str, dict]:
    """One double + one single block of the workload on the CPU oracle, extrapolated to a step;
    also returns the measured parts in ms."""
    from oracle import flux2 as ref
    from kinomlx_b200.flux2 import config as fcfg
    from kinomlx_b200.synthetic import flux_weights, normal

    torch.set_num_threads(threads)
    v = fcfg.BASELINE.with_blocks(1, 1)
    w = flux_weights(v, seed=42)
    nt, ni = 512, 4096
    image = normal((1, ni, v.dim), seed=1)
    text = normal((1, nt, v.dim), seed=2)
    ids = torch.cat([torch.zeros((1, nt, 2), dtype=torch.int64), ref.image_ids(64, 64, 2)], 1)
    cos, sin = ref.rotary_positions(ids, v)
    t = torch.tensor([0.5], dtype=torch.bfloat16)
    with torch.inference_mode():
        t0 = time.perf_counter()
        emb = ref.timestep_embedding(w, t * 1000)
        im = ref.modulation(w, "double_stream_modulation_img", emb)
        tm = ref.modulation(w, "double_stream_modulation_txt", emb)
        sm = ref.modulation(w, "single_stream_modulation", emb)
        t1 = time.perf_counter()
        img, txt = ref.double_block(w, 0, image, text, im, tm, cos, sin, v)
        t2 = time.perf_counter()
        value = ref.single_block(w, 0, torch.cat([txt, img], 1), sm, cos, sin, v)
        t3 = time.perf_counter()
    ms = 1e3 * ((t1 - t0) + 8 * (t2 - t1) + 24 * (t3 - t2))
    del value
    sample = (
        "CPU oracle (torch, bf16 values, fp32 matmul): timestep MLP + modulations + 1 double "
        "block + 1 single block at 4096+512 tokens, extrapolated x8 double / x24 single"
    )
    parts = {"modulations_ms": round(1e3 * (t1 - t0), 1), "double_block_ms": round(1e3 * (t2 - t1), 1),
             "single_block_ms": round(1e3 * (t3 - t2), 1)}
    return ms, sample, parts


def run_reference(args, world: int, rank: int) -> None:
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    for _ in range(args.warmup):
        cpu_sample_ms(threads)
    samples = [cpu_sample_ms(threads) for _ in range(args.steps)]
    ms = statistics.mean(x[0] for x in samples)
    measured = {k: round(statistics.mean(x[2][k] for x in samples), 1) for k in samples[0][2]}
    sample = (
        "CPU restatement of the reference formulas (oracle/, torch CPU): per step 1 double + 1 "
        "single block at 4096+512 tokens, extrapolated x8 / x24 (the reference's MLX path needs "
        "macOS and Python >= 3.15 and cannot run on this box)"
    )
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(ms, 3),
        "unit": UNIT,
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 3),
        "higher_is_better": False,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic",
        "config": config_dict(),
        "cpu_baseline": {"value": round(ms, 3), "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": sample, "measured": measured,
                         "extrapolated": "value = modulations + 8 x double + 24 x single"},
        "e2e": {"value": round(ms, 3), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    emit(line)


# ----------------------------------------------------------------------------- GPU arm
def run_kino(args, world: int, rank: int, local: int) -> None:
    from kinomlx_b200 import ops
    from kinomlx_b200.flux2 import config as fcfg
    from kinomlx_b200.flux2 import sampling
    from kinomlx_b200.flux2.transformer import Flux2Transformer
    from kinomlx_b200.sequence_parallel import SequenceParallel
    from kinomlx_b200.synthetic import flux_weights, normal

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    v = fcfg.BASELINE
    nt, side = 512, 64
    ni = side * side
    weights = flux_weights(v, seed=42, device=device)
    # N > 1: Ulysses sequence parallelism over all ranks (strong scaling: the same step, its
    # tokens sharded, one all-to-all each way around every attention)
    # N > 1: Ulysses over the peer transport (q/k/v and attention rows cross NVLink inside the
    # projection and attention kernels)
    model = Flux2Transformer(weights, v, device,
                             sp=SequenceParallel(peer=True) if world > 1 else None)
    del weights
    torch.cuda.empty_cache()
    i0, i1 = model.sp.shard(ni)
    noise = normal((1, ni, v.in_channels), seed=43, device=device)[:, i0:i1].contiguous()
    text = normal((1, nt, v.context_dim), seed=44, device=device)
    ids = torch.zeros((1, nt + ni, 2), dtype=torch.int64)
    ids[0, nt:, 0] = torch.arange(side).repeat_interleave(side)
    ids[0, nt:, 1] = torch.arange(side).repeat(side)
    sigmas = sampling.linear_sigmas(4)
    prepared = model.prepare(text, ids)
    current = noise.clone()
    nsched = len(sigmas) - 1

    for i in range(args.warmup):
        sampling.denoise_step(model, prepared, current, sigmas, i % nsched)
    torch.cuda.synchronize()
    ops.device_status()

    # ---- timed region: K device-resident steps, nothing else on the stream
    sampler = ClockSampler(physical_gpu(local)) if rank == 0 else None
    barrier(world)
    torch.cuda.synchronize()
    if sampler:
        sampler.start()
    launches0 = ops.launches
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for i in range(args.steps):
        sampling.denoise_step(model, prepared, current, sigmas, i % nsched)
    end.record()
    torch.cuda.synchronize()
    launches = ops.launches - launches0
    barrier(world)
    clocks = sampler.stop() if sampler else None
    ms = max_over_ranks(start.elapsed_time(end) / args.steps, world)
    ops.device_status()
    if not bool(torch.isfinite(current).all()):
        raise FloatingPointError("non-finite latent in the benchmark")

    # ---- the same K steps again with CUDA events around every launch (per-kernel durations on
    # the launching stream); kept out of the timed region because the events add ~3% gaps
    launch_log = ops.LaunchLog()
    ops.set_launch_log(launch_log)
    for i in range(args.steps):
        sampling.denoise_step(model, prepared, current, sigmas, i % nsched)
    torch.cuda.synchronize()
    ops.set_launch_log(None)

    # ---- e2e: the public step API with pinned host input/output copies inside the region
    host_in = noise.cpu().pin_memory()
    host_out = torch.empty_like(host_in).pin_memory()
    dev_cur = torch.empty_like(noise)
    barrier(world)
    torch.cuda.synchronize()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record()
    for i in range(args.steps):
        dev_cur.copy_(host_in, non_blocking=True)
        sampling.denoise_step(model, prepared, dev_cur, sigmas, i % nsched)
        host_out.copy_(dev_cur, non_blocking=True)
    e_end.record()
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e_start.elapsed_time(e_end) / args.steps, world)
    io_bytes = host_in.numel() * host_in.element_size()

    # ---- roofline of the dominant kernel class inside the timed region
    summary = launch_log.summary()
    total_ms = sum(s["ms"] for s in summary.values()) or 1.0
    kernels = {
        k: {"launches": int(s["launches"]), "ms": round(s["ms"], 3),
            "share": round(s["ms"] / total_ms, 4),
            "tflops": round(s["flops"] / (s["ms"] * 1e9), 1) if s["flops"] else None,
            "gbs": round(s["bytes"] / (s["ms"] * 1e6), 1) if s["bytes"] else None}
        for k, s in sorted(summary.items(), key=lambda kv: -kv[1]["ms"])
    }
    dom = max(summary, key=lambda k: summary[k]["ms"])
    pk, source = peaks()
    d = summary[dom]
    if d["flops"]:
        achieved = d["flops"] / (d["ms"] * 1e9)  # TFLOP/s
        peak = float(pk.get("bf16_tflops_sustained", pk.get("bf16_tflops")))
        bound, unit = "tensor", "TFLOP/s"
        per_launch_flops = d["flops"] / d["launches"]
    else:
        achieved = d["bytes"] / (d["ms"] * 1e6)
        peak = float(pk["hbm_gbs"])
        bound, unit = "hbm", "GB/s"
        per_launch_flops = None
    # DRAM bytes of one launch of the kernel class from an ncu capture: "<class> <read+write
    # bytes> <algorithmic bytes of that launch> <which launch>"
    traffic = traffic_alg = traffic_launch = None
    tf = ROOT / "profiles" / "traffic.txt"
    if tf.exists():
        for line in tf.read_text().splitlines():
            parts = line.split(maxsplit=3)
            if len(parts) >= 2 and parts[0] == dom:
                try:
                    traffic = float(parts[1])
                    traffic_alg = float(parts[2]) if len(parts) > 2 else None
                except ValueError:
                    traffic = traffic_alg = None
                traffic_launch = parts[3] if len(parts) > 3 else None
    roofline = {
        "kernel": dom,
        "bound": bound,
        "achieved": round(achieved, 1),
        "peak": peak,
        "unit": unit,
        "frac": round(achieved / peak, 4),
        "peak_source": f"{source} ({'sustained' if bound == 'tensor' else 'copy'})",
        "traffic": traffic,
        "traffic_launch": traffic_launch,
        "traffic_algorithmic_bytes": traffic_alg,
        "algorithmic_per_launch": per_launch_flops,
        "step_tflops": round(step_flops() / (ms * 1e9), 1),
        "timing": "per-launch CUDA events over a second pass of the same K steps",
    }
    if bound == "tensor":
        # the same achieved rate against the burst peak, and per MHz against the sustained
        # peak per MHz of the clock it was measured at (the bench and the peak run at different
        # clocks under the power cap)
        roofline["frac_of_burst"] = round(achieved / float(pk.get("bf16_tflops", peak)), 4)
        peak_mhz = (pk.get("clocks_under_load") or {}).get("sm_mhz_median")
        run_mhz = (clocks or {}).get("sm_mhz")
        if peak_mhz and run_mhz:
            roofline["frac_clock_normalised"] = round((achieved / run_mhz) / (peak / peak_mhz), 4)

    secondary = None
    model.sp.close()
    if not args.no_secondary:
        model = prepared = current = None
        torch.cuda.empty_cache()
        secondary = run_secondary(world, rank, local)

    cpu = None
    if world == 1 and rank == 0 and not args.no_cpu:
        threads = os.cpu_count() or 1
        cpu_sample_ms(threads)  # warm-up (allocator, thread pool)
        cms, sample, parts = cpu_sample_ms(threads)
        cpu = {"value": round(cms, 1), "unit": UNIT, "cores": threads, "kind": "port",
               "sample": sample, "measured": parts,
               "extrapolated": "value = modulations + 8 x double + 24 x single"}

    if rank == 0:
        line = {
            "metric": METRIC,
            "value": round(ms, 3),
            "unit": UNIT,
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms, 3),
            "higher_is_better": False,
            "scaling": "strong" if world > 1 else "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) latents and text, random-init N(0,0.02) weights)",
            "config": config_dict(),
            "parallelism": (f"ulysses sequence parallel x{world} (q/k/v and attention rows "
                            "exchanged over NVLink peer memory inside the projection and "
                            "attention kernels)") if world > 1 else "single GPU",
            "e2e": {"value": round(e2e_ms, 3), "unit": UNIT, "h2d_bytes_per_step": io_bytes,
                    "d2h_bytes_per_step": io_bytes},
            "roofline": roofline,
            "cpu_baseline": cpu,
            "gpu_launches": launches,
            "kernels": kernels,
            "clocks": clocks,
            "secondary": secondary,
        }
        emit(line)


def ltx_step_flops(tokens=9216, ctx=256, dim=4096, heads=32, blocks=48, ff=4, cin=128):
    """Algorithmic FLOPs of one LTX-2 video-stream transformer evaluation."""
    d = dim
    per = 2 * tokens * (4 * d * d + 2 * d * d + 2 * ff * d * d + 2 * heads * d) + 2 * ctx * 2 * d * d
    per += 4 * tokens * tokens * d + 4 * tokens * ctx * d
    return blocks * per + 2 * tokens * cin * d * 2


def vae_decode_flops(decoder, latent_shape, tile=8, overlap=2):
    """Conv FLOPs of the tiled decode (every tile, overlap included)."""
    from kinomlx_b200.ltx2.video_vae import tile_plan

    _, _, f, h, w = latent_shape
    total = 0
    for h0, h1, w0, w1, *_ in tile_plan(h, w, tile, overlap, decoder.spatial_scale):
        ff, hh, ww, c = f, h1 - h0, w1 - w0, decoder.v.top_width
        total += 2 * ff * hh * ww * c * 27 * decoder.v.latent_channels
        for blk in decoder.v.blocks:
            if blk[0] == "res":
                total += blk[1] * 2 * (2 * ff * hh * ww * c * 27 * c)
            else:
                (st, sh, sw), mult = blk[1], blk[2]
                n = st * sh * sw * (c // mult)
                total += 2 * ff * hh * ww * n * 27 * c
                ff, hh, ww, c = ff * st - (1 if st > 1 else 0), hh * sh, ww * sw, c // mult
        total += 2 * ff * hh * ww * decoder.v.out_channels * decoder.v.patch ** 2 * 27 * c
    return total


def _time(fn, warmup: int, steps: int, world: int) -> float:
    for _ in range(warmup):
        fn()
    barrier(world)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        fn()
    b.record()
    torch.cuda.synchronize()
    return max_over_ranks(a.elapsed_time(b) / steps, world)


def _kernel_shares(fn) -> dict:
    """One extra run of fn with per-launch CUDA events: time share of each kernel class."""
    from kinomlx_b200 import ops

    log_ = ops.LaunchLog()
    ops.set_launch_log(log_)
    try:
        fn()
        torch.cuda.synchronize()
    finally:
        ops.set_launch_log(None)
    summary = log_.summary()
    total = sum(v["ms"] for v in summary.values()) or 1.0
    return {k: {"launches": int(v["launches"]), "ms": round(v["ms"], 3),
                "share": round(v["ms"] / total, 4),
                "tflops": round(v["flops"] / (v["ms"] * 1e9), 1) if v["flops"] else None,
                "gbs": round(v["bytes"] / (v["ms"] * 1e6), 1) if v["bytes"] else None}
            for k, v in sorted(summary.items(), key=lambda kv: -kv[1]["ms"])}


CONFIG1_FLOP = 376.9e9  # one double block at config 1: 347.9 GFLOP linear + 29.0 attention


def config1_block(device: torch.device) -> dict:
    """one MMDiT double block (512 text + 1024 image tokens, hidden 3072,
    24 heads, t = 0.5) in bf16 on the tensor cores and in fp32 (parity mode) on the CUDA cores;
    each timed call also runs the timestep MLP and the modulation products."""
    from kinomlx_b200.flux2 import config as fcfg
    from kinomlx_b200.flux2.transformer import Flux2Transformer, rotary_positions
    from kinomlx_b200.flux2.transformer_f32 import Flux2TransformerF32
    from kinomlx_b200.synthetic import flux_weights, normal

    v = fcfg.BASELINE.with_blocks(1, 0)
    nt, side = 512, 32
    ids = torch.zeros((1, nt + side * side, 2), dtype=torch.int64)
    ids[0, nt:, 0] = torch.arange(side).repeat_interleave(side)
    ids[0, nt:, 1] = torch.arange(side).repeat(side)
    cos, sin = rotary_positions(ids, v)
    cos, sin = cos.to(device), sin.to(device)
    t = torch.tensor([500.0], device=device)
    out = {}
    for name, cls, dtype in (("bf16", Flux2Transformer, torch.bfloat16),
                             ("fp32", Flux2TransformerF32, torch.float32)):
        model = cls(flux_weights(v, seed=0, device=device, dtype=dtype), v, device)
        img = normal((1, side * side, v.dim), seed=1, device=device, dtype=dtype)
        txt = normal((1, nt, v.dim), seed=2, device=device, dtype=dtype)
        ms = _time(lambda: model.double_block(0, img, txt, t, cos, sin), 3, 5, 1)
        out[name] = {"ms": round(ms, 3), "tflops": round(CONFIG1_FLOP / (ms * 1e9), 1)}
        model = None
        torch.cuda.empty_cache()
    return out


def run_secondary(world: int, rank: int, local: int) -> dict:
    """BASELINE configs 1 (one GPU) and 3-5 on the same GPUs (2 warm-up + 3 timed repetitions each): the
    metric's second half (VAE decode frames/s) and the other step latencies, each with its
    whole-step throughput against the measured sustained bf16 peak."""
    from kinomlx_b200.flux2 import config as fcfg
    from kinomlx_b200.flux2 import sampling
    from kinomlx_b200.flux2.transformer import Flux2Transformer
    from kinomlx_b200.ltx2 import config as lcfg
    from kinomlx_b200.ltx2 import video_vae as vae
    from kinomlx_b200.ltx2.transformer import LTXVideoTransformer
    from kinomlx_b200.multi_gpu import CfgSplit, cfg_split_step, decode_tiles_distributed
    from kinomlx_b200.sequence_parallel import SequenceParallel
    from kinomlx_b200.synthetic import flux_weights, ltx_weights, make_weights, normal

    device = torch.device("cuda", local)
    pk, _ = peaks()
    peak = float(pk.get("bf16_tflops_sustained", pk.get("bf16_tflops")))
    out = {}

    # config 1: the double block alone, bf16 and fp32
    if world == 1:
        out["config1_double_block"] = config1_block(device)

    # config 3: CFG over a batch of 2 (1 GPU) or the branch split (+ Ulysses inside each half)
    v = fcfg.BASELINE
    nt, side = 512, 64
    ids = torch.zeros((1, nt + side * side, 2), dtype=torch.int64)
    ids[0, nt:, 0] = torch.arange(side).repeat_interleave(side)
    ids[0, nt:, 1] = torch.arange(side).repeat(side)
    text = normal((1, nt, v.context_dim), seed=44, device=device)
    negative = normal((1, nt, v.context_dim), seed=45, device=device)
    sig = sampling.linear_sigmas(28)
    weights = flux_weights(v, seed=42, device=device)
    if world == 1:
        model = Flux2Transformer(weights, v, device)
        prepared = model.prepare(torch.cat([text, negative]), ids)
        cur = normal((1, side * side, v.in_channels), seed=43, device=device)
        step = lambda: sampling.denoise_step(model, prepared, cur, sig, 0, guidance=4.0, cfg=True)
        mode = "batch 2 on one GPU"
    elif world % 2 == 0:
        cfg = CfgSplit(peer=True)
        model = Flux2Transformer(weights, v, device, sp=cfg.sp)
        prepared = model.prepare(text if cfg.branch == 0 else negative, ids)
        i0, i1 = cfg.sp.shard(side * side)
        cur = normal((1, side * side, v.in_channels), seed=43, device=device)[:, i0:i1].contiguous()
        step = lambda: cfg_split_step(model, prepared, cur, sig, 0, 4.0, cfg)
        mode = f"branches split over 2 x {world // 2} GPUs (Ulysses inside each half)"
    else:
        step = None
    del weights
    if step is not None:
        ms = _time(step, 2, 3, world)
        out["config3_cfg"] = {"ms_per_step": round(ms, 3), "mode": mode,
                              "step_tflops": round(2 * step_flops() / (ms * 1e9), 1),
                              "frac_of_peak": round(2 * step_flops() / (ms * 1e9) / peak, 4),
                              "kernels": _kernel_shares(step)}
    if step is not None:
        model.sp.close()
    model = prepared = None
    torch.cuda.empty_cache()

    # config 4: LTX-2 video DiT step, 9216 video tokens + 256 text tokens, 48 blocks
    lv = lcfg.BASELINE_VIDEO
    sp = SequenceParallel(peer=True) if world > 1 else None
    lmodel = LTXVideoTransformer(ltx_weights(lv, seed=0, device=device), lv, device, sp=sp)
    torch.cuda.empty_cache()
    from kinomlx_b200.ltx2.patchifier import latent_positions

    f, h, w = 16, 18, 32
    pix = latent_positions(f, h, w)
    context = normal((1, 256, lv.context_dim), seed=2, device=device)
    lprep = lmodel.prepare(context, pix)
    t0, t1 = lmodel.sp.shard(f * h * w)
    lat = normal((1, f * h * w, lv.in_channels), seed=1, device=device)[:, t0:t1].contiguous()
    lstep = lambda: lmodel.run(lprep, lat, 0.725, sigma_next=0.421875, out=lat)
    ms = _time(lstep, 2, 3, world)
    out["config4_video_dit"] = {"ms_per_step": round(ms, 3),
                                "mode": f"Ulysses x{world}" if world > 1 else "single GPU",
                                "step_tflops": round(ltx_step_flops() / (ms * 1e9), 1),
                                "frac_of_peak": round(ltx_step_flops() / (ms * 1e9) / peak, 4),
                                "kernels": _kernel_shares(lstep)}
    lmodel.sp.close()
    lmodel = lprep = lat = None
    torch.cuda.empty_cache()

    # config 5: tiled causal GroupNorm(32) VAE decode, 128x16x18x32 -> 3x121x576x1024, 15 tiles
    vv = vae.BASELINE_VAE
    dec = vae.VideoDecoder(make_weights(vae.vae_weight_specs(vv), seed=0, device=device), vv, device)
    latent = normal((1, 128, 16, 18, 32), seed=0, device=device)
    # N > 1: the video is assembled on rank 0 (NCCL reduce of the tile canvases)
    fn = (lambda: dec.decode(latent)) if world == 1 else (lambda: decode_tiles_distributed(dec, latent, dst=0))
    ms = _time(fn, 1, 2, world)
    flops = vae_decode_flops(dec, latent.shape)
    out["config5_vae_decode"] = {"frames_per_s": round(121 / (ms / 1e3), 2), "ms_per_decode": round(ms, 2),
                                 "mode": f"tiles over {world} GPUs, video on rank 0" if world > 1 else "single GPU",
                                 "tiled_tflop": round(flops / 1e12, 1),
                                 "tflops": round(flops / (ms * 1e9), 1),
                                 "frac_of_peak": round(flops / (ms * 1e9) / peak, 4),
                                 "kernels": _kernel_shares(fn)}
    return out


def run_kernel_case(case: str, sol_tau: float | None = None, sol_inputs: str | None = None,
                    na_grid: tuple[int, int, int] = (121, 112, 192)) -> None:
    """Three launches of one kernel at a workload shape (for ncu captures). `gemm`: the single
    block's fused projection, 4608 x 21504 x 3072, with its in-step epilogue (per-head RMSNorm +
    RoPE on k and q, GELU on the MLP columns); `attention`: the joint attention over 4608 tokens
    x 24 heads; `conv3d`: a 256-channel causal 3x3x3 VAE conv over 25 x 96 x 128 voxels;
    `conv3d_narrow`: a 128-channel one over 49 x 96 x 128 voxels with residual and GroupNorm
    statistics. Inputs exceed the L2 (weights 132 MB; conv activations 154-157 MB)."""
    from kinomlx_b200 import ops
    from kinomlx_b200.synthetic import normal

    dev = torch.device("cuda", 0)
    n, d = 4608, 3072
    if case == "gemm":
        x = normal((1, n, d), seed=1, device=dev)
        w = normal((3 * d + 4 * d, d), seed=2, device=dev, std=0.02)
        nk = normal((128,), seed=4, device=dev)
        nq = normal((128,), seed=5, device=dev)
        ang = torch.randn((1, n, 64), generator=torch.Generator().manual_seed(6))
        rope = ops.RopeTables(torch.cos(ang).repeat_interleave(2, -1).to(dev),
                              torch.sin(ang).repeat_interleave(2, -1).to(dev))
        out = torch.empty((1, n, 7 * d), device=dev, dtype=torch.bfloat16)
        for _ in range(3):
            ops.linear(x, w, out, kind=ops.EPI_GELU, act_col_begin=3 * d,
                       qk_norm=[(0, nk), (2 * d, nq)], norm_width=d, rope=(rope, 0))
    elif case == "attention":
        qkv = normal((1, n, 3 * d), seed=3, device=dev)
        q, k, v = qkv[..., :d], qkv[..., d : 2 * d], qkv[..., 2 * d :]
        out = torch.empty((1, n, d), device=dev, dtype=torch.bfloat16)
        for _ in range(3):
            ops.attention([q], [k], [v], [out], heads=24)
        # timed after the captured launches: the image step's 4608 x 24 heads and the video
        # step's 9216 x 32 heads (CUDA events, 20 launches each after 3 warm ones)
        res = {}
        for name, tokens, heads in (("4608x24", n, 24), ("9216x32", 9216, 32)):
            width = heads * 128
            qkv = normal((1, tokens, 3 * width), seed=3, device=dev)
            q, k, v = qkv[..., :width], qkv[..., width : 2 * width], qkv[..., 2 * width :]
            out = torch.empty((1, tokens, width), device=dev, dtype=torch.bfloat16)
            fn = lambda: ops.attention([q], [k], [v], [out], heads=heads)
            ms = _time(fn, 3, 20, 1)
            flop = 4.0 * tokens * tokens * heads * 128
            res[name] = {"us": round(ms * 1e3, 1), "tflops": round(flop / (ms * 1e9), 1)}
        torch.cuda.synchronize()
        ops.device_status()
        print(json.dumps({"kernel_case": case, "ok": True, **res}))
        return
    elif case == "conv3d":
        x = normal((25, 96, 128, 256), seed=7, device=dev)
        w = normal((256, 3, 3, 3, 256), seed=8, device=dev, std=0.02)
        bias = normal((256,), seed=9, device=dev)
        for _ in range(3):
            ops.conv3d(x, w, bias, causal=True)
        ms = _time(lambda: ops.conv3d(x, w, bias, causal=True), 0, 10, 1)
        flop = 2.0 * 25 * 96 * 128 * 256 * 27 * 256
        torch.cuda.synchronize()
        ops.device_status()
        print(json.dumps({"kernel_case": case, "ok": True, "ms": round(ms, 4),
                          "tflops": round(flop / (ms * 1e9), 1)}))
        return
    elif case == "bandwidth":
        run_bandwidth_case(dev)
        return
    elif case == "av_step":
        run_av_step(dev)
        return
    elif case == "kv_step":
        run_kv_step(dev)
        return
    elif case == "sol":
        run_sol_case(dev, tau=sol_tau, family=sol_inputs)
        return
    elif case == "sol_step":
        run_sol_step(dev)
        return
    elif case == "packed_block":
        run_packed_block(dev)
        return
    elif case == "neighborhood":
        run_neighborhood_case(dev, na_grid)
        return
    elif case == "diffusion_decoder":
        run_diffusion_decoder_case(dev)
        return
    elif case == "f32":
        # fp32 parity mode at config 1: the image stream's FF up projection (1024 x 12288 x 3072,
        # GELU epilogue) and the joint attention over 1536 tokens x 24 heads
        from kinomlx_b200 import ops_f32

        f32 = torch.float32
        x = normal((1, 1024, d), seed=1, device=dev, dtype=f32)
        w = normal((4 * d, d), seed=2, device=dev, dtype=f32, std=0.02)
        out = torch.empty((1, 1024, 4 * d), device=dev, dtype=f32)
        qkv = normal((1, 1536, 3 * d), seed=3, device=dev, dtype=f32)
        q, k, v = qkv[..., :d], qkv[..., d : 2 * d], qkv[..., 2 * d :]
        att = torch.empty((1, 1536, d), device=dev, dtype=f32)
        times = {}
        for name, fn, flop in (
            ("gemm_f32", lambda: ops_f32.linear(x, w, out, kind=ops.EPI_GELU), 2.0 * 1024 * 4 * d * d),
            ("attention_f32", lambda: ops_f32.attention(q, k, v, att, heads=24),
             4.0 * 1536 * 1536 * 24 * 128),
        ):
            fn()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            fn()
            b.record()
            torch.cuda.synchronize()
            ms = a.elapsed_time(b) / 2
            times[name] = {"ms": round(ms, 4), "tflops": round(flop / (ms * 1e9), 1)}
        ops.device_status()
        print(json.dumps({"kernel_case": case, "ok": True, "kernels": times}))
        return
    else:
        # the decoder's last stage: 128 -> 128 channels at full resolution, with the residual
        # and the GroupNorm statistics of the next norm
        x = normal((49, 96, 128, 128), seed=7, device=dev)
        w = normal((128, 3, 3, 3, 128), seed=8, device=dev, std=0.02)
        bias = normal((128,), seed=9, device=dev)
        res = normal((49, 96, 128, 128), seed=10, device=dev)
        stats = ops.conv_stats_buffer(dev)
        for _ in range(3):
            ops.conv3d(x, w, bias, causal=True, residual=res, stats=stats)
        ms = _time(lambda: ops.conv3d(x, w, bias, causal=True, residual=res, stats=stats), 0, 10, 1)
        flop = 2.0 * 49 * 96 * 128 * 128 * 27 * 128
        torch.cuda.synchronize()
        ops.device_status()
        print(json.dumps({"kernel_case": case, "ok": True, "ms": round(ms, 4),
                          "tflops": round(flop / (ms * 1e9), 1)}))
        return
    torch.cuda.synchronize()
    ops.device_status()
    print(json.dumps({"kernel_case": case, "ok": True}))


def run_av_step(dev: torch.device) -> None:
    """The joint audio/video LTX-2.3 step (48 blocks, video 4096 wide with 32 x 128 heads, audio
    2048 wide with 32 x 64 heads) at BASELINE config 4's video shape (16 x 18 x 32 = 9216 tokens,
    256 text tokens) plus 126 audio tokens (5 s at 25 tokens/s) and 128 audio text tokens:
    2 warm-up and 3 timed X0 + Euler steps, then one step with per-launch events."""
    from kinomlx_b200.ltx2 import av_transformer as avm
    from kinomlx_b200.ltx2 import config as lcfg
    from kinomlx_b200.synthetic import ltx_av_weight_specs, make_weights, normal

    video, audio = lcfg.BASELINE_VIDEO, avm.audio_variant(lcfg.BASELINE_VIDEO.blocks)
    model = avm.LTXAVTransformer(
        make_weights(ltx_av_weight_specs(video, audio, video.blocks), seed=0, device=dev),
        video, audio, dev)
    torch.cuda.empty_cache()
    f, h, w = 16, 18, 32
    fr, hr, wr = torch.meshgrid(torch.arange(f), torch.arange(h), torch.arange(w), indexing="ij")
    starts = torch.stack([fr, hr, wr]).reshape(3, -1).float()
    vpos = torch.stack([starts, starts + 1], -1)[None] * torch.tensor([8.0, 32.0, 32.0]).reshape(1, 3, 1, 1)
    vpos[:, 0] = torch.clamp(vpos[:, 0] + 1 - 8, min=0) / 24.0
    ta = 126
    at = torch.arange(ta, dtype=torch.float32) * 0.04
    apos = torch.stack([at, at + 0.04], -1)[None, None]
    prep = model.prepare(normal((1, 256, video.dim), seed=2, device=dev),
                         normal((1, 128, audio.dim), seed=3, device=dev), vpos, apos)
    vlat = normal((1, f * h * w, video.in_channels), seed=1, device=dev)
    alat = normal((1, ta, audio.in_channels), seed=4, device=dev)
    step = lambda: model.run(prep, vlat, alat, 0.725, sigma_next=0.421875, video_out=vlat,
                             audio_out=alat)
    ms = _time(step, 2, 3, 1)
    from kinomlx_b200 import ops

    ops.device_status()
    print(json.dumps({"kernel_case": "av_step", "ok": True, "ms_per_step": round(ms, 3),
                      "video_tokens": f * h * w, "audio_tokens": ta,
                      "video_only_step_tflop": round(ltx_step_flops() / 1e12, 1),
                      "kernels": _kernel_shares(step)}))


def run_neighborhood_case(dev: torch.device, grid: tuple[int, int, int] = (121, 112, 192)) -> None:
    """The LTX-2.5 diffusion decoder's neighborhood attention at its final-stage call (121 x 112 x
    192 queries, four 64-wide heads, 11 x 11 x 11 windows: the call the reference documents at
    632 ms on an M1 Max, kinomlx/models/ltx2/kernels/neighborhood_attention.py:21-25) and the
    3 x 7 x 7 and 3 x 5 x 5 windows on the same grid. Algorithmic work: 4 x 64 FLOP per (query,
    window key) pair; the MMAs also score the keys of each query tile's window union that lie
    outside a query's window."""
    from kinomlx_b200 import ops

    heads = 4
    shape = (1, *grid, heads, 64)
    g = torch.Generator(device=dev).manual_seed(5)
    q = (torch.randn(shape, generator=g, device=dev) * 0.125).half()
    k = torch.randn(shape, generator=g, device=dev).half()
    v = torch.randn(shape, generator=g, device=dev).half()
    out = torch.empty_like(q)
    tokens = grid[0] * grid[1] * grid[2]
    rows = []
    for window in ((11, 11, 11), (3, 7, 7), (3, 5, 5)):
        ms = _time(lambda: ops.neighborhood_attention(q, k, v, window=window, out=out), 3, 10, 1)
        keys = window[0] * window[1] * window[2]
        flop = 4.0 * 64 * tokens * heads * keys
        rows.append({"window": list(window), "ms": round(ms, 3),
                     "algorithmic_tflop": round(flop / 1e12, 3),
                     "tflops": round(flop / (ms * 1e9), 1)})
    ops.device_status()
    print(json.dumps({"kernel_case": "neighborhood", "ok": True, "grid": list(grid),
                      "heads": heads, "calls": rows,
                      "reference_m1_max_ms_final_stage": 632.0}))


def run_diffusion_decoder_case(dev: torch.device) -> None:
    """One LTX-2.5 diffusion-decoder decode of a (128, 16, 14, 24) latent into 121 frames of
    448 x 768 (the video of the reference's documented final-stage attention call: 121 x 112 x
    192 pixel-patch tokens, four 64-wide heads, 11 x 11 x 11 windows). The other stage widths,
    depths and windows are a synthetic choice (the reference takes them from a checkpoint):
    widths 1024 / 512 / 512 / 256 / 256, two blocks per stage, windows 3 x 5 x 5 (stages 1-2) and
    3 x 7 x 7 (stages 3-4), seeded random weights, one x0 step."""
    from kinomlx_b200 import ops
    from kinomlx_b200.ltx2.diffusion_decoder import DiffusionDecoderConfig, DiffusionVideoDecoder
    from kinomlx_b200.synthetic import diffusion_decoder_weights, normal

    cfg = DiffusionDecoderConfig(
        head_dim=64, stage_channels=(1024, 512, 512, 256, 256), stage_depths=(2, 2, 2, 2, 2),
        stage_kernels=((3, 5, 5), (3, 5, 5), (3, 7, 7), (3, 7, 7)),
        upsample_strides=((1, 2, 2), (2, 1, 1), (2, 2, 2), (2, 2, 2)),
        upsample_channel_reductions=(2, 1, 2, 1), stage5_kernel=(11, 11, 11))
    model = DiffusionVideoDecoder(diffusion_decoder_weights(cfg, seed=0, device=dev), cfg, dev)
    shape = (1, 128, 16, 14, 24)
    latent = normal(shape, seed=1, device=dev)
    noise = normal(cfg.working_pixel_shape(shape), seed=2, device=dev)
    fn = lambda: model(latent, noise)
    ms = _time(fn, 1, 3, 1)
    shares = _kernel_shares(fn)
    video = fn()
    torch.cuda.synchronize()
    ops.device_status()
    frames = video.shape[2]
    print(json.dumps({"kernel_case": "diffusion_decoder", "ok": True,
                      "video": list(video.shape), "ms_per_decode": round(ms, 2),
                      "frames_per_s": round(frames / (ms / 1e3), 1), "kernels": shares,
                      "finite": bool(torch.isfinite(video.float()).all())}))


def run_packed_block(dev: torch.device) -> None:
    """Packed (mxfp8) LTX-2 block linears against bf16 ones at config 4's shapes: one transformer
    forward over 2 blocks at 9216 video + 256 text tokens, in each `transformer_quantize` mode,
    and the mxfp8 dequantisation of the largest weight (16384 x 4096) alone. The packed modes
    dequantise each block linear into a bf16 scratch right before its GEMM."""
    from kinomlx_b200 import ops
    from kinomlx_b200.ltx2 import config as lcfg
    from kinomlx_b200.ltx2.patchifier import latent_positions
    from kinomlx_b200.ltx2.transformer import LTXVideoTransformer
    from kinomlx_b200.synthetic import ltx_weights, normal

    v = lcfg.BASELINE_VIDEO.with_blocks(2)
    grid = (16, 18, 32)
    w = ltx_weights(v, seed=0)
    latent = normal((1, grid[0] * grid[1] * grid[2], v.in_channels), seed=1, device=dev)
    context = normal((1, 256, v.context_dim), seed=2)
    pos = latent_positions(*grid)
    rows = {}
    for mode in ("off", "mxfp8-blocks", "mxfp8-blocks-pretranspose"):
        model = LTXVideoTransformer(w, v, dev, quantize=mode)
        prep = model.prepare(context, pos)
        ms = _time(lambda: model.run(prep, latent, 0.725), 3, 10, 1)
        rows[mode] = {"ms_per_forward": round(ms, 3), "ms_per_block": round(ms / v.blocks, 3)}
        del model, prep
        torch.cuda.empty_cache()
    base = rows["off"]["ms_per_forward"]
    for mode in rows:
        rows[mode]["vs_bf16"] = round(rows[mode]["ms_per_forward"] / base, 3)
    from kinomlx_b200.ltx2 import quantization as qz

    packed = qz.pack_linear(normal((16384, 4096), seed=3, device=dev, std=0.02), transposed=False,
                            device=dev)
    scratch = torch.empty((16384, 4096), device=dev, dtype=torch.bfloat16)
    dq = {}
    for transposed in (False, True):
        pw = packed if not transposed else qz.pack_linear(
            normal((16384, 4096), seed=3, device=dev, std=0.02), transposed=True, device=dev)
        ms = _time(lambda: pw.dequantize_into(scratch), 3, 20, 1)
        nbytes = pw.words.numel() * 4 + pw.scales.numel() + scratch.numel() * 2
        dq["pretransposed" if transposed else "packed"] = {
            "us": round(ms * 1e3, 1), "gbs": round(nbytes / (ms * 1e6), 1)}
    ops.device_status()
    print(json.dumps({"kernel_case": "packed_block", "ok": True, "tokens": latent.shape[1],
                      "blocks": v.blocks, "modes": rows, "dequant_16384x4096": dq}))


def run_sol_case(dev: torch.device, tau: float | None = None, family: str | None = None) -> None:
    """Sol-Attn at config 4's video self-attention (9216 tokens on a 16 x 18 x 32 Morton grid,
    32 heads of 128) against the dense kernel on the same q, k, v, for the published taus (or
    one `tau` and one input `family`, for a launch list: 3 warm-up calls, then the timed ones).
    The algorithmic work counts the exact (query, routed key) pairs and the (query, centroid)
    pairs, 4 x 128 FLOP each."""
    from kinomlx_b200 import ops
    from kinomlx_b200.kernels import sol_attention as sol
    from kinomlx_b200.synthetic import normal

    tokens, heads, d = 9216, 32, 4096
    grid = (16, 18, 32)
    out = torch.empty((tokens, d), device=dev, dtype=torch.bfloat16)
    order = sol.morton_order(*grid).to(dev)
    # input families: i.i.d. N(0, 1) q, k, v (routing uncorrelated between neighbouring query
    # blocks: the worst case for a CTA's shared block list), and smooth fields over the latent
    # grid plus noise (32 random low-frequency cosine modes mixed into each head, N(0, 0.3^2) on
    # top), without and with the block's 3-D RoPE on q and k
    gen = torch.Generator(device=dev).manual_seed(11)
    f_, h_, w_ = torch.meshgrid(*(torch.arange(n, device=dev, dtype=torch.float32) / n for n in grid),
                                indexing="ij")
    pos = torch.stack([f_, h_, w_], -1).reshape(-1, 3)
    freq = torch.rand((3, 32), generator=gen, device=dev) * 3.0
    phase = torch.rand((32,), generator=gen, device=dev) * 6.283
    modes = torch.cos(6.283 * pos @ freq + phase)  # (tokens, 32)
    smooth = lambda: (modes @ torch.randn((32, d), generator=gen, device=dev) / 4.0
                      + 0.3 * torch.randn((tokens, d), generator=gen, device=dev)).to(torch.bfloat16)
    from kinomlx_b200.ltx2 import config as lcfg
    from kinomlx_b200.ltx2.patchifier import latent_positions
    from kinomlx_b200.ltx2.transformer import precompute_freqs_cis

    cos, sin = (t.to(dev) for t in precompute_freqs_cis(latent_positions(*grid), lcfg.BASELINE_VIDEO))
    rope = lambda x: ops.split_rope(x[None], cos, sin)[0]
    inputs = {"iid": normal((tokens, 3 * d), seed=3, device=dev).split(d, 1),
              "smooth": (smooth(), smooth(), smooth()),
              # the same kind of fields after the video block's 3-D rotary embedding, as q and k
              # reach the self-attention
              "smooth_rope": (rope(smooth()), rope(smooth()), smooth())}
    dense_flop = 4.0 * heads * tokens * tokens * 128
    q, k, v = inputs["iid"]
    dense_ms = _time(lambda: ops.attention([q[None]], [k[None]], [v[None]], [out[None]], heads=heads),
                     3, 10, 1)
    rows = []
    taus = (0.5, 1.0, 1.25, 1.5) if tau is None else (tau,)
    chosen = [(name, t) for name, t in inputs.items() if family is None or name == family]
    for (family, (q, k, v)), tau in ((fam_t, t) for fam_t in chosen for t in taus):
        ms = _time(lambda: ops.sol_attention(q, k, v, heads=heads, tau=tau, order=order, out=out),
                   3, 10, 1)
        routes = sol.routed_blocks(q, k, v, heads=heads, tau=tau, order=order)
        nb = routes.shape[-1]
        lengths = torch.clamp(tokens - torch.arange(nb, device=dev) * 64, max=64).float()
        exact_keys = (routes.float() * lengths).sum(-1)  # (heads, blocks): keys per query row
        rows_per_block = lengths[None, :]
        exact = float((exact_keys * rows_per_block).sum())
        centroid = float(((nb - routes.sum(-1)).float() * rows_per_block).sum())
        flop = 4.0 * 128 * (exact + centroid)
        pad = (-nb) % sol.QUERY_BLOCKS_PER_CTA
        union = torch.nn.functional.pad(routes, (0, 0, 0, pad)).reshape(
            heads, -1, sol.QUERY_BLOCKS_PER_CTA, nb).any(2)
        rows.append({"inputs": family, "tau": tau, "ms": round(ms, 3),
                     "speedup_vs_dense": round(dense_ms / ms, 2),
                     "routed_fraction": round(float(routes.float().mean()), 4),
                     "cta_block_union_fraction": round(float(union.float().mean()), 4),
                     "algorithmic_tflop": round(flop / 1e12, 3),
                     "tflops": round(flop / (ms * 1e9), 1)})
    ops.device_status()
    print(json.dumps({"kernel_case": "sol", "ok": True, "tokens": tokens, "heads": heads,
                      "dense_ms": round(dense_ms, 3),
                      "dense_tflops": round(dense_flop / (dense_ms * 1e9), 1), "sol": rows}))


def run_sol_step(dev: torch.device) -> None:
    """The 48-block LTX-2 video step at config 4 with a Sol-Attn step (tau 1, layer 0 dense)
    against the dense step, X0 + Euler fused, 2 warm-up and 3 timed steps each."""
    from kinomlx_b200 import ops
    from kinomlx_b200.kernels import sol_attention as sol
    from kinomlx_b200.ltx2 import config as lcfg
    from kinomlx_b200.ltx2.patchifier import latent_positions
    from kinomlx_b200.ltx2.sparse_attention import SparseAttentionStep
    from kinomlx_b200.ltx2.transformer import LTXVideoTransformer
    from kinomlx_b200.synthetic import ltx_weights, normal

    grid = (16, 18, 32)
    tokens = grid[0] * grid[1] * grid[2]
    v4 = lcfg.BASELINE_VIDEO
    model = LTXVideoTransformer(ltx_weights(v4, seed=0, device=dev), v4, dev)
    torch.cuda.empty_cache()
    prep = model.prepare(normal((1, 256, v4.context_dim), seed=5, device=dev), latent_positions(*grid))
    latent = normal((1, tokens, v4.in_channels), seed=4, device=dev)
    nxt = latent.clone()
    steps = {}
    for name, sparse in (("dense", None),
                         ("sol_tau1_layer0_dense", SparseAttentionStep(1.0, frozenset({0}),
                                                                       sol.morton_order(*grid))),
                         ("sol_tau1.5_layer0_dense", SparseAttentionStep(1.5, frozenset({0}),
                                                                         sol.morton_order(*grid)))):
        steps[name] = round(_time(lambda: model.run(prep, latent, 0.725, sigma_next=0.421875,
                                                    out=nxt, sparse=sparse), 2, 3, 1), 3)
    ops.device_status()
    print(json.dumps({"kernel_case": "sol_step", "ok": True, "tokens": tokens,
                      "ltx_step_ms": steps}))


def run_kv_step(dev: torch.device) -> None:
    """Klein KV editing at the reference's graph (4096 wide, 32 heads, 8 double + 24 single
    blocks, SwiGLU): 512 text tokens, a 64 x 64 target and a 64 x 64 reference. Times the
    extracting evaluation ([text | reference | target] rows, reference keys/values kept), a
    reusing one ([text | target] rows against the kept rows) and a plain evaluation of the target
    alone, each with its Euler update fused; 2 warm-up and 3 timed evaluations each."""
    from kinomlx_b200 import ops
    from kinomlx_b200.flux2 import config as fcfg
    from kinomlx_b200.flux2.transformer import Flux2Transformer
    from kinomlx_b200.synthetic import flux_weights, normal

    v = fcfg.KLEIN
    model = Flux2Transformer(flux_weights(v, seed=0, device=dev), v, dev)
    torch.cuda.empty_cache()
    nt, side = 512, 64
    text_ids = torch.zeros((1, nt, 4), dtype=torch.int64)
    text_ids[0, :, 3] = torch.arange(nt)
    grid = torch.stack(torch.meshgrid(torch.arange(side), torch.arange(side), indexing="ij"), -1).reshape(1, -1, 2)
    image_ids = torch.zeros((1, side * side, 4), dtype=torch.int64)
    image_ids[..., 1:3] = grid
    ref_ids = image_ids.clone()
    ref_ids[..., 0] = 10
    text = normal((1, nt, v.context_dim), seed=1, device=dev)
    extract, reuse = model.prepare_layouts(
        text, (torch.cat([text_ids, ref_ids, image_ids], 1), torch.cat([text_ids, image_ids], 1)))
    plain = model.prepare(text, torch.cat([text_ids, image_ids], 1))
    nr = side * side
    image = normal((1, 2 * nr, v.in_channels), seed=2, device=dev)  # [reference | target]
    target = image[:, nr:]
    cache = model.new_reference_kv(nr)
    t, dt = 500.0, -0.25

    def extracting():
        cache.extracting = True
        model.run(extract, image, t, euler_dt=dt, sample=target, out=target, reference_kv=cache)

    def reusing():
        cache.extracting = False
        model.run(reuse, target, t, euler_dt=dt, sample=target, out=target, reference_kv=cache)

    times = {}
    for name, fn in (("extracting", extracting), ("reusing", reusing),
                     ("plain_target", lambda: model.run(plain, target, t, euler_dt=dt,
                                                        sample=target, out=target))):
        times[name] = round(_time(fn, 2, 3, 1), 3)
    ops.device_status()
    cache.clear()
    print(json.dumps({"kernel_case": "kv_step", "ok": True, "ms_per_evaluation": times,
                      "text_tokens": nt, "target_tokens": nr, "reference_tokens": nr}))


def run_bandwidth_case(dev: torch.device) -> None:
    """The HBM-bound kernels at workload shapes, three launches each with the L2 flushed before
    every launch (a 256 MB write) and the GPU held busy while the launch is queued: achieved GB/s = algorithmic bytes / CUDA-event time of
    launches 2 and 3, against the measured copy bandwidth. Shapes: the LTX video block's rows
    (9216 x 4096) for AdaLN and the full-row QK norm + split RoPE, the Flux step's rows
    (4608 x 3072) for its LayerNorm AdaLN, the LTX FF width (9216 x 16384) for the standalone
    GELU, the last VAE stage (49 x 96 x 128 voxels x 128 channels) for PixelNorm + SiLU and the
    GroupNorm apply pass, one decoded VAE tile for the blend, a 16384 x 4096 mxfp8 weight for the
    dequantisation."""
    from kinomlx_b200 import ops
    from kinomlx_b200.synthetic import normal

    bf = torch.bfloat16
    flush = torch.empty(256 << 20, device=dev, dtype=torch.uint8)
    results = {}

    def measure(name: str, nbytes: float, fn) -> None:
        fn()
        total = 0.0
        for _ in range(2):
            flush.fill_(1)
            # keep the GPU busy while the host queues the events and the launch, so the timed
            # span holds the kernel and not the host's enqueue latency
            torch.cuda._sleep(400_000)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            torch.cuda.synchronize()
            total += a.elapsed_time(b)
        ms = total / 2
        results[name] = {"bytes": nbytes, "ms": round(ms, 4), "gbs": round(nbytes / (ms * 1e6), 1)}

    n, d = 9216, 4096
    x = normal((1, n, d), seed=1, device=dev)
    shift = normal((1, d), seed=2, device=dev)
    scale = normal((1, d), seed=3, device=dev)
    y = torch.empty_like(x)
    measure("adaln_rms_9216x4096", 4.0 * n * d,
            lambda: ops.adaln(x, shift, scale, y, norm=ops.NORM_RMS))
    xf = normal((1, 4608, 3072), seed=4, device=dev)
    yf = torch.empty_like(xf)
    sf, cf = normal((1, 3072), seed=5, device=dev), normal((1, 3072), seed=6, device=dev)
    measure("adaln_layer_4608x3072", 4.0 * 4608 * 3072,
            lambda: ops.adaln(xf, sf, cf, yf, norm=ops.NORM_LAYER))
    xf = yf = None
    wq = normal((d,), seed=7, device=dev)
    ang = torch.rand((1, 32, n, 64), device=dev) * 6.0
    cos, sin = torch.cos(ang).contiguous(), torch.sin(ang).contiguous()
    ang = None
    measure("qk_norm_rope_fullrow_split_9216x4096", 4.0 * n * d + 8.0 * n * d / 2,
            lambda: ops.qk_norm_rope(x, heads=32, weight=wq, norm=ops.QKNORM_FULL_ROW,
                                     rope=ops.ROPE_SPLIT, cos=cos, sin=sin))
    measure("split_rope_9216x4096", 4.0 * n * d + 8.0 * n * d / 2,
            lambda: ops.split_rope(x, cos, sin))
    x = y = cos = sin = None
    h = normal((n, 16384), seed=8, device=dev)
    measure("gelu_tanh_9216x16384", 4.0 * h.numel(), lambda: ops.gelu_tanh(h))
    h = None
    torch.cuda.empty_cache()
    vox = normal((49, 96, 128, 128), seed=9, device=dev)
    measure("pixel_norm_silu_49x96x128x128", 4.0 * vox.numel(),
            lambda: ops.pixel_norm(vox, silu=True))
    w = normal((128, 3, 3, 3, 128), seed=10, device=dev, std=0.02)
    bias = normal((128,), seed=11, device=dev)
    stats = ops.conv_stats_buffer(dev)
    conv = ops.conv3d(vox, w, bias, causal=True, stats=stats)
    gw, gb = normal((128,), seed=12, device=dev), normal((128,), seed=13, device=dev)
    gout = torch.empty_like(conv)
    measure("group_norm_from_stats_silu_49x96x128x128", 4.0 * conv.numel(),
            lambda: ops.group_norm_from_stats(conv, gw, gb, 1e-6, stats, silu=True, out=gout))
    vox = conv = gout = None
    torch.cuda.empty_cache()
    tile = normal((121, 64, 64, 48), seed=14, device=dev)
    canvas = torch.zeros((1, 3, 121, 576, 1024), device=dev, dtype=torch.float32)
    weights = torch.zeros((576, 1024), device=dev, dtype=torch.float32)
    ramp = torch.ones(256, device=dev)
    measure("tile_blend_121x256x256x3", 2.0 * tile.numel() + 8.0 * tile.numel(),
            lambda: ops.tile_blend(tile, canvas, weights, 0, 0, ramp, ramp))
    tile = canvas = weights = None
    torch.cuda.empty_cache()
    rows, cols = 16384, 4096
    words = torch.randint(-2**31, 2**31 - 1, (rows, cols // 4), device=dev, dtype=torch.int32)
    scales = torch.randint(118, 130, (rows, cols // 32), device=dev, dtype=torch.uint8)
    wout = torch.empty((rows, cols), device=dev, dtype=bf)
    measure("dequant_mxfp8_16384x4096", 4.0 * words.numel() + scales.numel() + 2.0 * rows * cols,
            lambda: ops.dequantize(words, scales, None, mode="mxfp8", group_size=32, bits=8,
                                   out=wout))
    torch.cuda.synchronize()
    ops.device_status()
    pk, source = peaks()
    for r in results.values():
        r["frac_of_copy_peak"] = round(r["gbs"] / float(pk["hbm_gbs"]), 4)
    print(json.dumps({"kernel_case": "bandwidth", "ok": True, "peak_gbs": pk["hbm_gbs"],
                      "peak_source": source, "kernels": results}))


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["kino", "reference"], default="kino")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--no-secondary", action="store_true",
                    help="skip the configs 3-5 measurements (CFG, video DiT, VAE decode)")
    ap.add_argument("--kernel-case", choices=["gemm", "attention", "conv3d", "conv3d_narrow", "sol", "sol_step",
                                              "packed_block", "neighborhood", "diffusion_decoder", "bandwidth", "f32", "av_step", "kv_step"],
                    help="run 3 launches of one kernel and exit (for ncu captures)")
    ap.add_argument("--sol-tau", type=float, help="--kernel-case sol: this tau only")
    ap.add_argument("--na-grid", default="121,112,192",
                    help="--kernel-case neighborhood: the T,H,W token grid")
    ap.add_argument("--sol-inputs", choices=["iid", "smooth", "smooth_rope"],
                    help="--kernel-case sol: this input family only")
    args = ap.parse_args()
    if args.kernel_case:
        run_kernel_case(args.kernel_case, args.sol_tau, args.sol_inputs,
                        tuple(int(x) for x in args.na_grid.split(",")))
        return
    if args.warmup < 3:
        log("warm-up raised to 3 steps (timing rule)")
        args.warmup = 3
    if args.impl == "reference":
        reserve_stdout()
        rank = int(os.environ.get("RANK", "0"))
        run_reference(args, int(os.environ.get("WORLD_SIZE", "1")), rank)
        return
    reserve_stdout()
    world, rank, local = dist_setup()
    try:
        run_kino(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
