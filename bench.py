"""Benchmark: SD-1.5-shaped UNet denoise steps/s.

Workload: bf16 UNet (random init, seed 0) on latents [64, 4, 64, 64] ~ N(0,1) with context
[64, 77, 768] ~ N(0,1); one "step" = one UNet evaluation of the whole batch + the fused DDIM
update.  Under torchrun with N ranks the batch is sharded (64/N samples per GPU, strong scaling),
weights are replicated, and the output latents are all-gathered once over NCCL at the end of the
timed region.  `value` = steps/s of the whole 64-sample job.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python bench.py --workload sampler|vae|text [--batch B]   (the workloads around the UNet)

`--impl reference` times the reference mtorch's own CPU implementation (built from its sources
into oracle/_ref; the restated C oracle when that is absent) on all host cores: each step runs
every op of one sample's UNet forward at full widths on 1/R of its output rows (oracle/cpu_bench.py),
and `value` is the C5 steps/s that implies (one C5 step = 64 * R sampled steps).
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

BATCH = 64
H = W = 64
CTX = 77
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per launch per sample, from one ncu
# capture of `bench.py --kernel attn|conv --batch 64` (the ncu summaries under profiles/): 654.3 MB
# and 296.6 MB per 64-sample launch.
DRAM_BYTES_PER_SAMPLE = {"attn": (503461632 + 150793472) / 64, "conv": (169706752 + 126914048) / 64}
METRIC = "UNet denoise steps/s (SD-1.5 shape, bf16, batch 64 latents 64x64, context 77x768)"


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["hbm_gbs"], d["bf16_tflops"], d.get("bf16_tflops_sustained", d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


# ---------------------------------------------------------------------------------------------
# clocks


def smi_index(local: int):
    """nvidia-smi's index of torch device `local` (matched by UUID; CUDA_VISIBLE_DEVICES as the
    fallback), so that each rank samples only the GPU it runs on."""
    try:
        import torch

        uuid = str(torch.cuda.get_device_properties(local).uuid)
        out = subprocess.run(["nvidia-smi", "--query-gpu=index,uuid", "--format=csv,noheader"], capture_output=True,
                             text=True, timeout=30).stdout
        for line in out.splitlines():
            idx, u = [x.strip() for x in line.split(",")[:2]]
            if u.lower().removeprefix("gpu-") == uuid.lower().removeprefix("gpu-"):
                return int(idx)
    except Exception:  # noqa: BLE001
        pass
    vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    parts = [v.strip() for v in vis.split(",") if v.strip()]
    if local < len(parts) and parts[local].isdigit():
        return int(parts[local])
    return local


class ClockSampler:
    """nvidia-smi sampling (200 ms) of ONE GPU during the timed region."""

    def __init__(self, path: Path, gpu_index: int):
        self.path, self.gpu_index = path, gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu_index),
                 "--query-gpu=index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (FileNotFoundError, OSError):
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            self.proc.wait()


def clock_summary(paths):
    """Median SM clock, max clock and the throttle reasons seen, over the samples of the GPUs the
    ranks ran on (one file per rank, each holding only its own GPU's samples)."""
    sm, mx, reasons, gpus = [], None, set(), set()
    names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    for path in paths:
        if not Path(path).exists():
            continue
        for line in Path(path).read_text().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            gpus.add(f[0])
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
    if not sm:
        return None
    return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm),
            "gpus": sorted(gpus, key=int)}


# ---------------------------------------------------------------------------------------------
# CPU baseline (reference mtorch on the host cores)


def cpu_sampled_steps(processes: int, warmup: int, steps: int):
    """Times the reference's CPU path on every op of the UNet (oracle/cpu_bench.py: all ops of one
    sample's forward at full widths on 1/R of their output rows, spread over `processes` single-
    threaded processes).  Returns (seconds per sampled step [list], sampler)."""
    from oracle import cpu_bench

    r = cpu_bench.default_r(processes)
    s = cpu_bench.SampledUNet(processes, r, size=H)
    try:
        for _ in range(warmup):
            s.step()
        times = [s.step() for _ in range(steps)]
    finally:
        s.close()
    return times, s


def cpu_result(times, s, processes):
    """steps/s of the 64-sample C5 step from the sampled steps: one C5 step = 64 * R sampled steps."""
    sec = statistics.median(times)
    value = 1.0 / (BATCH * s.r * sec)
    return {"value": value, "unit": "steps/s", "cores": processes, "kind": s.kind,
            "sample": s.describe() + f"; median {sec:.2f} s per sampled step over {len(times)} steps",
            "sampled_fraction_of_step": 1.0 / (BATCH * s.r), "seconds_per_sampled_step": sec,
            "gflops_per_s": s.full_flops / s.r / sec / 1e9}


# ---------------------------------------------------------------------------------------------


def run_reference(args):
    """The reference arm: the reference mtorch's own CPU implementation, all host cores, a
    bounded sample per step (see cpu_sampled_steps).  `ms_per_step` is the measured wall time of
    one sampled step; `value` is the C5 steps/s it implies (64 * R sampled steps per C5 step)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    procs = os.cpu_count() or 1
    times, s = cpu_sampled_steps(procs, args.warmup, max(args.steps, 1))
    base = cpu_result(times, s, procs)
    value = base["value"]
    cfg = {"workload": "C5: SD-1.5 UNet, batch 64 latents [64,4,64,64], context [64,77,768], 1 UNet eval "
           "per step (fp32 reference CPU path, row-sampled)", "global_batch": BATCH, "seq_len": H * W,
           "parallelism": f"{procs} host processes, ops of one sample spread over them", "l2": "n/a (CPU)"}
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "steps/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * base["seconds_per_sampled_step"],
            "ms_per_step_is": "wall time of one sampled step (1/(64*R) of a C5 step)",
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": cfg, "cpu_baseline": base,
            "e2e": {"value": value, "unit": "steps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


def run_ours(args):
    import torch

    import mtorch_b200 as mt
    from mtorch_b200 import _lib, ops
    from mtorch_b200 import parallel
    from mtorch_b200.graphs import Graphed
    from mtorch_b200.unet import DDIM, UNet, timestep_embedding, unet_flops_per_sample

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    mt.cuda.set_device(local)
    dist = comm = None
    if world > 1:  # host plumbing over gloo; the device all-gather is NCCL through the C ABI
        os.environ.setdefault("GLOO_SOCKET_IFNAME", "lo")  # single node: loopback rendezvous
        dist = parallel.init("gloo")
        comm = parallel.NcclCommunicator(rank, world, dist.distributed_c10d._get_default_store())
    gb = args.global_batch
    lo, hi = parallel.shard(gb, world, rank)
    nb = hi - lo
    dev = f"cuda:{local}"
    out_dir = ROOT / "gpurun_out"
    out_dir.mkdir(exist_ok=True)

    # ---- model and inputs (seeded; every rank builds the same weights) ----
    mt.manual_seed(0)
    unet = UNet(device=dev, dtype="bfloat16")
    mt.manual_seed(1)
    lat_all = mt.randn(gb, 4, H, W)
    ctx_all = mt.randn(gb, CTX, 768)
    lat_h = lat_all[lo:hi].to("bfloat16")
    ctx_h = ctx_all[lo:hi].to("bfloat16")
    sched = DDIM(steps=50)
    temb_all = [mt.tensor(timestep_embedding(np.full(nb, float(t))), dtype="bfloat16", device=dev)
                for t in sched.timesteps]
    x = lat_h.to(dev)
    ctx = ctx_h.to(dev)
    stream = mt.cuda.current_stream()

    # The UNet forward is captured once as a CUDA graph (static latent / time-embedding / context
    # buffers); each step copies its inputs in, replays it and applies the fused DDIM update.
    use_graph = not args.eager
    graphed = Graphed(unet, x, temb_all[0], ctx) if use_graph else None

    def step(i, x):
        t = sched.timesteps[i % len(sched.timesteps)]
        te = temb_all[i % len(temb_all)]
        eps = graphed(x, te, ctx) if use_graph else unet(x, te, ctx)
        return sched.step(x, eps, t)

    for i in range(args.warmup):
        x = step(i, x)
    if comm:  # NCCL connects its channels on the first collective: keep that out of the timed region
        comm.all_gather(x)
    mt.cuda.synchronize()

    # ---- device-timed region ----
    lib = _lib.lib()
    clocks = ClockSampler(out_dir / f"clocks_rank{rank}.csv", smi_index(local))
    with clocks:
        if dist:
            dist.barrier()
        mt.cuda.synchronize()
        n0 = lib.mt_cuda_launch_count()
        r0 = graphed.replays if use_graph else 0
        e0, e1 = mt.cuda.Event(), mt.cuda.Event()
        e0.record(stream)
        for i in range(args.steps):
            x = step(args.warmup + i, x)
        gathered = None
        if comm:  # output latents, all ranks
            gathered = comm.all_gather(x)
        e1.record(stream)
        mt.cuda.synchronize()
        if dist:
            dist.barrier()
        # kernels launched directly + this library's kernels replayed inside the CUDA graph
        launches = lib.mt_cuda_launch_count() - n0
        if use_graph:
            launches += (graphed.replays - r0) * graphed.kernels_per_replay
    ms = e0.elapsed_time(e1)
    if dist:
        tt = torch.tensor([ms])
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())
    ms_per_step = ms / args.steps
    value = 1000.0 / ms_per_step

    # ---- end to end through the public API with host buffers (pinned), every step ----
    lat_pin = lat_h.pin_memory()
    ctx_pin = ctx_h.pin_memory()
    out_pin = mt.empty(nb, 4, H, W, dtype="bfloat16").pin_memory()
    xd = mt.empty(nb, 4, H, W, dtype="bfloat16", device=dev)
    cd = mt.empty(nb, CTX, 768, dtype="bfloat16", device=dev)
    h2d = (lat_pin.numel() + ctx_pin.numel()) * 2
    d2h = out_pin.numel() * 2
    if dist:
        dist.barrier()
    mt.cuda.synchronize()
    e2, e3 = mt.cuda.Event(), mt.cuda.Event()
    e2.record(stream)
    if use_graph:  # copy straight into the graph's static input buffers
        xd, cd = graphed.static_in[0], graphed.static_in[2]
    for i in range(args.steps):
        lib.mt_cuda_memcpy(xd.data_ptr(), lat_pin.data_ptr(), h2d - ctx_pin.numel() * 2, 0, stream.cuda_stream)
        lib.mt_cuda_memcpy(cd.data_ptr(), ctx_pin.data_ptr(), ctx_pin.numel() * 2, 0, stream.cuda_stream)
        t = sched.timesteps[i % len(sched.timesteps)]
        te = temb_all[i % len(temb_all)]
        eps = graphed(xd, te, cd) if use_graph else unet(xd, te, cd)
        y = sched.step(xd, eps, t)
        lib.mt_cuda_memcpy(out_pin.data_ptr(), y.data_ptr(), d2h, 1, stream.cuda_stream)
        stream.synchronize()
    e3.record(stream)
    mt.cuda.synchronize()
    ms_e2e = e2.elapsed_time(e3)
    if dist:
        tt = torch.tensor([ms_e2e])
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms_e2e = float(tt.item())
    e2e = {"value": 1000.0 * args.steps / ms_e2e, "unit": "steps/s", "h2d_bytes_per_step": h2d * world,
           "d2h_bytes_per_step": d2h * world}

    # ---- rooflines: the dominant kernel (level-0 flash attention) and the 3x3 conv ----
    hbm, tf_burst, tf_sust, peak_kind = peaks()

    def timed(fn, reps=10):
        for _ in range(3):
            fn()
        ev = [mt.cuda.Event() for _ in range(2)]
        mt.cuda.synchronize()
        ev[0].record(stream)
        for _ in range(reps):
            fn()
        ev[1].record(stream)
        mt.cuda.synchronize()
        return ev[0].elapsed_time(ev[1]) / reps

    # self-attention of the 64x64 level: 8 heads x 4096 tokens x head dim 40 (Q, K, V, O 168 MB
    # each at nb = 64, > L2); the same kernel the UNet launches for these shapes
    q, k, v = (mt.empty(nb, 8, H * W, 40, dtype="bfloat16", device=dev).uniform_(-1, 1) for _ in range(3))
    attn_ms = timed(lambda: mt.scaled_dot_product_attention(q, k, v))
    attn_flops = 4.0 * nb * 8 * (H * W) ** 2 * 40
    achieved = attn_flops / (attn_ms * 1e-3) / 1e12
    del q, k, v
    # per-launch DRAM bytes of one ncu capture at nb = 64, scaled by nb
    traffic = DRAM_BYTES_PER_SAMPLE["attn"] * nb
    roofline = {"bound": "tensor", "kernel": f"fa_lazy_sm100_kernel<48,48,bf16,sumcol> (8 heads x 4096 x 40, "
                f"batch {nb})", "achieved": achieved, "peak": tf_burst, "unit": "TFLOP/s",
                "frac": achieved / tf_burst, "peak_kind": f"{peak_kind} bf16 burst", "traffic": traffic,
                "algorithmic_bytes": 4 * nb * 8 * H * W * 40 * 2, "ms_per_launch": attn_ms,
                "step_tflops": unet_flops_per_sample() * nb / (ms_per_step * 1e-3) / 1e12}
    conv = unet.down[0].conv2  # 320 -> 320, 3x3 at 64x64 (the UNet's most frequent conv shape)
    xin = mt.empty(nb, 320, H, W, dtype="bfloat16", device=dev).uniform_(-1, 1).contiguous(
        memory_format=mt.channels_last)
    conv_ms = timed(lambda: conv(xin))  # input 168 MB at nb = 64 > L2
    conv_ach = 2.0 * nb * H * W * 320 * 320 * 9 / (conv_ms * 1e-3) / 1e12
    roofline_conv = {"bound": "tensor", "kernel": f"gemm_sm100_kernel<320,bf16,implicit conv> (3x3 320->320, "
                     f"64x64, batch {nb})", "achieved": conv_ach, "peak": tf_burst, "unit": "TFLOP/s",
                     "frac": conv_ach / tf_burst, "peak_kind": f"{peak_kind} bf16 burst",
                     "traffic": DRAM_BYTES_PER_SAMPLE["conv"] * nb, "ms_per_launch": conv_ms}

    # memory-bound kernels of the step at the 64x64 level (activation [nb*4096, 320] bf16, > L2 at
    # nb = 64): GroupNorm + SiLU and LayerNorm, one read and one write of the activation each
    xg = mt.empty(nb, 320, H, W, dtype="bfloat16", device=dev).uniform_(-1, 1).contiguous(
        memory_format=mt.channels_last)
    gn = unet.down[0].norm1
    ln = unet.down[1].block.norm1
    act_bytes = 2.0 * nb * H * W * 320 * 2
    gn_ms = timed(lambda: gn(xg, fuse_silu=True))
    ln_ms = timed(lambda: ln(xg.permute(0, 2, 3, 1).reshape(nb * H * W, 320)))
    del xg
    roofline_hbm = {"bound": "hbm", "unit": "GB/s", "peak": hbm, "peak_kind": f"{peak_kind} copy bandwidth",
                    "algorithmic_bytes": act_bytes}
    for key, kms, kname in (("group_norm_silu", gn_ms, "gn_partial_persist + gn_finalize_table + gn_apply_img"),
                            ("layer_norm", ln_ms, "layer_norm_bf16_persist_kernel")):
        roofline_hbm[key] = {"kernel": kname, "ms_per_call": kms, "achieved": act_bytes / (kms * 1e-3) / 1e9,
                             "frac": act_bytes / (kms * 1e-3) / 1e9 / hbm}

    # ---- N-GPU result vs a 1-GPU run of the whole batch (rank 0, untimed): the sharded latents
    # after W + K steps must equal, bit for bit, the same steps on all 64 samples on one GPU ----
    bitwise = None
    if dist:
        if rank == 0:
            del graphed
            x64 = lat_all.to("bfloat16").to(dev)
            ctx64 = ctx_all.to("bfloat16").to(dev)
            temb64 = [mt.tensor(timestep_embedding(np.full(gb, float(t))), dtype="bfloat16", device=dev)
                      for t in sched.timesteps]
            g64 = Graphed(unet, x64, temb64[0], ctx64) if use_graph else None
            for i in range(args.warmup + args.steps):
                te = temb64[i % len(temb64)]
                eps = g64(x64, te, ctx64) if use_graph else unet(x64, te, ctx64)
                x64 = sched.step(x64, eps, sched.timesteps[i % len(sched.timesteps)])
            mt.cuda.synchronize()
            ref = x64.contiguous().to("cpu")._buf[:x64.numel()]
            bitwise = bool(np.array_equal(ref, gathered.to("cpu")._buf[:gathered.numel()]))
        dist.barrier()

    clk = clock_summary([out_dir / f"clocks_rank{r}.csv" for r in range(world)]) if rank == 0 else None
    if rank == 0:
        # the attention kernel is bound by the exponential unit: 16 ex2 per SM per clock (the
        # same for .f32 / .f16x2 / .bf16x2, measured), at the median SM clock of the timed region
        # on the GPUs that ran it
        if clk and clk["samples"] > 0:
            mhz = clk["sm_mhz"]
            exp_rate = nb * 8 * float(H * W) ** 2 / (attn_ms * 1e-3)
            exp_peak = 16.0 * 148 * mhz * 1e6
            roofline["exp_unit"] = {"achieved": exp_rate, "peak": exp_peak, "unit": "exp2/s",
                                    "frac": exp_rate / exp_peak, "sm_mhz": mhz}
        base = None
        if world == 1 and gb == BATCH and not args.no_cpu_baseline:  # reference CPU path, bounded sample
            try:
                procs = os.cpu_count() or 1
                times, smp = cpu_sampled_steps(procs, 1, 2)
                base = cpu_result(times, smp, procs)
            except Exception as e:  # noqa: BLE001
                base = {"value": None, "unit": "steps/s", "cores": 0, "kind": "unavailable", "sample": str(e)[:200]}
        line = {"metric": METRIC, "value": value, "unit": "steps/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) latents/context, random-init "
                "weights)", "config": {"workload": f"C5: SD-1.5 UNet bf16, batch {gb} latents [{gb},4,64,64], "
                f"context [{gb},77,768], 1 UNet eval + DDIM update per step", "model": "SD-1.5-shaped UNet (859.5M params)",
                "global_batch": gb, "seq_len": H * W, "parallelism": f"batch-shard dp{world} + NCCL all-gather",
                "l2": "activations > L2 (126 MB) at batch 64/GPU; no flush"},
                "gpu_launches": int(launches), "e2e": e2e, "roofline": roofline, "roofline_conv": roofline_conv,
                "roofline_hbm": roofline_hbm,
                "cpu_baseline": base, "bitwise_equal_to_1gpu": bitwise,
                "clocks": clk}
        print(json.dumps(line))
    if comm:
        comm.close()
    if dist:
        dist.destroy_process_group()


def run_kernel(args):
    """One hot kernel alone at its level-0 UNet shape: `steps` timed launches after `warmup`,
    CUDA events on the library stream.  Used for ncu captures of a single kernel."""

    import mtorch_b200 as mt
    from mtorch_b200 import _lib, ops

    nb = args.batch
    stream = mt.cuda.current_stream()
    mt.manual_seed(0)
    if args.kernel == "conv":
        conv = mt.nn.Conv2d(320, 320, 3, padding=1, device="cuda", dtype="bfloat16")
        x = mt.empty(nb, 320, H, W, dtype="bfloat16", device="cuda").uniform_(-1, 1).contiguous(
            memory_format=mt.channels_last)
        fn = lambda: conv(x)  # noqa: E731
        flops = 2.0 * nb * H * W * 320 * 320 * 9
        name = "implicit-GEMM conv 3x3 320->320 at 64x64"
    elif args.kernel in ("gn", "ln"):
        x = mt.empty(nb, 320, H, W, dtype="bfloat16", device="cuda").uniform_(-1, 1).contiguous(
            memory_format=mt.channels_last)
        if args.kernel == "gn":
            gn = mt.nn.GroupNorm(32, 320, device="cuda", dtype="bfloat16")
            fn = lambda: gn(x, fuse_silu=True)  # noqa: E731
            name = "GroupNorm(32) + SiLU, 320 channels at 64x64, channels-last"
        else:
            ln = mt.nn.LayerNorm(320, device="cuda", dtype="bfloat16")
            t = x.permute(0, 2, 3, 1).reshape(nb * H * W, 320)
            fn = lambda: ln(t)  # noqa: E731
            name = "LayerNorm over 320 columns, 64x64 tokens"
        flops = None
        nbytes = 2.0 * nb * H * W * 320 * 2  # one read + one write of the activation
    elif args.kernel == "geglu":
        x = mt.empty(nb * H * W, 320, dtype="bfloat16", device="cuda").uniform_(-1, 1)
        w = mt.empty(2560, 320, dtype="bfloat16", device="cuda").uniform_(-0.05, 0.05)
        fn = lambda: ops.linear(x, w, None, epilogue=_lib.EPI_GEGLU)  # noqa: E731
        flops = 2.0 * nb * H * W * 320 * 2560
        name = "GEGLU linear 320->2x1280 over 64x64 tokens"
    else:
        q, k, v = (mt.empty(nb, 8, H * W, 40, dtype="bfloat16", device="cuda").uniform_(-1, 1) for _ in range(3))
        fn = lambda: mt.scaled_dot_product_attention(q, k, v)  # noqa: E731
        flops = 4.0 * nb * 8 * (H * W) ** 2 * 40
        name = "flash attention, 8 heads x 4096 tokens x 40"
    for _ in range(args.warmup):
        fn()
    mt.cuda.synchronize()
    e0, e1 = mt.cuda.Event(), mt.cuda.Event()
    e0.record(stream)
    for _ in range(args.steps):
        fn()
    e1.record(stream)
    mt.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    hbm, tf_burst, _, kind = peaks()
    if flops is None:
        gbs = nbytes / (ms * 1e-3) / 1e9
        print(json.dumps({"kernel": name, "batch": nb, "ms_per_launch": ms, "GB/s": gbs, "frac_of_hbm": gbs / hbm,
                          "algorithmic_bytes": nbytes, "peak_kind": kind}))
        return
    tflops = flops / (ms * 1e-3) / 1e12
    print(json.dumps({"kernel": name, "batch": nb, "ms_per_launch": ms, "tflops": tflops,
                      "frac_of_bf16_peak": tflops / tf_burst, "peak_kind": kind}))


def run_workload(args):
    """The §8(f) workloads around the UNet, one GPU, device-timed (CUDA events on the library's
    stream, after `warmup` untimed runs), each as one JSON line with its FLOP rate against the
    measured bf16 peak:
      sampler  guided denoising (classifier-free guidance 7.5) of `batch` latents: the UNet on the
               doubled batch, device timestep embedding and the fused guidance + DDIM kernel, one
               CUDA graph per step; unit = denoise steps/s of the whole batch
      vae      SD-1.5 VAE decode of `batch` latents 64x64 -> 512x512 images; unit = images/s
      text     SD-1.5 CLIP text encoder on `batch` sequences of 77 tokens; unit = sequences/s
      c4       BASELINE config C4: the fp32 UNet on one latent, one UNet eval + DDIM update (CUDA
               graph); unit = steps/s, beside the reference CPU path on the same per-sample work
      c1-c3    BASELINE configs C1 (fp32 matmul 2048^2), C2 (fp32 ResNet block), C3 (bf16 attention
               block), beside the reference CPU path computing each in full (see run_config)"""

    import mtorch_b200 as mt

    stream = mt.cuda.current_stream()
    nb = args.batch
    mt.manual_seed(0)
    base = None
    if args.workload in ("c1", "c2", "c3"):
        run_config(args)
        return
    if args.workload == "c4":
        from mtorch_b200.graphs import Graphed
        from mtorch_b200.unet import DDIM, UNet, timestep_embedding, unet_flops_per_sample

        nb = 1
        unet = UNet(device="cuda", dtype="float32")
        mt.manual_seed(1)
        lat = mt.randn(1, 4, H, W).cuda()
        ctx = mt.randn(1, CTX, 768).cuda()
        temb = mt.tensor(timestep_embedding(np.array([999.0]))).cuda()
        sched = DDIM(steps=50)
        g = Graphed(unet, lat, temb, ctx)
        fn = lambda: sched.step(lat, g(lat, temb, ctx), 999)  # noqa: E731
        flops, unit = unet_flops_per_sample(), "steps/s"
        name = "C4: SD-1.5 UNet fp32 (3xTF32 GEMM/conv, fp32 SIMT attention), batch 1, one UNet eval + DDIM update"
        if not args.no_cpu_baseline:
            procs = os.cpu_count() or 1
            times, smp = cpu_sampled_steps(procs, 1, 2)
            base = cpu_result(times, smp, procs)
            base["value"] *= BATCH  # one sample per C4 step
            base["sample"] += "; C4 step = R sampled steps"
    elif args.workload == "sampler":
        from mtorch_b200.unet import DDIM, Sampler, UNet, unet_flops_per_sample

        unet = UNet(device="cuda", dtype="bfloat16")
        mt.manual_seed(1)
        lat = mt.randn(nb, 4, H, W).to("bfloat16").cuda()
        ctx = mt.randn(nb, CTX, 768).to("bfloat16").cuda()
        unc = mt.randn(nb, CTX, 768).to("bfloat16").cuda()
        sampler = Sampler(unet, DDIM(steps=50), ctx, uncond_ctx=unc, guidance_scale=7.5, graph=True)
        fn = lambda: sampler(lat, steps=1)  # noqa: E731
        flops, unit = unet_flops_per_sample() * 2 * nb, "denoise steps/s"
        name = f"guided denoise step, {nb} latents (UNet batch {2 * nb}), CUDA graph"
    elif args.workload == "vae":
        from mtorch_b200.vae import VAEDecoder, vae_decoder_flops

        dec = VAEDecoder(device="cuda", dtype="bfloat16")
        z = mt.randn(nb, 4, H, W).to("bfloat16").cuda()
        fn = lambda: dec(z)  # noqa: E731
        flops, unit = vae_decoder_flops(H, W) * nb, "images/s"
        name = f"SD-1.5 VAE decode, {nb} latents 64x64 -> 512x512"
    else:
        from mtorch_b200.text_encoder import CLIPTextEncoder, clip_text_flops

        enc = CLIPTextEncoder(device="cuda", dtype="bfloat16")
        ids = mt.tensor((np.arange(nb * CTX).reshape(nb, CTX) * 7919) % 49408)
        fn = lambda: enc(ids)  # noqa: E731
        flops, unit = clip_text_flops() * nb, "sequences/s"
        name = f"SD-1.5 CLIP text encoder, {nb} x 77 tokens"
    for _ in range(max(args.warmup, 1)):
        fn()
    mt.cuda.synchronize()
    e0, e1 = mt.cuda.Event(), mt.cuda.Event()
    e0.record(stream)
    for _ in range(args.steps):
        fn()
    e1.record(stream)
    mt.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    _, tf_burst, tf_sust, kind = peaks()
    tflops = flops / (ms * 1e-3) / 1e12
    per = 1 if args.workload in ("sampler", "c4") else nb
    line = {"workload": name, "value": 1000.0 * per / ms, "unit": unit, "ms_per_run": ms, "batch": nb,
            "dtype": "f32" if args.workload == "c4" else "bf16", "data": "synthetic, random-init weights",
            "tflops": tflops, "frac_of_bf16_peak": tflops / tf_burst, "peak_kind": f"{kind} bf16 burst"}
    if args.workload == "c4":
        line["note"] = ("fp32 throughput is bounded by 3xTF32 (three tf32 MMAs per product) and fp32 SIMT attention; "
                        "frac is against the bf16 peak for reference only")
    if base is not None:
        line["cpu_baseline"] = base
    print(json.dumps(line))


def run_config(args):
    """BASELINE configs C1-C3 on one GPU (CUDA events, `steps` runs after `warmup`), beside the
    reference's own CPU path computing the same configuration in full on all host cores (each op
    cut into row slices spread over single-threaded processes; oracle/cpu_bench.FullRun)."""

    import mtorch_b200 as mt
    from mtorch_b200 import ops
    from mtorch_b200.unet import BasicTransformerBlock

    stream = mt.cuda.current_stream()
    mt.manual_seed(0)
    if args.workload == "c1":
        a = mt.randn(2048, 2048).cuda()
        b = mt.randn(2048, 2048).cuda()
        fn = lambda: mt.matmul(a, b)  # noqa: E731
        flops, name, dtype = 2.0 * 2048 ** 3, "C1: fp32 matmul 2048 x 2048 x 2048 (3xTF32)", "f32"
    elif args.workload == "c2":
        x = mt.randn(2, 320, 64, 64).cuda().contiguous(memory_format=mt.channels_last)
        gn1, gn2 = mt.nn.GroupNorm(32, 320, device="cuda"), mt.nn.GroupNorm(32, 320, device="cuda")
        c1 = mt.nn.Conv2d(320, 320, 3, padding=1, device="cuda")
        c2 = mt.nn.Conv2d(320, 320, 3, padding=1, device="cuda")
        fn = lambda: c2(gn2(c1(gn1(x, fuse_silu=True)), fuse_silu=True), residual=x)  # noqa: E731
        flops, name, dtype = 2 * 2.0 * 2 * 4096 * 320 * 320 * 9, "C2: SD ResNet block fp32, [2, 320, 64, 64]", "f32"
    else:
        blk = BasicTransformerBlock(320, 8, 768, device="cuda", dtype="bfloat16")
        h = mt.randn(2 * 4096, 320).to("bfloat16").cuda()
        ctx = mt.randn(2, 77, 768).to("bfloat16").cuda()
        fn = lambda: blk(h, ctx, 2, 4096)  # noqa: E731
        from oracle.cpu_bench import config_ops, op_flops

        flops = sum(op_flops(o) for o in config_ops("c3"))
        name, dtype = "C3: SD attention block bf16 (self 4096 + cross 77 + GEGLU FFN), [2, 4096, 320]", "bf16"
    for _ in range(max(args.warmup, 3)):
        fn()
    mt.cuda.synchronize()
    e0, e1 = mt.cuda.Event(), mt.cuda.Event()
    e0.record(stream)
    for _ in range(args.steps):
        fn()
    e1.record(stream)
    mt.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    _, tf_burst, _, kind = peaks()
    tflops = flops / (ms * 1e-3) / 1e12
    line = {"workload": name, "value": 1000.0 / ms, "unit": "runs/s", "ms_per_run": ms, "dtype": dtype,
            "data": "synthetic (mtorch.manual_seed(0) N(0,1) inputs), random-init weights", "tflops": tflops,
            "frac_of_bf16_peak": tflops / tf_burst, "peak_kind": f"{kind} bf16 burst"}
    if not args.no_cpu_baseline:
        from oracle import cpu_bench

        procs = os.cpu_count() or 1
        run = cpu_bench.FullRun(args.workload, procs)
        try:
            run.step()
            times = [run.step() for _ in range(2)]
        finally:
            run.close()
        sec = statistics.median(times)
        line["cpu_baseline"] = {"value": 1.0 / sec, "unit": "runs/s", "cores": procs, "kind": run.kind,
                                "sample": run.describe(f"{args.workload.upper()} in full",
                                                      "one run = 1") + f"; median {sec:.2f} s per run",
                                "gflops_per_s": run.full_flops / run.r / sec / 1e9}
    print(json.dumps(line))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--eager", action="store_true", help="launch the UNet op by op instead of replaying a CUDA graph")
    ap.add_argument("--kernel", choices=["conv", "attn", "geglu", "gn", "ln"], default=None,
                    help="time one hot kernel alone at its UNet shape (for profiling), not the UNet")
    ap.add_argument("--batch", type=int, default=BATCH, help="samples for --kernel / --workload runs")
    ap.add_argument("--global-batch", type=int, default=BATCH,
                    help="UNet bench: samples of the whole job (64 = config C5; smaller for profiling)")
    ap.add_argument("--no-cpu-baseline", action="store_true", help="skip the reference CPU timing (cpu_baseline)")
    ap.add_argument("--workload", choices=["sampler", "vae", "text", "c1", "c2", "c3", "c4"], default=None,
                    help="time one of the workloads around the UNet instead of the UNet step")
    args = ap.parse_args()
    if args.workload:
        run_workload(args)
    elif args.kernel:
        run_kernel(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
