"""Benchmark: restored Mpx/s per B200 for MAXIM-3S on 1280x853 images.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--impl native|reference]
    python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N ...   (N > 1)

Workload (BASELINE metric, config: MAXIM-3S, 1280x853; at N=1 also the
metric's 2048x2048 latency, BASELINE config 4, as `latency_2048`, and the
MAXIM-2S throughput of config 5 as `config5_s2`):
  * MAXIM-3S with seeded random-init He-normal weights (no checkpoint offline);
  * each GPU runs B distinct synthetic 1280x853 images (U[0,1), padded by the
    reference pipeline to 1280x896) per step; a step is one forward pass of
    the plan over each of them; images are independent, so ranks shard them
    with no collective (weak scaling: per-GPU work is fixed as N grows);
  * Mpx counts OUTPUT pixels (1280*853 per image).
`value`: inputs resident in HBM, timed with CUDA events on the executor's
stream, max over ranks. `e2e`: the same through the C ABI's mx_gpu_run from
pinned host memory (H2D of the image and D2H of the result inside the timed
region). Each pass touches a 2012 MiB arena, far beyond the 126 MB L2, so no
L2 flush is needed between passes.

`--impl reference` times the reference's CPU algorithm on this box's host cores
(the C++ restatement of its exec_cpu.rs: the Rust original cannot be built
offline) on a bounded sample of the same workload.
"""
import argparse
import importlib
import json
import os
import re
import statistics
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

VARIANT, W_SEED, IN_SEED = "S-3", 1, 4
IMG_W, IMG_H = 1280, 853
PAD_H, PAD_W = 896, 1280
OUT_MPX = IMG_W * IMG_H / 1e6
METRIC = "restored Mpx/s per B200 (MAXIM-3S, 1280x853) at 1/2/4/8 GPUs; 2048² latency"


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p["hbm_gbs"], p["bf16_tflops"], p.get("bf16_tflops_sustained", p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, 1400.0, "fallback"


class Clocks:
    """Samples SM clock and throttle reasons of one GPU while running."""

    FIELDS = ("uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid):
        self.uuid, self.rows, self.proc = uuid, [], None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "--query-gpu=" + self.FIELDS, "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9 and (not self.uuid or parts[0] == self.uuid):
                self.rows.append(parts)

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


def shard(n, rank, world):
    """The stream indices of this rank's n images: image i of the one seeded
    stream goes to rank i % world (replicas, no image is split)."""
    return [rank + world * k for k in range(n)]


def max_over_ranks(x, world, device=None):
    """The largest of x over all ranks (every rank passes its own x); the
    job's time is its slowest rank's."""
    if world <= 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(x)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def job_mpx_per_s(images_per_rank, world, seconds):
    """Whole-job throughput: every rank's images, over the slowest rank's time."""
    return images_per_rank * world * OUT_MPX / seconds


def make_images(n, rank, world):
    """This rank's share of one seeded image stream (see shard)."""
    synth = importlib.import_module("maxim-rs_b200.synth")
    mx = importlib.import_module("maxim-rs_b200")
    rng = synth.input_rng(IN_SEED)
    want = set(shard(n, rank, world))
    out = []
    for i in range(max(want) + 1):
        img = synth.image_uniform(rng, IMG_H, IMG_W)
        if i in want:
            padded, _ = mx.preprocess(img, 64)
            out.append(padded)
    return out


def checkpoint_path():
    synth = importlib.import_module("maxim-rs_b200.synth")
    d = os.path.join(tempfile.gettempdir(), "maxim_b200_bench")
    os.makedirs(d, exist_ok=True)
    path = os.path.join(d, "%s_seed%d.safetensors" % (VARIANT, W_SEED))
    synth.checkpoint(path, VARIANT, W_SEED)
    return path


def cpu_sample(threads, budget_s=20.0):
    """Time the CPU oracle on a bounded sample of the workload: MAXIM-3S on the
    largest image size whose estimated time fits the budget (FLOPs per padded
    pixel are size independent for this model), extrapolated to a 1280x853
    image by padded pixels. Returns (Mpx/s, sample description)."""
    mx = importlib.import_module("maxim-rs_b200")
    synth = importlib.import_module("maxim-rs_b200.synth")
    oracle = importlib.import_module("oracle")
    work = importlib.import_module("maxim-rs_b200.work")
    w = mx.Weights(checkpoint_path())
    probe = mx.Plan(w, 128, 128)
    img = synth.image_uniform(synth.input_rng(IN_SEED), 128, 128)
    t = time.perf_counter()
    oracle.output(probe, img, threads)
    rate = (128 * 128) / (time.perf_counter() - t)  # padded px / s
    h, wd = 128, 128
    for (hh, ww) in [(448, 640), (320, 448), (256, 384), (192, 256)]:
        if hh * ww / rate <= budget_s:
            h, wd = hh, ww
            break
    plan = mx.Plan(w, h, wd)
    img = synth.image_uniform(synth.input_rng(IN_SEED), h, wd)
    t = time.perf_counter()
    oracle.output(plan, img, threads)
    dt = time.perf_counter() - t
    per_image = dt * (PAD_H * PAD_W) / (h * wd)
    gflop = sum(v[1] for v in work.census(plan).values()) / 1e9
    desc = ("MAXIM-3S forward on one %dx%d image (%.0f GFLOP, %.1f s), extrapolated by padded pixels to a "
            "1280x853 image (1280x896 padded)" % (wd, h, gflop, dt))
    return OUT_MPX / per_image, desc, dt


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    threads = len(os.sched_getaffinity(0))
    importlib.import_module("__graft_entry__").build()
    times = []
    desc = ""
    for step in range(args.warmup + args.steps):
        v, desc, dt = cpu_sample(threads)
        if step >= args.warmup:
            times.append(OUT_MPX / v)  # seconds per full image
    value = args.steps / sum(times) if times else 0.0
    line = {"metric": METRIC, "value": value, "unit": "Mpx/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1000.0 * sum(times) / max(len(times), 1),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "impl": "reference",
            "config": {"workload": "MAXIM-3S 1280x853 (padded 1280x896), random-init He-normal weights seed %d"
                                   % W_SEED, "images_per_step": 1, "parallelism": "host threads"},
            "cpu_baseline": {"value": value, "unit": "Mpx/s", "cores": threads, "kind": "port",
                             "sample": desc + "; the reference's exec_cpu.rs restated in C++ (oracle/exec_cpu.cpp)"},
            "e2e": {"value": value, "unit": "Mpx/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def traffic_from_profiles(kind):
    """Per-launch DRAM bytes of `kind` from the committed ncu summary, if any."""
    p = os.path.join(ROOT, "profiles")
    if not os.path.isdir(p):
        return None
    for f in sorted(os.listdir(p)):
        if f.endswith(".md"):
            for line in open(os.path.join(p, f)):
                m = re.match(r"\s*traffic_bytes_per_launch\[%s\]\s*:\s*([0-9.eE+]+)" % re.escape(kind), line)
                if m:
                    return float(m.group(1))
    return None


def run_timeline(args):
    """Per-op-family device time of one pass (CUDA events around every op on
    the executor's stream), plus the most expensive op shapes. The same
    census the reference's `--profile` prints (src/main.rs:586-656)."""
    import collections
    mx = importlib.import_module("maxim-rs_b200")
    work = importlib.import_module("maxim-rs_b200.work")
    synth = importlib.import_module("maxim-rs_b200.synth")
    path = checkpoint_path() if args.variant == VARIANT else os.path.join(
        tempfile.gettempdir(), "maxim_b200_%s.safetensors" % args.variant)
    synth.checkpoint(path, args.variant, W_SEED)
    img = synth.image_uniform(synth.input_rng(IN_SEED), args.height, args.width)
    padded, _ = mx.preprocess(img, 64)
    plan = mx.Plan(mx.Weights(path), padded.shape[1], padded.shape[2])
    gpu = mx.Gpu(plan)
    for _ in range(args.warmup):
        gpu.run(padded)
    gpu.set_timeline(True)
    gpu.run(padded)
    per, tot = gpu.timeline()
    st = gpu.stats()
    ops = plan.ops()
    fam = collections.defaultdict(lambda: [0, 0.0, 0, 0])
    shp = collections.defaultdict(lambda: [0, 0.0, 0, 0])
    prim, flags = gpu.schedule(flags=True)
    for p, members in work.schedule_steps(prim).items():
        o = ops[p]
        k, f, b = work.step_work(plan, ops, members, flags)
        kind = work.KINDS[o.kind]
        if kind in ("conv1x1", "conv3x3", "conv4x4s2", "convt2x2"):
            d = "%s %d->%d @%dx%d" % (k, o.c_in, o.c_out, o.h, o.wd)
        elif kind == "gate_mm":
            d = "%s c=%d %dx%d mode%d" % (k, o.c, o.outer, o.inner, o.mode)
        else:
            c, h, w = plan.buf(o.dst)
            d = "%s %dx%dx%d" % (k, c, h, w)
        for tab, key in ((fam, k), (shp, d)):
            e = tab[key]
            e[0] += 1
            e[1] += float(per[p])
            e[2] += f
            e[3] += b
    print("%s %dx%d (padded %dx%d): one pass %.2f ms, %d ops in %d steps (%d fused, %d permutations dropped), "
          "%d kernel launches" % (args.variant, args.width, args.height, padded.shape[2], padded.shape[1], tot,
                                  plan.n_ops, st["steps"], st["ops_fused"], st["perms_dropped"], st["kernels"]))
    print("%-26s %5s %9s %6s %9s %9s" % ("step family", "steps", "ms", "share", "TFLOP/s", "GB/s"))
    for k, (n, ms, f, b) in sorted(fam.items(), key=lambda kv: -kv[1][1]):
        ms_ = max(ms, 1e-9)
        print("%-26s %5d %9.2f %5.1f%% %9.1f %9.0f" % (k, n, ms, 100 * ms / tot, f / ms_ / 1e9, b / ms_ / 1e6))
    print("top shapes:")
    for k, (n, ms, f, b) in sorted(shp.items(), key=lambda kv: -kv[1][1])[:24]:
        ms_ = max(ms, 1e-9)
        print("  %8.2f ms %4dx  %-48s %7.1f TFLOP/s %6.0f GB/s" % (ms, n, k, f / ms_ / 1e9, b / ms_ / 1e6))
    gpu.close()
    return 0


def latency_2048(mx, local, reps=3, warmup=2):
    """BASELINE config 4, the metric's latency: MAXIM-3S with seed-3 weights
    on one 2048x2048 dark image (U[0,0.25) plus noise of std 0.02 sqrt(v),
    synth.image_dark), batch 1. `ms`: device time of one pass with the image
    already in HBM (CUDA events on the executor's stream, median of `reps`);
    `e2e_ms`: the same through mx_gpu_run from pinned host memory."""
    import torch
    synth = importlib.import_module("maxim-rs_b200.synth")
    d = os.path.join(tempfile.gettempdir(), "maxim_b200_bench")
    os.makedirs(d, exist_ok=True)
    path = os.path.join(d, "S-3_seed3.safetensors")
    synth.checkpoint(path, "S-3", 3)
    img = synth.image_dark(synth.input_rng(3), 2048, 2048)
    padded, _ = mx.preprocess(img, 64)
    plan = mx.Plan(mx.Weights(path), padded.shape[1], padded.shape[2])
    g = mx.Gpu(plan, device=local)
    arena_mib = g.stats()["arena_bytes"] / 2**20
    x = torch.from_numpy(np.ascontiguousarray(padded)).cuda(local)
    y = torch.empty(g.out_shape, dtype=torch.float32, device="cuda:%d" % local)
    stream = torch.cuda.ExternalStream(g.stream(), device=torch.device("cuda", local))

    def one():
        g.upload_input_device(x.data_ptr())
        g.enqueue()
        g.download_output_device(y.data_ptr())

    for _ in range(warmup):
        one()
    g.sync()
    dev = []
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        one()
        e1.record(stream)
        e1.synchronize()
        dev.append(e0.elapsed_time(e1))
    g.sync()
    pin_in = torch.from_numpy(np.ascontiguousarray(padded)).pin_memory()
    pin_out = torch.empty(g.out_shape, dtype=torch.float32).pin_memory()
    host = []
    for _ in range(reps):
        t0 = time.perf_counter()
        g.run(pin_in.numpy(), pin_out.numpy())
        host.append((time.perf_counter() - t0) * 1e3)
    finite = bool(np.isfinite(pin_out.numpy()).all())
    g.close()
    return {"ms": statistics.median(dev), "e2e_ms": statistics.median(host), "reps": reps,
            "config": "MAXIM-3S 2048x2048 (BASELINE config 4), seed-3 weights, one dark image, batch 1",
            "arena_mib": round(arena_mib, 1), "output_finite": finite}


def config5_s2(mx, local, n_img=4, reps=3, warmup=2):
    """BASELINE config 5 on one GPU: MAXIM-2S with seed-4 weights over 1280x853
    U[0,1) images (padded to 1280x896), in HBM, one pass per image; Mpx/s of
    output pixels by CUDA events on the executor's stream (the scaling over
    GPUs is the headline's, which runs the S-3 target)."""
    import torch
    synth = importlib.import_module("maxim-rs_b200.synth")
    d = os.path.join(tempfile.gettempdir(), "maxim_b200_bench")
    os.makedirs(d, exist_ok=True)
    path = os.path.join(d, "S-2_seed4.safetensors")
    synth.checkpoint(path, "S-2", 4)
    rng = synth.input_rng(4)
    imgs = [mx.preprocess(synth.image_uniform(rng, IMG_H, IMG_W), 64)[0] for _ in range(n_img)]
    plan = mx.Plan(mx.Weights(path), PAD_H, PAD_W)
    g = mx.Gpu(plan, device=local)
    x = torch.from_numpy(np.stack(imgs)).cuda(local)
    y = torch.empty((n_img,) + g.out_shape, dtype=torch.float32, device="cuda:%d" % local)
    stream = torch.cuda.ExternalStream(g.stream(), device=torch.device("cuda", local))

    def step():
        for b in range(n_img):
            g.upload_input_device(x[b].data_ptr())
            g.enqueue()
            g.download_output_device(y[b].data_ptr())

    for _ in range(warmup):
        step()
    g.sync()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        step()
    e1.record(stream)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / (reps * n_img)
    g.close()
    return {"value": OUT_MPX / (ms / 1000.0), "unit": "Mpx/s", "ms_per_image": ms,
            "config": "MAXIM-2S 1280x853 (BASELINE config 5, one GPU), seed-4 weights, U[0,1) images"}


def run_native(args):
    import torch
    import torch.distributed as dist

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        log("bench: --gpus %d but WORLD_SIZE %d; using WORLD_SIZE" % (args.gpus, world))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    importlib.import_module("__graft_entry__").build()
    mx = importlib.import_module("maxim-rs_b200")
    work = importlib.import_module("maxim-rs_b200.work")

    w = mx.Weights(checkpoint_path())
    plan = mx.Plan(w, PAD_H, PAD_W)
    gpu = mx.Gpu(plan, device=local)
    stats = gpu.stats()
    B = args.batch
    imgs = make_images(B, rank, world)
    in_dev = torch.from_numpy(np.stack(imgs)).cuda(local)
    out_dev = torch.empty((B,) + gpu.out_shape, dtype=torch.float32, device="cuda:%d" % local)
    stream = torch.cuda.ExternalStream(gpu.stream(), device=torch.device("cuda", local))

    def step():
        for b in range(B):
            gpu.upload_input_device(in_dev[b].data_ptr())
            gpu.enqueue()
            gpu.download_output_device(out_dev[b].data_ptr())

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        step()
    gpu.sync()
    torch.cuda.synchronize()
    barrier()
    uuid = str(getattr(torch.cuda.get_device_properties(local), "uuid", ""))
    uuid = ("GPU-" + uuid) if uuid and not uuid.startswith("GPU-") else uuid
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(uuid) as clk:
        torch.cuda.synchronize()
        ev0.record(stream)
        for _ in range(args.steps):
            step()
        ev1.record(stream)
        ev1.synchronize()
        gpu.sync()
        torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    barrier()
    ms = max_over_ranks(ms, world, "cuda:%d" % local)
    value = job_mpx_per_s(args.steps * B, world, ms / 1000.0)

    # e2e: the public API from pinned host memory, H2D + pass + D2H per image.
    pin_in = [torch.from_numpy(im).pin_memory() for im in imgs]
    pin_out = torch.empty((B,) + gpu.out_shape, dtype=torch.float32).pin_memory()
    gpu.run(pin_in[0].numpy(), pin_out[0].numpy())
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        for b in range(B):
            gpu.run(pin_in[b].numpy(), pin_out[b].numpy())
    e2e_s = time.perf_counter() - t0
    barrier()
    e2e_s = max_over_ranks(e2e_s, world, "cuda:%d" % local)
    e2e = job_mpx_per_s(args.steps * B, world, e2e_s)

    # Roofline of the dominant kernel family, from per-op CUDA events on the
    # executor's stream over one pass of the same workload.
    hbm, tf_burst, tf_sus, src = peaks()
    gpu.set_timeline(True)
    gpu.upload_input_device(in_dev[0].data_ptr())
    gpu.enqueue()
    per, total = gpu.timeline()
    gpu.set_timeline(False)
    fam = {}
    ops = plan.ops()
    prim, flags = gpu.schedule(flags=True)
    for p, members in work.schedule_steps(prim).items():
        k, f, b = work.step_work(plan, ops, members, flags)
        e = fam.setdefault(k, [0, 0.0, 0, 0])
        e[0] += 1
        e[1] += float(per[p])
        e[2] += f
        e[3] += b
    dom = max(fam, key=lambda k: fam[k][1])
    n_l, ms_tot, fl, by = fam[dom]
    avg_s = ms_tot / 1000.0 / n_l
    t_mem, t_tc = (by / n_l) / (hbm * 1e9), (fl / n_l) / (tf_sus * 1e12)
    if t_tc > t_mem:
        roof = {"bound": "tensor", "achieved": fl / n_l / avg_s / 1e12, "peak": tf_sus, "unit": "TFLOP/s"}
    else:
        roof = {"bound": "hbm", "achieved": by / n_l / avg_s / 1e9, "peak": hbm, "unit": "GB/s"}
    roof["frac"] = roof["achieved"] / roof["peak"]
    roof["traffic"] = traffic_from_profiles(dom)
    roof["kernel"] = dom
    roof["launches_per_pass"] = n_l
    roof["share_of_pass"] = ms_tot / total
    roof["peak_source"] = src + (" bf16 sustained" if roof["bound"] == "tensor" else " copy")
    roof["algorithmic_per_launch"] = {"flop": fl / n_l, "bytes": by / n_l}

    line = {"metric": METRIC, "value": value, "unit": "Mpx/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "MAXIM-3S 1280x853 (padded 1280x896), random-init He-normal weights seed %d, "
                                   "U[0,1) images" % W_SEED, "images_per_gpu_per_step": B,
                       "parallelism": "replicas x%d (images sharded, no collective)" % world,
                       "l2": "no flush: each pass streams a 2012 MiB arena (L2 is 126 MB)"},
            "e2e": {"value": e2e, "unit": "Mpx/s", "h2d_bytes_per_step": int(B * in_dev[0].numel() * 4),
                    "d2h_bytes_per_step": int(B * out_dev[0].numel() * 4)},
            "gpu_launches": int(stats["kernels"] * args.steps * B),
            "roofline": roof, "clocks": clk.summary()}
    if rank == 0 and world == 1:
        with Clocks(uuid) as clk4:
            line["latency_2048"] = latency_2048(mx, local)
        line["latency_2048"]["clocks"] = clk4.summary()
        with Clocks(uuid) as clk5:
            line["config5_s2"] = config5_s2(mx, local)
        line["config5_s2"]["clocks"] = clk5.summary()
    if rank == 0 and world == 1 and not args.no_cpu:
        threads = len(os.sched_getaffinity(0))
        v, desc, _ = cpu_sample(threads)
        line["cpu_baseline"] = {"value": v, "unit": "Mpx/s", "cores": threads, "kind": "port",
                                "sample": desc + "; oracle/exec_cpu.cpp, the reference's exec_cpu.rs in C++"}
    gpu.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--batch", type=int, default=4, help="images per GPU per step")
    ap.add_argument("--impl", choices=["native", "reference"], default="native")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--timeline", action="store_true",
                    help="print the per-op-family device time of one pass and exit (no JSON line)")
    ap.add_argument("--variant", default=VARIANT, help="--timeline only: model variant")
    ap.add_argument("--height", type=int, default=IMG_H, help="--timeline only: image height")
    ap.add_argument("--width", type=int, default=IMG_W, help="--timeline only: image width")
    args = ap.parse_args()
    if args.warmup < 3:
        log("bench: raising --warmup to 3")
        args.warmup = 3
    if args.timeline:
        return run_timeline(args)
    if args.impl == "reference":
        return run_reference(args)
    return run_native(args)


if __name__ == "__main__":
    sys.exit(main())
