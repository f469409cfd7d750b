"""Benchmark: restored Mpx/s per B200 for MAXIM-3S on 1280x853 images.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--impl native|reference]
    python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N ...   (N > 1)

Workload (BASELINE metric, config: MAXIM-3S, 1280x853; at N=1 also the
metric's 2048x2048 latency, BASELINE config 4, as `latency_2048`, and the
MAXIM-2S throughput of config 5 as `config5_s2`):
  * MAXIM-3S with seeded random-init He-normal weights (no checkpoint offline);
  * each GPU runs B (default 1) distinct synthetic 1280x853 images (U[0,1), padded by the
    reference pipeline to 1280x896) per step; a step is one forward pass of
    the plan over each of them; images are independent, so ranks shard them
    with no collective (weak scaling: per-GPU work is fixed as N grows);
  * Mpx counts OUTPUT pixels (1280*853 per image).
`value`: inputs resident in HBM, timed with CUDA events on the executor's
stream, max over ranks. `e2e`: the same through the C ABI's batch runner
(mx_batch_run) from the caller's host arrays (the copy into pinned staging,
the H2D of the image and the D2H of the result inside the timed region). Each pass touches a 1.9 GB arena, far beyond the 126 MB L2, so no
L2 flush is needed between passes. `value` is the whole job's (all ranks);
`value_per_gpu` is value / n_gpus, the metric's per-B200 figure.

`--impl reference` times the reference's CPU algorithm on this box's host cores
(the C++ restatement of its exec_cpu.rs: the Rust original cannot be built
offline) on whole images of the same workload, through the oracle library
alone (the GPU product library is never mapped into that process).
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


def make_images(n, rank, world, pre=None):
    """This rank's share of one seeded image stream (see shard). `pre` pads an
    image as the reference pipeline does (default: the product library's)."""
    synth = importlib.import_module("maxim-rs_b200.synth")
    if pre is None:
        pre = importlib.import_module("maxim-rs_b200").preprocess
    rng = synth.input_rng(IN_SEED)
    want = set(shard(n, rank, world))
    out = []
    for i in range(max(want) + 1):
        img = synth.image_uniform(rng, IMG_H, IMG_W)
        if i in want:
            padded, _ = pre(img, 64)
            out.append(padded)
    return out


def bench_config(B):
    """The workload both arms run (identical dict on both lines)."""
    return {"workload": "MAXIM-3S 1280x853 (padded 1280x896), random-init He-normal weights seed %d, U[0,1) images"
                        % W_SEED,
            "images_per_gpu_per_step": B,
            "parallelism": "replicas (images sharded round-robin over ranks, one arena per GPU, no collective)",
            "l2": "no flush: each pass streams a 1.9 GB arena (L2 is 126 MB)"}


def checkpoint_path(spec=None):
    """The bench checkpoint (written once per box). `spec` is the parameter
    inventory to generate from; by default the product library's builder's,
    which is the same list the oracle library's own copy of the builder gives."""
    synth = importlib.import_module("maxim-rs_b200.synth")
    d = os.path.join(tempfile.gettempdir(), "maxim_b200_bench")
    os.makedirs(d, exist_ok=True)
    path = os.path.join(d, "%s_seed%d.safetensors" % (VARIANT, W_SEED))
    synth.checkpoint(path, VARIANT, W_SEED, spec=spec)
    return path


def oracle_only():
    """The CPU oracle library alone: built, loaded, and nothing of the GPU
    product library mapped into this process."""
    importlib.import_module("maxim-rs_b200.build").build()
    oracle = importlib.import_module("oracle")
    oracle.lib()
    return oracle


def cpu_baseline(threads):
    """The reference's CPU algorithm (oracle/exec_cpu.cpp, the C++ restatement
    of src/exec_cpu.rs) timed on this box's host cores, through the oracle
    library's own plan builder:
      * value: one whole MAXIM-3S pass over the bench's first 1280x853 image
        (padded 1280x896) with every host thread - measured, not scaled;
      * one_thread: the same algorithm on one thread over a 256x256 image
        (a bounded sample: a full-size image would take about ten minutes on
        one core), as padded pixels per second; FLOPs per padded pixel do not
        depend on the image size for this model (the gating matmuls contract
        fixed 256- or 64-cell axes), so the Mpx/s it implies for a 1280x853
        image is stated beside it."""
    oracle = oracle_only()
    synth = importlib.import_module("maxim-rs_b200.synth")
    path = checkpoint_path(oracle.param_spec(VARIANT))
    img = make_images(1, 0, 1, pre=oracle.preprocess)[0]
    plan = oracle.HostPlan(path, PAD_H, PAD_W)
    t = time.perf_counter()
    oracle.output(plan, img, threads)
    dt = time.perf_counter() - t
    del plan
    small = oracle.HostPlan(path, 256, 256)
    simg = synth.image_uniform(synth.input_rng(IN_SEED), 256, 256)
    t = time.perf_counter()
    oracle.output(small, simg, 1)
    dt1 = time.perf_counter() - t
    px_per_s = 256 * 256 / dt1
    return {"value": OUT_MPX / dt, "unit": "Mpx/s", "cores": threads, "kind": "port",
            "sample": "one whole MAXIM-3S pass over one 1280x853 image (padded 1280x896), %.1f s on %d threads; "
                      "oracle/exec_cpu.cpp, the reference's exec_cpu.rs restated in C++" % (dt, threads),
            "one_thread": {"padded_px_per_s": px_per_s, "seconds": dt1,
                           "sample": "one MAXIM-3S pass over a 256x256 image on 1 thread",
                           "implied_mpx_per_s_1280x853": OUT_MPX * px_per_s / (PAD_H * PAD_W)}}


def run_reference(args):
    """`--impl reference`: the reference's CPU algorithm on this box's host
    cores, on the native arm's workload (same config, metric and unit).

    Each step is B whole 1280x853 images (padded 1280x896) through the oracle
    with every host thread, timed end to end: nothing is scaled. A full image
    takes tens of seconds here, so the arm runs at most --ref-steps steps
    (default 2) and one warm-up pass on a 128x128 image, and reports the steps
    it actually ran. The process maps only the oracle library."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    threads = len(os.sched_getaffinity(0))
    oracle = oracle_only()
    synth = importlib.import_module("maxim-rs_b200.synth")
    path = checkpoint_path(oracle.param_spec(VARIANT))
    B = args.batch
    imgs = make_images(B, 0, 1, pre=oracle.preprocess)
    plan = oracle.HostPlan(path, PAD_H, PAD_W)
    warm = oracle.HostPlan(path, 128, 128)
    oracle.output(warm, synth.image_uniform(synth.input_rng(IN_SEED), 128, 128), threads)
    del warm
    steps = max(1, min(args.steps, args.ref_steps))
    t0 = time.perf_counter()
    for _ in range(steps):
        for b in range(B):
            oracle.output(plan, imgs[b], threads)
    dt = time.perf_counter() - t0
    value = steps * B * OUT_MPX / dt
    line = {"metric": METRIC, "value": value, "unit": "Mpx/s", "n_gpus": args.gpus, "steps": steps,
            "steps_requested": args.steps, "warmup": 1, "warmup_requested": args.warmup,
            "ms_per_step": 1000.0 * dt / steps, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic", "impl": "reference", "config": bench_config(B),
            "cpu_baseline": {"value": value, "unit": "Mpx/s", "cores": threads, "kind": "port",
                             "sample": "%d step(s) of %d whole 1280x853 image(s) (padded 1280x896) each, %.1f s "
                                       "in all, on %d threads; warm-up one 128x128 pass; oracle/exec_cpu.cpp, the "
                                       "reference's exec_cpu.rs restated in C++ (the Rust original cannot be built "
                                       "offline)" % (steps, B, dt, threads)},
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
    hbm, _, tf_sus, _ = peaks()
    print("roofline per family: the slower of HBM (algorithmic bytes at %.0f GB/s) and the tensor pipe (3 TF32 "
          "products per useful MAC at %.0f TFLOP/s, half the sustained bf16 figure)" % (hbm, tf_sus / 2))
    print("%-26s %5s %9s %6s %9s %9s %6s %6s" % ("step family", "steps", "ms", "share", "TFLOP/s", "GB/s", "bound",
                                                 "frac"))
    for k, (n, ms, f, b) in sorted(fam.items(), key=lambda kv: -kv[1][1]):
        ms_ = max(ms, 1e-9)
        r = work.roofline(k, f, b, ms_ / 1e3, hbm, tf_sus / 2)
        print("%-26s %5d %9.2f %5.1f%% %9.1f %9.0f %6s %6.2f" % (k, n, ms, 100 * ms / tot, f / ms_ / 1e9,
                                                                 b / ms_ / 1e6, r["bound"], r["frac"]))
    print("top shapes:")
    for k, (n, ms, f, b) in sorted(shp.items(), key=lambda kv: -kv[1][1])[:24]:
        ms_ = max(ms, 1e-9)
        r = work.roofline(k, f, b, ms_ / 1e3, hbm, tf_sus / 2)
        print("  %8.2f ms %4dx  %-48s %7.1f TFLOP/s %6.0f GB/s  %s %.2f" % (ms, n, k, f / ms_ / 1e9, b / ms_ / 1e6,
                                                                          r["bound"], r["frac"]))
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


def config3_gmlp(mx, local, reps=5, warmup=3):
    """BASELINE config 3, the isolated multi-axis gMLP block op: one residual
    split-head multi-axis gMLP layer (the builder's own split_head_gmlp,
    src/model.rs:576-603, as the "gMLP-64" plan) over an NHWC [1,512,512,64]
    N(0,1) tensor, Dense weights N(0, 0.02), seed 2. `ms`: device time of one
    pass with the tensor in HBM (CUDA events on the executor's stream, median
    of `reps`); `e2e_ms`: the same through mx_gpu_run from pinned host memory.
    The roofline: 39.5 GFLOP of useful products issued as 3 TF32 products
    each, against the TF32 dense rate (half the measured bf16 burst), and the
    134 MB the layer must move (read x, write y) against the measured copy
    bandwidth."""
    import torch
    synth = importlib.import_module("maxim-rs_b200.synth")
    work = importlib.import_module("maxim-rs_b200.work")
    d = os.path.join(tempfile.gettempdir(), "maxim_b200_bench")
    os.makedirs(d, exist_ok=True)
    path = os.path.join(d, "gMLP-64_seed2.safetensors")
    if not os.path.exists(path):
        synth.write_safetensors(path, synth.make_params("gMLP-64", 2, dense_std=0.02), "gMLP-64")
    x = synth.input_rng(2).standard_normal((1, 512, 512, 64)).astype(np.float32)[0].transpose(2, 0, 1).copy()
    plan = mx.Plan(mx.Weights(path), 512, 512)
    g = mx.Gpu(plan, device=local)
    flop = sum(v[1] for v in work.census(plan).values())
    xd = torch.from_numpy(x).cuda(local)
    yd = torch.empty(g.out_shape, dtype=torch.float32, device="cuda:%d" % local)
    stream = torch.cuda.ExternalStream(g.stream(), device=torch.device("cuda", local))

    def one():
        g.upload_input_device(xd.data_ptr())
        g.enqueue()
        g.download_output_device(yd.data_ptr())

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
    pin_in = torch.from_numpy(x).pin_memory()
    pin_out = torch.empty(g.out_shape, dtype=torch.float32).pin_memory()
    host = []
    for _ in range(reps):
        t0 = time.perf_counter()
        g.run(pin_in.numpy(), pin_out.numpy())
        host.append((time.perf_counter() - t0) * 1e3)
    g.close()
    ms = statistics.median(dev)
    hbm, tf_burst, _, _ = peaks()
    tf32 = tf_burst / 2
    issued = 3 * flop
    min_bytes = 2 * x.nbytes
    return {"ms": ms, "e2e_ms": statistics.median(host), "reps": reps,
            "config": "one split-head multi-axis gMLP layer, NHWC [1,512,512,64] N(0,1), Dense N(0,0.02), seed 2",
            "gflop": flop / 1e9, "useful_tflops": flop / ms / 1e9,
            "roofline": {"bound": "tensor", "achieved": issued / ms / 1e9, "peak": tf32, "unit": "TFLOP/s",
                         "frac": issued / ms / 1e9 / tf32, "peak_source": "TF32 dense = half the measured bf16 burst",
                         "min_bytes": min_bytes, "hbm_frac_of_min_traffic": min_bytes / (ms / 1e3) / 1e9 / hbm}}


def startup_times(mx, local):
    """Seconds to bring an executor up for the headline workload: opening the
    checkpoint and building the plan (host), then mx_gpu_new deriving every
    tensor-core layout, mx_gpu_new_cached writing a fresh converted-weights
    cache, and mx_gpu_new_cached reading it back."""
    import tempfile
    t0 = time.perf_counter()
    w = mx.Weights(checkpoint_path())
    plan = mx.Plan(w, PAD_H, PAD_W)
    t_plan = time.perf_counter() - t0
    out = {"weights_and_plan_s": t_plan}
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "weights.mxw")
        for key, kw in (("gpu_new_s", {}), ("gpu_new_cache_write_s", {"weight_cache": path}),
                        ("gpu_new_cache_read_s", {"weight_cache": path})):
            t0 = time.perf_counter()
            g = mx.Gpu(plan, device=local, **kw)
            out[key] = time.perf_counter() - t0
            out[key.replace("_s", "_phases")] = g.build_info()
            g.close()
        out["cache_file_bytes"] = os.path.getsize(path)
    return out


def e2e_rgb8(mx, gpu, steps):
    """The single-image public path with its per-pixel steps on the device
    (mx_gpu_run_rgb8): 8-bit 1280x853 RGB from host memory in, the restored
    8-bit image out, one synchronous call per image."""
    synth = importlib.import_module("maxim-rs_b200.synth")
    rng = synth.input_rng(IN_SEED)
    imgs = [np.ascontiguousarray((np.floor(synth.image_uniform(rng, IMG_H, IMG_W) * np.float32(255) +
                                           np.float32(0.5))).astype(np.uint8).transpose(1, 2, 0))
            for _ in range(2)]
    out = np.empty_like(imgs[0])
    for i in range(3):
        gpu.run_rgb8(imgs[i % 2], out=out)
    t0 = time.perf_counter()
    for i in range(steps):
        gpu.run_rgb8(imgs[i % 2], out=out)
    dt = time.perf_counter() - t0
    nbytes = IMG_H * IMG_W * 3
    return {"value": steps * IMG_H * IMG_W / dt / 1e6, "unit": "Mpx/s", "images": steps, "seconds": dt,
            "h2d_bytes_per_step": nbytes, "d2h_bytes_per_step": nbytes,
            "api": "mx_gpu_run_rgb8 (one image per call, no overlap)"}


def e2e_png(mx, plan, local, steps):
    """PNG files in, PNG files out through the batch runner's PNG path
    (mx_batch_run_png) on this GPU: decode, device-side pad / crop / round,
    encode and file I/O all inside the timed region."""
    import tempfile
    synth = importlib.import_module("maxim-rs_b200.synth")
    rng = synth.input_rng(IN_SEED)
    with tempfile.TemporaryDirectory() as d:
        ins = []
        for k in range(2):
            im = (np.floor(synth.image_uniform(rng, IMG_H, IMG_W) * np.float32(255) + np.float32(0.5))).astype(
                np.uint8).transpose(1, 2, 0)
            ins.append(os.path.join(d, "in%d.png" % k))
            mx.png_write_rgb8(ins[-1], im)
        runner = mx.Batch(plan, devices=(local,))
        outs = [os.path.join(d, "out%d.png" % i) for i in range(steps)]
        runner.run_png(ins, outs[:2])
        t0 = time.perf_counter()
        runner.run_png([ins[i % 2] for i in range(steps)], outs)
        dt = time.perf_counter() - t0
        in_bytes = sum(os.path.getsize(p) for p in ins) / 2
        runner.close()
    nbytes = IMG_H * IMG_W * 3
    return {"value": steps * IMG_H * IMG_W / dt / 1e6, "unit": "Mpx/s", "images": steps, "seconds": dt,
            "h2d_bytes_per_step": nbytes, "d2h_bytes_per_step": nbytes, "png_bytes_per_image": in_bytes,
            "api": "mx_batch_run_png (decode and encode overlapping the passes)"}


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

    # e2e: the public batch API (mx_batch_run) from the caller's host arrays:
    # per image the runner copies it into pinned staging, uploads it, runs
    # the pass and copies the result back, all inside the timed region.
    # The K steps' images go in as one batch call, which keeps two images in
    # flight (a caller restoring a batch makes one call).
    runner = mx.Batch(plan, devices=(local,))
    outs = [np.empty(gpu.out_shape, np.float32) for _ in range(B)]
    runner.run(imgs, outs)
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    runner.run([imgs[b] for _ in range(args.steps) for b in range(B)], [outs[b] for _ in range(args.steps)
                                                                          for b in range(B)])
    e2e_s = time.perf_counter() - t0
    runner.close()
    barrier()
    e2e_s = max_over_ranks(e2e_s, world, "cuda:%d" % local)
    e2e = job_mpx_per_s(args.steps * B, world, e2e_s)

    # Roofline of the dominant step family, from per-step CUDA events on the
    # executor's stream over one pass of the same workload (a kernel timed
    # inside a long pass: the sustained peaks).
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
    roof = work.roofline(dom, fl / n_l, by / n_l, ms_tot / 1000.0 / n_l, hbm, tf_sus / 2)
    roof["traffic"] = traffic_from_profiles(dom)
    roof["kernel"] = dom
    roof["launches_per_pass"] = n_l
    roof["share_of_pass"] = ms_tot / total
    roof["peak_source"] = src + (" copy" if roof["bound"] == "hbm" else
                                 " TF32 dense = half the sustained bf16 figure (3 TF32 products per useful MAC)")
    roof["algorithmic_per_launch"] = {"flop": fl / n_l, "bytes": by / n_l}

    line = {"metric": METRIC, "value": value, "value_per_gpu": value / world, "unit": "Mpx/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": bench_config(B),
            "e2e": {"value": e2e, "unit": "Mpx/s", "h2d_bytes_per_step": int(B * in_dev[0].numel() * 4),
                    "d2h_bytes_per_step": int(B * out_dev[0].numel() * 4)},
            "gpu_launches": int(stats["kernels"] * args.steps * B),
            "roofline": roof, "clocks": clk.summary()}
    if rank == 0 and world == 1:
        line["e2e_rgb8"] = e2e_rgb8(mx, gpu, args.steps)
        line["e2e_png"] = e2e_png(mx, plan, local, args.steps)
        with Clocks(uuid) as clk4:
            line["latency_2048"] = latency_2048(mx, local)
        line["latency_2048"]["clocks"] = clk4.summary()
        with Clocks(uuid) as clk5:
            line["config5_s2"] = config5_s2(mx, local)
        line["config5_s2"]["clocks"] = clk5.summary()
        with Clocks(uuid) as clk3:
            line["config3_gmlp"] = config3_gmlp(mx, local)
        line["config3_gmlp"]["clocks"] = clk3.summary()
    gpu.close()
    if rank == 0 and world == 1:
        line["startup"] = startup_times(mx, local)
    if rank == 0 and world == 1 and not args.no_cpu:
        line["cpu_baseline"] = cpu_baseline(len(os.sched_getaffinity(0)))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--batch", type=int, default=1, help="images per GPU per step")
    ap.add_argument("--impl", choices=["native", "reference"], default="native")
    ap.add_argument("--ref-steps", type=int, default=2,
                    help="--impl reference: most steps to run (each is B whole images on the CPU)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline")
    ap.add_argument("--timeline", action="store_true",
                    help="print the per-op-family device time of one pass and exit (no JSON line)")
    ap.add_argument("--variant", default=VARIANT, help="--timeline only: model variant")
    ap.add_argument("--height", type=int, default=IMG_H, help="--timeline only: image height")
    ap.add_argument("--width", type=int, default=IMG_W, help="--timeline only: image width")
    args = ap.parse_args()
    if args.timeline:
        return run_timeline(args)  # a census, not a timed number: any warm-up count
    if args.warmup < 3:
        log("bench: raising --warmup to 3")
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    return run_native(args)


if __name__ == "__main__":
    sys.exit(main())
