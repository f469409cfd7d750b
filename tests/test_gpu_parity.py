"""GPU parity: the executor behind the C ABI against the CPU oracle (the
restatement of the reference's exec_cpu.rs) and against the reference's own
golden outputs, on the same seeded weights and inputs.

Bars (the north star's, plus the reference's own per-op bar):
  * per op, in lockstep: max|gpu - cpu| <= 1e-3 * max|cpu| for every op's
    destination (src/main.rs:709-713, `--verify-gpu`);
  * end to end: float PSNR >= 50 dB against the CPU path, with peak 1.0 (as
    stated) and with peak = max|cpu| (scale-aware: the He-normal init diverges
    to |y| ~ 1e7, where a peak of 1 is meaningless);
  * >= 99.9% of 8-bit output pixels within 1 LSB after the reference's clamp
    and round-half-up.
Numerics: contractions run on tensor cores with TF32 operands in a 3-pass
split (a*b + a*b_lo + a_lo*b, FP32 accumulate), or FP32 FMA on the SIMT
fallback; LayerNorm statistics and resize taps follow the reference's order
exactly.
"""
import numpy as np
import pytest

from conftest import GOLDEN_CASES, golden, lsb_fraction, psnr, rel_rms

pytestmark = pytest.mark.gpu


def golden_setup(mx, checkpoint, case):
    z = golden(case)
    variant, seed, gain, rich = str(z["meta_variant"]), int(z["meta_seed"]), float(z["meta_gain"]), bool(
        z["meta_rich"])
    w = mx.Weights(checkpoint(variant, seed, gain, rich))
    img = z["input"]
    return z, w, img


@pytest.mark.parametrize("case", GOLDEN_CASES)
def test_gpu_matches_oracle_and_reference(case, mx, oracle, checkpoint):
    z, w, img = golden_setup(mx, checkpoint, case)
    plan = mx.Plan(w, img.shape[1], img.shape[2])
    cpu = oracle.output(plan, img)
    gpu = mx.Gpu(plan)
    out = gpu.run(img)
    again = gpu.run(img)
    assert np.array_equal(out, again), "two runs of the same graph differ"
    assert np.isfinite(out).all()
    assert psnr(cpu, out) >= 50.0
    assert psnr(z["final"], out) >= 50.0
    if np.abs(cpu).max() < 10:
        assert psnr(cpu, out, peak=1.0) >= 50.0
    assert lsb_fraction(cpu, out) >= 0.999
    assert rel_rms(cpu, out) <= 1e-3


def test_gpu_per_op_lockstep(mx, oracle, checkpoint):
    """`--verify-gpu` (src/main.rs:671-730): both executors walk the plan one
    op at a time from the same input; each op's destination must agree to
    1e-3 of its own magnitude. This localises any kernel or layout bug to the
    op that produced it."""
    z, w, img = golden_setup(mx, checkpoint, "s2_64_rich")
    plan = mx.Plan(w, 64, 64)
    gpu = mx.Gpu(plan)
    gpu.begin(img)
    arena = oracle.new_arena(plan, img)
    bad = []
    for i, op in enumerate(plan.ops()):
        oracle.run_range(plan, arena, i, i + 1, threads=4)
        gpu.step_op(i)
        cpu = oracle.take(plan, arena, op.dst)
        got = gpu.read_buf(op.dst)
        scale = max(float(np.abs(cpu).max()), 1e-6)
        err = float(np.abs(got.astype(np.float64) - cpu).max())
        if not err <= 1e-3 * scale:
            bad.append((i, op.kind, err / scale))
    assert not bad, bad[:10]


def test_gpu_per_op_lockstep_multi_tile(mx, synth, oracle, checkpoint):
    """The same walk at 256x320: every tensor-core conv now has more output
    tiles than the GPU has SMs, so each persistent CTA cycles its pipeline
    stages and both TMEM accumulators several times."""
    w = mx.Weights(checkpoint("S-1", 7, 0.5, True))
    img = synth.image_uniform(synth.input_rng(7), 256, 320)
    plan = mx.Plan(w, 256, 320)
    gpu = mx.Gpu(plan)
    gpu.begin(img)
    arena = oracle.new_arena(plan, img)
    bad = []
    for i, op in enumerate(plan.ops()):
        oracle.run_range(plan, arena, i, i + 1)
        gpu.step_op(i)
        cpu = oracle.take(plan, arena, op.dst)
        got = gpu.read_buf(op.dst)
        scale = max(float(np.abs(cpu).max()), 1e-6)
        err = float(np.abs(got.astype(np.float64) - cpu).max())
        if not err <= 1e-3 * scale:
            bad.append((i, op.kind, err / scale))
    assert not bad, bad[:10]
    out = gpu.run(img)
    assert psnr(oracle.output(plan, img), out) >= 50.0


def test_gpu_read_arena_and_stats(mx, checkpoint):
    z, w, img = golden_setup(mx, checkpoint, "m1_64")
    plan = mx.Plan(w, 64, 64)
    gpu = mx.Gpu(plan)
    out = gpu.run(img)
    s = gpu.stats()
    assert s["arena_bytes"] == plan.arena_bytes
    assert s["ops"] == plan.n_ops
    assert s["kernels"] > 0
    assert "B200" in s["device_name"] or s["device_name"]
    a = gpu.read_arena()
    assert a.size == plan.arena_len
    o = plan.off(plan.output)
    assert np.array_equal(a[o:o + out.size].reshape(out.shape), out)


def test_gpu_read_into_and_read_arena_match_the_plan_layout(mx, oracle, checkpoint):
    """`run_gpu`'s two read paths (src/main.rs:494-501): `read_into` at
    plan.offs[output] and, for `--dump`, `read_arena` followed by slicing every
    named activation out of it at its plan offset in [c][h][w] order. A plan
    built with dumps keeps those activations live to the end, so each must
    match the CPU path's arena at the same offset; the output must be exactly
    what mx_gpu_run returned, through either read."""
    z, w, img = golden_setup(mx, checkpoint, "s2_64_rich")
    plan = mx.Plan(w, 64, 64, dumps=True)
    gpu = mx.Gpu(plan)
    out = gpu.run(img)
    o, n = plan.off(plan.output), out.size
    assert np.array_equal(gpu.read_into(o, n).reshape(out.shape), out)
    assert np.array_equal(gpu.read_buf(plan.output), out)
    arena = gpu.read_arena()
    assert arena.size == plan.arena_len
    assert np.array_equal(arena[o:o + n].reshape(out.shape), out)
    cpu = oracle.run(plan, img)
    dumps = plan.dumps()
    assert len(dumps) > 10
    for name, bid in dumps:
        c, h, ww = plan.buf(bid)
        off, k = plan.off(bid), c * h * ww
        ref, got = cpu[off:off + k], arena[off:off + k]
        if np.abs(ref).max() > 0:
            assert psnr(ref, got) >= 50.0, name
        else:
            assert np.abs(got).max() == 0, name
    name, bid = dumps[len(dumps) // 2]
    off, k = plan.off(bid), int(np.prod(plan.buf(bid)))
    assert np.array_equal(gpu.read_into(off, k), arena[off:off + k]), name
    assert np.array_equal(gpu.read_buf(bid).reshape(-1), arena[off:off + k]), name
    # The op-by-op walk leaves the same arena.
    gpu.begin(img)
    for i in range(plan.n_ops):
        gpu.step_op(i)
    assert np.array_equal(gpu.read_arena(), arena)
    # And a pass after the walk reads its output without a replay.
    again = gpu.run(img)
    assert np.array_equal(again, out)
    assert np.array_equal(gpu.read_into(o, n).reshape(out.shape), out)


def test_timeline_covers_every_op(mx, checkpoint):
    z, w, img = golden_setup(mx, checkpoint, "s2_64_he")
    plan = mx.Plan(w, 64, 64)
    gpu = mx.Gpu(plan)
    ref = gpu.run(img)
    gpu.set_timeline(True)
    out = gpu.run(img)
    per, total = gpu.timeline()
    kern = gpu.timeline_kernels()
    assert np.array_equal(ref, out)
    assert per.shape == (plan.n_ops,) and total > 0 and (per >= 0).all()
    # `kernels_per_op` (src/exec_gpu.rs:68-72): every launch of the pass but
    # the two boundary transposes belongs to a plan op.
    assert kern.shape == (plan.n_ops,) and (kern >= 0).all()
    assert int(kern.sum()) == gpu.stats()["kernels"] - 2


def test_oversized_pass_is_refused_before_allocating(mx, checkpoint):
    """`Gpu::new` sizes the pass and refuses it with the numbers
    (src/exec_gpu.rs:96-146): 16384 x 16384 needs far more than 180 GB."""
    plan = mx.Plan(mx.Weights(checkpoint("S-1", 11)), 16384, 16384)
    with pytest.raises(mx.MaximError, match="not enough device memory"):
        mx.Gpu(plan)


def test_plan_without_weights_is_refused(mx):
    plan = mx.Plan(variant="S-1", h=64, w=64)
    with pytest.raises(mx.MaximError, match="without a checkpoint"):
        mx.Gpu(plan)


@pytest.mark.parametrize("gain", [1.0, 0.5])
def test_config2_s3_600x400_parity(mx, synth, oracle, checkpoint, gain):
    """MAXIM-3S, seed 1, a 600x400 smooth-plus-noise image
    padded to 640x448, against the CPU path, at the He-normal init and at the
    companion x0.5 init (outputs O(1), where the 8-bit bar is meaningful)."""
    w = mx.Weights(checkpoint("S-3", 1, gain))
    img = synth.image_smooth_noisy(synth.input_rng(1), 400, 600)
    padded, _ = mx.preprocess(img, 64)
    assert padded.shape == (3, 448, 640)
    plan = mx.Plan(w, 448, 640)
    cpu = oracle.output(plan, padded)
    out = mx.Gpu(plan).run(padded)
    assert psnr(cpu, out) >= 50.0
    if gain == 0.5:
        assert psnr(cpu, out, peak=1.0) >= 50.0
    assert lsb_fraction(cpu, out) >= 0.999


# Ops whose device kernels follow the CPU path's operation order exactly
# (no fused multiply-add, the same summation order), so that from the same
# input they must give the same bits: copies, elementwise add / multiply /
# gate / leaky ReLU, the channel LayerNorm, channel scale, block
# permutation, resize and nearest downsampling.
EXACT_KINDS = {0: "copy", 1: "add", 2: "mul", 3: "gate_apply", 5: "lrelu", 7: "chan_ln", 9: "chan_scale",
               15: "block_perm", 16: "resize", 17: "down_s"}


def test_gpu_memory_bound_ops_are_bit_exact(mx, synth, oracle, checkpoint):
    """For every op of those kinds in an S-1 walk at 256x320, hand the CPU
    oracle the device's own inputs (read back from the GPU arena) and require
    the device's output bit for bit."""
    w = mx.Weights(checkpoint("S-1", 5, 0.5, True))
    img = synth.image_uniform(synth.input_rng(5), 256, 320)
    plan = mx.Plan(w, 256, 320)
    gpu = mx.Gpu(plan)
    gpu.begin(img)
    arena = oracle.new_arena(plan, img)
    seen, bad = {}, []
    for i, op in enumerate(plan.ops()):
        if op.kind in EXACT_KINDS:
            for b in (op.src, op.src2):
                if b >= 0:
                    c, h, ww = plan.buf(b)
                    o = plan.off(b)
                    arena[o:o + c * h * ww] = gpu.read_buf(b).reshape(-1)
            oracle.run_range(plan, arena, i, i + 1, threads=4)
            gpu.step_op(i)
            cpu, got = oracle.take(plan, arena, op.dst), gpu.read_buf(op.dst)
            seen[EXACT_KINDS[op.kind]] = seen.get(EXACT_KINDS[op.kind], 0) + 1
            if not np.array_equal(cpu.view(np.uint32), got.view(np.uint32)):
                bad.append((i, EXACT_KINDS[op.kind], int((cpu.view(np.uint32) != got.view(np.uint32)).sum())))
        else:
            gpu.step_op(i)
    assert {"resize", "chan_ln", "add", "copy", "block_perm"} <= set(seen), seen
    assert not bad, bad[:10]
