"""The executor's schedule of a plan, worked out on the host (no device):
which ops fuse into which, which block permutations go, and the re-packed
arena. The GPU tests check the fused pass computes the same values; these
check the schedule's shape and its liveness-safe packing rules on CPU."""
import os

import numpy as np
import pytest

BLOCK_PERM, GATE_MM, CONV1X1, CONV3X3, GELU, ADD, COPY, GATE_APPLY, LN = 15, 14, 10, 11, 4, 1, 0, 3, 7


def _sched(mx, plan, fuse=True):
    if fuse:
        return mx.plan_schedule(plan)
    os.environ["MAXIM_NO_FUSE"] = "1"
    try:
        return mx.plan_schedule(plan)
    finally:
        del os.environ["MAXIM_NO_FUSE"]


@pytest.mark.parametrize("variant,h,w", [("S-2", 64, 64), ("S-3", 256, 320), ("S-3", 896, 1280)])
def test_schedule_shape(variant, h, w, mx):
    plan = mx.Plan(None, h, w, variant=variant)
    ops = plan.ops()
    st, primary = _sched(mx, plan)
    kinds = np.array([o.kind for o in ops])
    forward = np.array([o.kind == BLOCK_PERM and bool(o.forward) for o in ops], dtype=bool)
    # Every forward block permutation goes (the gating reads the blocks in
    # place); otherwise only Copies are removed outright (their readers read
    # the source).
    assert st["perms_dropped"] == forward.sum()
    assert (primary[forward] < 0).all()
    assert (kinds[(primary < 0) & ~forward] == COPY).all()
    # An absorbed op runs in the step of an earlier op.
    idx = np.arange(len(ops))
    assert (primary[primary >= 0] <= idx[primary >= 0]).all()
    assert st["steps"] == (primary == idx).sum()
    assert st["ops_fused"] == ((primary >= 0) & (primary != idx)).sum()
    # Every GELU after a tensor-core 1x1 conv is that conv's epilogue, and
    # every backward permutation (now a Copy) is forwarded into its producer.
    for i in np.nonzero(kinds == GELU)[0]:
        assert kinds[primary[i]] == CONV1X1
    for i in np.nonzero((kinds == BLOCK_PERM) & ~forward)[0]:
        assert primary[i] != i
    # The re-packed arena is no larger than the plan's.
    assert st["pass_arena_bytes"] <= st["arena_bytes"]
    # Every LayerNorm read by a 1x1 conv alone is normalised on load, paired
    # with exactly one conv: its statistics come from a statistics step or,
    # where a tensor-core conv produced its input, from that conv's epilogue.
    _, _, flags = mx.plan_schedule(plan, flags=True)
    stats_only = (flags & mx._native.SCHED_STATS_ONLY) > 0
    on_load = (flags & mx._native.SCHED_LN_ON_LOAD) > 0
    ln_out = (flags & mx._native.SCHED_LN_IN_EPILOGUE) > 0
    ln = kinds == LN
    in_epilogue = ln & (primary >= 0) & (primary != idx) & ~ln_out
    assert on_load.sum() > 0 and stats_only.sum() + in_epilogue.sum() == on_load.sum()
    assert (kinds[stats_only] == LN).all() and (kinds[on_load] == CONV1X1).all()
    assert np.isin(kinds[primary[in_epilogue]], [CONV1X1, CONV3X3, 12]).all()
    assert in_epilogue.sum() > stats_only.sum()
    # A LayerNorm over one 32-channel chunk of a tensor-core 1x1 conv's output
    # is written whole by that conv's epilogue (the gMLP gates' v halves).
    assert ln_out.sum() > 0 and (ln_out <= ln).all()
    assert (kinds[primary[ln_out]] == CONV1X1).all() and all(ops[i].c == 32 for i in np.nonzero(ln_out)[0])


def test_schedule_off_keeps_every_op(mx):
    plan = mx.Plan(None, 128, 192, variant="S-2")
    st, primary = _sched(mx, plan, fuse=False)
    assert st["ops_fused"] == 0 and st["perms_dropped"] == 0
    assert (primary == np.arange(plan.n_ops)).all()
    assert st["steps"] == plan.n_ops


def test_schedule_without_tensor_cores_fuses_only_copies(mx):
    """With the tensor-core kernel off only the small-conv kernel (1x1 convs
    over fewer than 128 pixels: the channel attention's on the squeezed 1x1
    plane, and at 64x64 the bottleneck's) takes an epilogue, a unary tail;
    otherwise only Copies are forwarded and the
    channel-attention residual add joins its channel scale; block
    permutations stay (the SIMT gating reads blocks)."""
    plan = mx.Plan(None, 64, 64, variant="S-2")
    os.environ["MAXIM_NO_UMMA"] = "1"
    try:
        st, primary = mx.plan_schedule(plan)
    finally:
        del os.environ["MAXIM_NO_UMMA"]
    kinds = np.array([o.kind for o in plan.ops()])
    assert st["perms_dropped"] == 0
    moved = (primary >= 0) & (primary != np.arange(plan.n_ops))
    assert moved.any() and np.isin(kinds[moved], [COPY, ADD, GELU, 5, 6]).all()
    assert (kinds[primary[moved & (kinds == ADD)]] == 9).all()  # an add only ever joins a channel scale
    ops = plan.ops()
    for i in np.nonzero(moved & np.isin(kinds, [GELU, 5, 6]))[0]:  # GELU / LeakyReLU / sigmoid: a small conv's tail
        p = ops[primary[i]]
        assert p.kind == CONV1X1 and p.h * p.wd < 128


def test_step_work_counts_what_a_fused_step_must_move(mx):
    """The roofline numerators: a fused step moves its members' bytes less
    the intermediates fusion removes. A GELU tail removes its input both
    ways (the conv no longer writes it, the GELU no longer reads it); a
    LayerNorm written whole by the epilogue normalises a tensor that other
    ops still read, so only its read goes and its own output is counted;
    where nothing else reads that tensor, it goes both ways like the GELU's."""
    import importlib
    work = importlib.import_module("maxim-rs_b200.work")
    plan = mx.Plan(None, 256, 320, variant="S-3")
    ops = plan.ops()
    _, prim, flags = mx.plan_schedule(plan, flags=True)
    seen_gelu = seen_ln = False
    for p, members in work.schedule_steps(prim).items():
        fam, f, b = work.step_work(plan, ops, members, flags)
        if flags[p] & mx._native.SCHED_STATS_ONLY:  # a LayerNorm reduced to its statistics
            o = ops[p]
            assert fam == "ln_stats" and b == 4 * o.c * o.hw + 8 * o.hw
            continue
        own = sum(work.op_work(plan, ops[j])[1] for j in members)
        removed = 0
        for j in members[1:]:
            c, h, w = plan.buf(ops[j].dst)
            if flags[j] & mx._native.SCHED_LN_IN_EPILOGUE and not flags[j] & mx._native.SCHED_LN_INPUT_UNSTORED:
                removed += 4 * c * h * w
                seen_ln = True
            else:
                removed += 8 * c * h * w
                seen_gelu |= ops[j].kind == GELU
        assert b == own - removed
    assert seen_gelu and seen_ln


def _steps_and_writers(mx, plan):
    import importlib
    work = importlib.import_module("maxim-rs_b200.work")
    ops = plan.ops()
    _, prim = mx.plan_schedule(plan)
    writers = {}
    for i, o in enumerate(ops):
        writers.setdefault(o.dst, []).append(i)
    return ops, work.schedule_steps(prim), writers


def test_schedule_moves_a_producer_to_its_consumer(mx):
    """A tensor-core conv whose only reader is a multiply by a tensor made
    after the conv (the gMLP block's gelu(conv_a(x)) * conv_b(x), conv_b
    first in the plan) runs at the multiply's position with the multiply as
    its epilogue; nothing between the two rewrites the conv's input."""
    plan = mx.Plan(None, 256, 320, variant="S-3")
    ops, steps, writers = _steps_and_writers(mx, plan)
    moved = 0
    for p, members in steps.items():
        if ops[p].kind not in (CONV1X1, CONV3X3):
            continue
        for m in members[1:]:
            if ops[m].kind != 2:  # MUL
                continue
            other = ops[m].src2 if ops[m].src == ops[p].dst else ops[m].src
            if any(p < w < m for w in writers.get(other, [])):
                moved += 1
                assert not any(p < w < m for w in writers.get(ops[p].src, []))
    assert moved >= 21


def test_schedule_channel_scale_takes_two_residual_adds(mx):
    """x * s + r followed by + r2 is one channel-scale step over both adds."""
    plan = mx.Plan(None, 256, 320, variant="S-3")
    ops, steps, _ = _steps_and_writers(mx, plan)
    two = [p for p, members in steps.items()
           if ops[p].kind == 9 and sum(ops[m].kind == ADD for m in members) == 2]
    assert len(two) >= 24


def test_schedule_places_a_copied_concatenation_inside_its_copy(mx):
    """A Copy of a whole root (a concatenation) into a view of a wider root
    goes: the root is placed where the Copy would have written it, so the
    steps that write its slices write the wider root's (MAXIM-3S: the three
    UpSampleRatio stacks per stage, nine Copies)."""
    plan = mx.Plan(None, 256, 320, variant="S-3")
    ops = plan.ops()
    _, prim = mx.plan_schedule(plan)

    def root(b):
        while plan.alias(b) is not None:
            b = plan.alias(b)[0]
        return b
    readers = {}
    for o in ops:
        for s in (o.src, o.src2):
            if s >= 0:
                readers[root(s)] = readers.get(root(s), 0) + 1
    merged = 0
    for i, o in enumerate(ops):
        if o.kind != COPY or plan.alias(o.src) is not None or plan.alias(o.dst) is None or readers[o.src] != 1:
            continue
        parent = plan.alias(o.dst)[0]
        if plan.buf(parent)[0] > plan.buf(o.dst)[0] and plan.buf(o.src) == plan.buf(o.dst):
            # Forwarded into the source's producer, or placed away: never a
            # step of its own.
            assert prim[i] != i
            merged += prim[i] < 0
    assert merged == 9
