"""The plan builder and arena packer (a C++ restatement of src/model.rs) against
the figures the reference publishes and the invariants its tests pin
(tests/arena.rs, tests/packing.rs). These need shapes only, so they build the
plan for a named variant without a checkpoint."""
import math

import numpy as np
import pytest

MIB = 1048576.0


@pytest.mark.parametrize("variant,ops,bufs,tensors,params", [
    ("S-2", 1840, 2089, 1760, 14176178),   # docs/DEVELOPING.md:102, src/host.rs:10, README.md:56-66
    ("S-3", 2885, 3276, 2754, 22212795),   # docs/DEVELOPING.md:103
])
def test_graph_size_matches_the_reference(mx, variant, ops, bufs, tensors, params):
    plan = mx.Plan(variant=variant, h=64, w=64)
    assert plan.n_ops == ops
    assert plan.n_bufs == bufs
    spec = mx.param_spec(variant)
    assert len(spec) == tensors
    assert sum(math.prod(s) for _, s in spec) == params


@pytest.mark.parametrize("variant,h,w,mib", [
    ("S-2", 256, 256, 115.0),     # docs/DEVELOPING.md:102
    ("S-2", 448, 640, 503.1),     # docs/DEVELOPING.md:104
    ("S-2", 1408, 2048, 5059.3),  # docs/DEVELOPING.md:141-144 (2048x1362 padded)
    ("S-3", 2048, 2048, 7359.0),  # docs/DEVELOPING.md:141-144
    ("S-3", 896, 1280, 2012.2),   # the bench shape (1280x853 padded)
])
def test_arena_matches_the_reference_packer(mx, variant, h, w, mib):
    plan = mx.Plan(variant=variant, h=h, w=w)
    assert round(plan.arena_bytes / MIB, 1) == mib


def operands(op):
    # `Op::operands` (src/model.rs:117-139): dst first.
    if op.kind in (1, 2, 3, 9):
        return [op.dst, op.src, op.src2]
    if op.kind == 16:
        return [op.dst, op.src, op.tmp]
    return [op.dst, op.src]


def live_set_peak(plan):
    """tests/arena.rs:38-82: the peak of the live set in bytes."""
    n = plan.n_bufs
    owner = list(range(n))
    for i in range(n):
        a, j = plan.alias(i), i
        while a is not None:
            j = a[0]
            a = plan.alias(j)
        owner[i] = j
    first, last = {}, {}
    for oi, op in enumerate(plan.ops()):
        for b in operands(op):
            o = owner[b]
            first.setdefault(o, oi)
            last[o] = oi
    size = {b: 4 * np.prod(plan.buf(b)) for b in first}
    events = np.zeros(plan.n_ops + 1)
    for b in first:
        events[first[b]] += size[b]
        events[last[b] + 1] -= size[b]
    return float(np.cumsum(events).max())


@pytest.mark.parametrize("h,w", [(480, 640), (832, 1280)])
def test_the_arena_is_close_to_the_live_set(mx, h, w):
    """tests/arena.rs:84-106: packed arena <= 1.20x the live-set peak."""
    plan = mx.Plan(variant="S-2", h=h, w=w)
    assert plan.arena_bytes / live_set_peak(plan) <= 1.20


def test_naming_activations_is_what_costs_the_memory(mx):
    """tests/arena.rs:108-126."""
    named = mx.Plan(variant="S-2", h=480, w=640, dumps=True)
    lean = mx.Plan(variant="S-2", h=480, w=640, dumps=False)
    assert len(named.dumps()) > 0
    assert named.arena_bytes / lean.arena_bytes > 1.5


def test_no_op_overlaps_its_own_inputs(mx):
    """tests/packing.rs:92-118."""
    plan = mx.Plan(variant="S-2", h=64, w=64)
    for i, op in enumerate(plan.ops()):
        ids = operands(op)
        d, dn = plan.off(ids[0]), np.prod(plan.buf(ids[0]))
        for s in ids[1:]:
            so, sn = plan.off(s), np.prod(plan.buf(s))
            assert not (d < so + sn and so < d + dn), "op %d aliases its input %d" % (i, s)


def test_the_plan_is_the_size_it_claims(mx):
    """tests/packing.rs:70-85: every named buffer lies inside the arena."""
    plan = mx.Plan(variant="S-2", h=64, w=64, dumps=True)
    for name, bid in plan.dumps():
        assert plan.off(bid) + np.prod(plan.buf(bid)) <= plan.arena_len, name


def test_every_buffer_lies_inside_the_arena(mx):
    plan = mx.Plan(variant="S-3", h=128, w=192)
    for b in range(plan.n_bufs):
        assert plan.off(b) + np.prod(plan.buf(b)) <= plan.arena_len, plan.label(b)


def test_too_small_for_the_gmlp_is_refused_by_name(mx):
    """src/model.rs:529-535: a sub-block feature map is refused, not run."""
    with pytest.raises(mx.MaximError, match="too small for this model"):
        mx.Plan(variant="S-2", h=32, w=32)


def test_unknown_variant_is_refused(mx):
    with pytest.raises(mx.MaximError, match="unknown variant"):
        mx.Plan(variant="S-9", h=64, w=64)


def test_checkpoint_derives_its_variant(mx, checkpoint):
    """src/config.rs:71-100: the variant is a property of the file."""
    for v in ("S-1", "S-2", "M-1"):
        assert mx.Weights(checkpoint(v, 11)).variant == v


def test_a_missing_tensor_fails_at_build_time(mx, synth, tmp_path):
    params = synth.make_params("S-1", 3)
    params.pop("stage_0_encoder_block_1/Conv_1/kernel")
    path = str(tmp_path / "broken.safetensors")
    synth.write_safetensors(path, params, "S-1")
    w = mx.Weights(path)
    with pytest.raises(mx.MaximError, match="Conv_1/kernel"):
        mx.Plan(w, 64, 64)


def test_a_misshapen_tensor_fails_at_build_time(mx, synth, tmp_path):
    params = synth.make_params("S-1", 3)
    params["stage_0_encoder_block_0/Conv_0/bias"] = np.zeros(7, np.float32)
    path = str(tmp_path / "broken.safetensors")
    synth.write_safetensors(path, params, "S-1")
    with pytest.raises(mx.MaximError, match="expected shape"):
        mx.Plan(mx.Weights(path), 64, 64)
