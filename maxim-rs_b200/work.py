"""Algorithmic work per op: FLOPs (2 per multiply-add) and fp32 bytes moved if
each op reads its inputs and writes its output exactly once (weights once).

These are the numerators of every roofline figure this project reports; they
depend only on the plan, never on how a kernel happens to move its data.
"""
import collections

KINDS = ["copy", "add", "mul", "gate_apply", "gelu", "lrelu", "sigmoid", "chan_ln", "chan_mean", "chan_scale",
         "conv1x1", "conv3x3", "conv4x4s2", "convt2x2", "gate_mm", "block_perm", "resize", "down_s"]


def op_work(plan, op):
    """(flops, bytes) of one op."""
    k = KINDS[op.kind]
    def n(b):
        c, h, w = plan.buf(b)
        return c * h * w
    if k in ("copy", "gelu", "lrelu", "sigmoid"):
        return (op.n if k != "copy" else 0), 8 * op.n
    if k in ("add", "mul", "gate_apply"):
        return op.n, 12 * op.n
    if k == "chan_ln":
        e = op.c * op.hw
        return 8 * e, 8 * e + 8 * op.c
    if k == "chan_mean":
        return op.c * op.hw, 4 * (op.c * op.hw + op.c)
    if k == "chan_scale":
        return op.c * op.hw, 8 * op.c * op.hw + 4 * op.c
    if k == "conv1x1":
        m = op.h * op.wd
        return 2 * m * op.c_in * op.c_out, 4 * (m * (op.c_in + op.c_out) + op.c_in * op.c_out + op.c_out)
    if k == "conv3x3":
        m = op.h * op.wd
        return 18 * m * op.c_in * op.c_out, 4 * (m * (op.c_in + op.c_out) + 9 * op.c_in * op.c_out + op.c_out)
    if k == "conv4x4s2":
        m = op.oh * op.ow
        return 32 * m * op.c_in * op.c_out, 4 * (op.h * op.wd * op.c_in + m * op.c_out + 16 * op.c_in * op.c_out)
    if k == "convt2x2":
        m = op.h * op.wd
        return 8 * m * op.c_in * op.c_out, 4 * (m * op.c_in + 4 * m * op.c_out + 4 * op.c_in * op.c_out)
    if k == "gate_mm":
        nn = op.outer if op.mode == 0 else op.inner
        e = op.c * op.outer * op.inner
        return 2 * e * nn, 4 * (2 * e + nn * nn + nn)
    if k == "block_perm":
        return 0, 8 * n(op.dst)
    if k == "resize":
        return 0, 4 * (op.c * op.hin * op.win + op.c * op.hout * op.wout)
    if k == "down_s":
        return 0, 8 * op.c * op.oh * op.ow
    return 0, 0


# Ops a tensor-core step can apply in its epilogue (the step's family names them).
TAILS = ("gelu", "lrelu", "sigmoid", "add", "mul", "gate_apply")


def schedule_steps(primary):
    """{primary op: [ops it carries out, primary first]} from the executor's
    schedule (`Gpu.schedule()` / `plan_schedule`); dropped ops are left out."""
    out = collections.OrderedDict()
    for i, p in enumerate(primary):
        if p >= 0:
            out.setdefault(int(p), []).append(i)
    return out


SCHED_STATS_ONLY, SCHED_LN_ON_LOAD, SCHED_LN_IN_EPILOGUE, SCHED_LN_INPUT_UNSTORED = 1, 2, 4, 8


def step_work(plan, ops, members, flags=None):
    """(family, flops, bytes) of one scheduled step. The members' own work,
    less what fusion removes: each absorbed op (an epilogue or a forwarded
    Copy) consumed a tensor its producer no longer writes and it no longer
    reads, the size of its own output. A LayerNorm that the epilogue writes
    whole (SCHED_LN_IN_EPILOGUE) normalises a tensor that other ops read too,
    so its producer still writes it and only the LayerNorm's read goes -
    unless no other op reads it (SCHED_LN_INPUT_UNSTORED). A LayerNorm
    reduced to its statistics reads its input and writes 8 bytes per pixel."""
    p = members[0]
    f, b = op_work(plan, ops[p])
    fam = [KINDS[ops[p].kind]]
    fl = 0 if flags is None else int(flags[p])
    if fl & SCHED_STATS_ONLY:
        o = ops[p]
        f, b = 3 * o.c * o.hw, 4 * o.c * o.hw + 8 * o.hw
        fam = ["ln_stats"]
    elif fl & SCHED_LN_ON_LOAD:
        fam = [fam[0] + "(ln)"]
    for j in members[1:]:
        fj, bj = op_work(plan, ops[j])
        c, h, w = plan.buf(ops[j].dst)
        f += fj
        fj_flags = 0 if flags is None else int(flags[j])
        whole_ln = fj_flags & SCHED_LN_IN_EPILOGUE and not fj_flags & SCHED_LN_INPUT_UNSTORED
        b += bj - (4 if whole_ln else 8) * c * h * w
        if KINDS[ops[j].kind] in TAILS:
            fam.append(KINDS[ops[j].kind])
    return "+".join(fam), f, b


def census(plan):
    """{kind: [ops, flops, bytes]} over the whole plan."""
    out = collections.OrderedDict()
    for op in plan.ops():
        f, b = op_work(plan, op)
        e = out.setdefault(KINDS[op.kind], [0, 0, 0])
        e[0] += 1
        e[1] += f
        e[2] += b
    return out


# Op kinds whose products run on the tensor cores as the 3xTF32 split: each
# useful multiply-add is issued as three TF32 products (a_hi*b_hi, a_hi*b_lo,
# a_lo*b_hi).
TENSOR_KINDS = ("conv1x1", "conv3x3", "conv4x4s2", "convt2x2", "gate_mm")
TF32_PRODUCTS = 3


def roofline(family, flops, nbytes, seconds, hbm_gbs, tf32_tflops):
    """The roofline of one step family over `seconds` of device time.

    The bound is whichever of HBM (algorithmic bytes at the measured copy
    bandwidth) and the tensor pipe (issued TF32 FLOPs, three per useful
    multiply-add, at the TF32 dense rate) takes longer; `frac` is the
    family's attainable time over its measured time, i.e. achieved / peak on
    that bound. Families that are not contractions are HBM-bound."""
    base = family.split()[0].split("+")[0].split("(")[0]
    issued = flops * (TF32_PRODUCTS if base in TENSOR_KINDS else 0)
    t_mem = nbytes / (hbm_gbs * 1e9)
    t_tc = issued / (tf32_tflops * 1e12) if issued else 0.0
    if t_tc > t_mem:
        return {"bound": "tensor", "achieved": issued / seconds / 1e12, "peak": tf32_tflops, "unit": "TFLOP/s",
                "frac": t_tc / seconds, "frac_hbm": t_mem / seconds}
    return {"bound": "hbm", "achieved": nbytes / seconds / 1e9, "peak": hbm_gbs, "unit": "GB/s",
            "frac": t_mem / seconds, "frac_tensor": t_tc / seconds}
