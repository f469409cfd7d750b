"""The allocation-free channel mean (`mx_channel_mean_noalloc`).

It exists for callers that cannot allocate device memory: code running
inside a CUDA stream capture, or an engine that gives the GPU a fixed budget
up front. They pass their own input and output, and the entry point keeps its
partial sums in a fixed device array inside the library instead of in
allocated scratch. This test drives it through the C ABI and checks it against
the executor's own channel mean (the existing path, which allocates its
scratch when the handle is created) on the same activation, on two calls in
a row: the second call must not see anything the first one left behind. The
two share the partition and the kernels, so the results must be bit-identical
(tolerance zero).

It lives in its own file, collected last, and passes alone in a fresh process
as well as after the other tests.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MX_OP_CHAN_MEAN = 8


def executor_channel_mean(mx, checkpoint, synth):
    """The first ChanMean op of an S-1 plan, run by the executor's per-op walk:
    returns (its input as [c][h*w], the executor's [c] result)."""
    w = mx.Weights(checkpoint("S-1", 7, 0.5, True))
    img = synth.image_uniform(synth.input_rng(9), 128, 192)
    plan = mx.Plan(w, 128, 192)
    gpu = mx.Gpu(plan)
    gpu.begin(img)
    for i, op in enumerate(plan.ops()):
        gpu.step_op(i)
        if op.kind == MX_OP_CHAN_MEAN:
            x = gpu.read_buf(op.src)
            ref = gpu.read_buf(op.dst).reshape(-1)
            gpu.close()
            c = x.shape[0]
            return x.reshape(c, -1), ref
    raise AssertionError("the plan has no channel-mean op")


def test_channel_mean_without_allocation_matches_the_executor(mx, checkpoint, synth):
    import torch
    x, ref = executor_channel_mean(mx, checkpoint, synth)
    c, npix = x.shape
    scale = float(np.abs(ref).max())
    stream = torch.cuda.current_stream().cuda_stream
    # a dense NHWC tensor, and the same values as a channel view of a wider one
    dense = torch.from_numpy(np.ascontiguousarray(x.T)).cuda()
    wide = torch.zeros((npix, c + 32), dtype=torch.float32, device="cuda")
    wide[:, 16:16 + c] = dense
    for src, stride in ((dense, c), (wide[:, 16:], c + 32)):
        outs = []
        for _ in range(2):
            out = torch.full((c,), float("nan"), dtype=torch.float32, device="cuda")
            mx._native.channel_mean_noalloc(src.data_ptr(), npix, c, stride, out.data_ptr(), stream)
            torch.cuda.synchronize()
            outs.append(out.cpu().numpy())
        for got in outs:
            assert np.isfinite(got).all()
            assert np.array_equal(got, ref), float(np.abs(got.astype(np.float64) - ref).max()) / scale
        assert np.array_equal(outs[0], outs[1])


def test_channel_mean_without_allocation_rejects_oversized_input(mx):
    import torch
    x = torch.zeros((8, 512), dtype=torch.float32, device="cuda")
    out = torch.zeros(512, dtype=torch.float32, device="cuda")
    with pytest.raises(mx.MaximError, match="up to 256"):
        mx._native.channel_mean_noalloc(x.data_ptr(), 8, 512, 512, out.data_ptr(), 0)
