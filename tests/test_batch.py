"""The batch runner's host logic (mx_batch_*) without a GPU: a Python
executor stands in for the GPU one through the runner's executor interface,
and fails on purpose where a test needs it. Covers round-robin sharding,
worker status, a device that cannot be opened, a worker that fails mid-batch
(its unfinished images go to the others), and a batch nobody can finish (a
clean error, per-image status, no hang)."""
import threading

import numpy as np
import pytest

N_IN, N_OUT = 12, 12


class Fake:
    """y = 2 x + device; records which device ran which image (x[0])."""

    in_len, out_len = N_IN, N_OUT

    def __init__(self, bad_open=(), bad_run=(), fail_after=0):
        self.bad_open, self.bad_run, self.fail_after = set(bad_open), set(bad_run), fail_after
        self.log, self.closed, self.mu = [], [], threading.Lock()
        self.runs = {}

    def open(self, device):
        if device in self.bad_open:
            raise RuntimeError("cannot open device %d" % device)
        return {"device": device}

    def run(self, h, x, y):
        d = h["device"]
        with self.mu:
            self.runs[d] = self.runs.get(d, 0) + 1
            n = self.runs[d]
        if d in self.bad_run and n > self.fail_after:
            raise RuntimeError("device %d broke" % d)
        y[:] = 2 * x + d
        with self.mu:
            self.log.append((d, int(x[0])))

    def close(self, h):
        with self.mu:
            self.closed.append(h["device"])


def images(n):
    return [np.full(N_IN, i, np.float32) for i in range(n)]


@pytest.mark.timeout(60)
def test_round_robin_over_devices(mx):
    f = Fake()
    b = mx.Batch(devices=(0, 1, 2), executor=f)
    outs, st = b.run(images(10))
    assert st == [0] * 10
    for i, o in enumerate(outs):
        assert np.array_equal(o, 2 * np.full(N_OUT, i, np.float32) + (i % 3))
    assert sorted(f.log) == sorted((i % 3, i) for i in range(10))
    ws = b.workers()
    assert [w["images_done"] for w in ws] == [4, 3, 3]
    assert all(w["state"] == "ready" for w in ws)
    b.close()
    assert sorted(f.closed) == [0, 1, 2]


@pytest.mark.timeout(60)
def test_a_device_that_cannot_open_is_left_out(mx):
    f = Fake(bad_open={1})
    b = mx.Batch(devices=(0, 1, 2), executor=f)
    ws = b.workers()
    assert ws[1]["state"] == "failed" and "device 1" in ws[1]["error"]
    outs, st = b.run(images(6))
    assert st == [0] * 6
    assert {d for d, _ in f.log} == {0, 2}
    assert sorted(i for _, i in f.log) == list(range(6))


@pytest.mark.timeout(60)
def test_a_worker_that_fails_hands_its_images_to_the_others(mx):
    f = Fake(bad_run={1}, fail_after=1)  # device 1 restores one image, then breaks
    b = mx.Batch(devices=(0, 1, 2), executor=f)
    outs, st = b.run(images(12))
    assert st == [0] * 12
    for i, o in enumerate(outs):
        d = [dd for dd, ii in f.log if ii == i]
        assert len(d) == 1, (i, d)  # every image restored exactly once
        assert np.array_equal(o, 2 * np.full(N_OUT, i, np.float32) + d[0])
    ws = b.workers()
    assert ws[1]["state"] == "failed" and ws[1]["images_done"] == 1
    assert "device 1 failed on image 4" in ws[1]["error"]
    assert ws[0]["state"] == ws[2]["state"] == "ready"
    assert sum(w["images_done"] for w in ws) == 12


@pytest.mark.timeout(60)
def test_nobody_can_finish_a_clean_error_and_no_hang(mx):
    f = Fake(bad_run={0, 1})
    b = mx.Batch(devices=(0, 1), executor=f)
    with pytest.raises(mx.MaximError, match="3 of 3 images were not restored"):
        b.run(images(3))
    outs, st = b.run(images(3), raise_on_error=False)
    assert all(s != 0 for s in st)
    assert all(w["state"] == "failed" for w in b.workers())
    # A later batch on the same runner fails fast, too.
    with pytest.raises(mx.MaximError):
        b.run(images(2))


def test_no_device_can_open(mx):
    with pytest.raises(mx.MaximError, match="no device could take the batch"):
        mx.Batch(devices=(0, 1), executor=Fake(bad_open={0, 1}))


def test_empty_batch(mx):
    b = mx.Batch(devices=(0,), executor=Fake())
    outs, st = b.run([])
    assert outs == [] and st == []


def test_input_size_is_checked(mx):
    b = mx.Batch(devices=(0,), executor=Fake())
    with pytest.raises(ValueError):
        b.run([np.zeros(N_IN + 1, np.float32)])


def test_png_mode_needs_the_gpu_executor(mx, tmp_path):
    """mx_batch_run_png runs over the device-side image path, which a
    caller-supplied executor does not have: refused, nothing run."""
    ex = Fake()
    b = mx.Batch(devices=(0,), executor=ex)
    with pytest.raises(mx.MaximError, match="built-in GPU executor"):
        b.run_png([str(tmp_path / "a.png")], [str(tmp_path / "b.png")])
    assert ex.log == []
    b.close()
