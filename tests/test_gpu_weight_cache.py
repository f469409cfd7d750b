"""The converted-weights cache (mx_gpu_new_cached): the tensor-core layouts an
executor derives from the checkpoint (src/weights.rs:57-211 gives the plan's
own; the executor adds tap-major orders, TF32 hi/lo halves and transposes)
written to a file and read back by the next executor. The bar: passes built
from the cache are bit for bit those of an executor that derived everything,
at the size the cache was written for and at another, and a cache made from
other weights is not used."""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def image(synth, seed, h, w):
    return synth.image_uniform(synth.input_rng(seed), h, w)


def test_cached_layouts_give_the_same_pass(mx, synth, checkpoint, tmp_path):
    w = mx.Weights(checkpoint("S-2", 0, 0.5, rich=True))
    plan = mx.Plan(w, 128, 192)
    x = image(synth, 3, 128, 192)
    g0 = mx.Gpu(plan)
    want = g0.run(x)
    g0.close()
    path = str(tmp_path / "s2.mxw")
    g1 = mx.Gpu(plan, weight_cache=path)
    loaded, derived, saved = g1.weight_cache_info()
    assert loaded == 0 and derived > 0 and saved == 1 and os.path.getsize(path) > 0
    assert np.array_equal(g1.run(x), want)
    g1.close()
    g2 = mx.Gpu(plan, weight_cache=path)
    assert g2.weight_cache_info() == (derived, 0, 0)
    assert np.array_equal(g2.run(x), want)
    g2.close()
    # another image size: the layouts do not depend on it
    plan2 = mx.Plan(w, 64, 64)
    x2 = image(synth, 4, 64, 64)
    g3 = mx.Gpu(plan2)
    want2 = g3.run(x2)
    g3.close()
    g4 = mx.Gpu(plan2, weight_cache=path)
    loaded4, derived4, _ = g4.weight_cache_info()
    assert loaded4 > 0
    assert np.array_equal(g4.run(x2), want2)
    g4.close()


def test_a_cache_of_other_weights_is_not_used(mx, synth, checkpoint, tmp_path):
    path = str(tmp_path / "s1.mxw")
    x = image(synth, 5, 64, 128)
    pa = mx.Plan(mx.Weights(checkpoint("S-1", 1, 0.5)), 64, 128)
    ga = mx.Gpu(pa, weight_cache=path)
    derived_a = ga.weight_cache_info()[1]
    ga.close()
    pb = mx.Plan(mx.Weights(checkpoint("S-1", 2, 0.5)), 64, 128)
    gb = mx.Gpu(pb)
    want = gb.run(x)
    gb.close()
    gc = mx.Gpu(pb, weight_cache=path)
    loaded, derived, saved = gc.weight_cache_info()
    # only layouts of weights the two checkpoints share bit for bit (say a
    # bias both initialise to zero) may come from the file
    assert loaded + derived == derived_a and derived > derived_a // 2 and saved == 1
    assert np.array_equal(gc.run(x), want)
    gc.close()
    # the file now holds the second checkpoint's layouts
    gd = mx.Gpu(pb, weight_cache=path)
    assert gd.weight_cache_info()[1] == 0
    gd.close()


def test_a_file_that_is_not_a_cache_is_refused(mx, checkpoint, tmp_path):
    path = tmp_path / "not_a_cache.mxw"
    path.write_bytes(b"PK\x03\x04 something else entirely")
    plan = mx.Plan(mx.Weights(checkpoint("S-1", 1, 0.5)), 64, 64)
    with pytest.raises(mx.MaximError, match="not a converted-weights cache") as e:
        mx.Gpu(plan, weight_cache=str(path))
    assert e.value.code == -2  # MX_E_IO
