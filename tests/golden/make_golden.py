"""Generate the golden fixtures in this directory from the REFERENCE itself.

    python tests/golden/make_golden.py /path/to/maxim-rs     (the reference checkout)

Runs the reference's PyTorch transcription of MAXIM (`tools/reference.py`,
the model class `Maxim` and its `preprocess`) on seeded synthetic weights and
inputs, and stores what it computes. The reference tree is needed only to
regenerate the fixtures; the tests read the committed .npz files.

Weights are regenerated at test time from the recorded (variant, seed, gain,
rich) by `maxim-rs_b200.synth.make_params`; the fixture stores a SHA-256 of the
weight bytes so a test can tell a changed generator from a changed model.

Fixture contents (float32):
  input        the padded [3][H][W] image the model ran on
  final        the last stage's full-resolution output (`outs[-1][-1]`)
  t/<name>     a selection of the named activations (`Maxim.rec`), the same
               names the plan records as dumps (src/model.rs `rec` calls)
"""
import hashlib
import importlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
mx = importlib.import_module("maxim-rs_b200")
synth = importlib.import_module("maxim-rs_b200.synth")

# (name, variant, H, W, seed, gain, rich, traced names)
CASES = [
    ("s2_64_he", "S-2", 64, 64, 0, 1.0, False,
     ["stage0_input_conv0", "stage0_input_conv2", "stage0_enc2_out", "stage0_global", "stage0_skip2",
      "stage0_skip0", "stage0_dec2", "stage0_sam2", "stage0_out0", "stage1_global", "stage1_dec1", "stage1_out0"]),
    ("s2_64_rich", "S-2", 64, 64, 5, 0.5, True,
     ["stage0_input_conv1", "stage0_enc1_out", "stage0_global", "stage0_skip1", "stage0_out0", "stage1_global",
      "stage1_out0"]),
    ("s3_64x128", "S-3", 64, 128, 1, 0.5, False, ["stage0_global", "stage1_global", "stage2_global"]),
    ("m1_64", "M-1", 64, 64, 6, 0.5, False, ["stage0_global", "stage0_skip2"]),
]


def weights_digest(params):
    h = hashlib.sha256()
    for k in sorted(params):
        h.update(k.encode())
        h.update(np.ascontiguousarray(params[k], np.float32).tobytes())
    return h.hexdigest()


def main(ref_root):
    sys.path.insert(0, os.path.join(ref_root, "tools"))
    import torch
    reference = importlib.import_module("reference")
    torch.set_num_threads(os.cpu_count() or 1)
    for name, variant, H, W, seed, gain, rich, traced in CASES:
        params = synth.make_params(variant, seed, gain, rich)
        rng = synth.input_rng(seed)
        img = synth.image_uniform(rng, H, W)
        m = reference.Maxim(params, reference.model_config(variant))
        m.trace = {}
        with torch.no_grad():
            outs = m(torch.from_numpy(img).unsqueeze(0))
        out = {"input": img, "final": outs[-1][-1][0].numpy().astype(np.float32),
               "meta_variant": np.array(variant), "meta_seed": np.array(seed), "meta_gain": np.array(gain),
               "meta_rich": np.array(rich), "meta_weights_sha256": np.array(weights_digest(params))}
        for t in traced:
            out["t/" + t] = m.trace[t][0].numpy().astype(np.float32)
        path = os.path.join(HERE, name + ".npz")
        np.savez_compressed(path, **out)
        print("wrote", path, os.path.getsize(path), "bytes")

    # The pad pipeline: reference.preprocess (make_shape_even + the centred
    # reflect to a multiple of 64) on odd and even sizes.
    rng = np.random.default_rng(7)
    pad = {}
    for i, (h, w) in enumerate([(37, 53), (22, 22), (33, 33), (64, 100), (101, 64), (131, 67)]):
        a = rng.random((3, h, w), dtype=np.float32)
        p, even = reference.preprocess(torch.from_numpy(a).unsqueeze(0), 64)
        pad["in%d" % i] = a
        pad["out%d" % i] = p[0].numpy()
        pad["even%d" % i] = np.array(even)
    np.savez_compressed(os.path.join(HERE, "preprocess.npz"), **pad)
    print("wrote preprocess.npz")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <reference checkout>")
    main(sys.argv[1])
