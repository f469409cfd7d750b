"""B200-native MAXIM forward pass.

The native library (libmaxim_b200.so, C ABI in include/maxim_b200.h) holds the
GPU executor and the C++ host contract; this package is its Python binding plus
the synthetic-checkpoint and synthetic-input generators (`synth`).
"""
from ._native import (Batch, Gpu, MaximError, Plan, Weights, crop_out, device_count, driver_ready, exported_symbols, lib,
                      pad_geometry, param_spec, plan_schedule, png_read, png_read_bytes, png_read_rgb8_bytes,
                      png_size, png_write, png_write_rgb8, preprocess)

__all__ = ["Batch", "Gpu", "MaximError", "Plan", "Weights", "crop_out", "device_count", "driver_ready", "exported_symbols",
           "lib", "pad_geometry", "param_spec", "plan_schedule", "png_read", "png_read_bytes", "png_read_rgb8_bytes",
           "png_size", "png_write", "png_write_rgb8", "preprocess"]
