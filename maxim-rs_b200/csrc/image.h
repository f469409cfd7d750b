// Image I/O and the reference eval pipeline's pad / crop (src/image.rs).
#pragma once

#include <cstdint>
#include <string>
#include <vector>

namespace mx {

// [c][h][w] floats in 0..1.
struct Image {
  int64_t c = 0, h = 0, w = 0;
  std::vector<float> data;
  Image() = default;
  Image(int64_t c_, int64_t h_, int64_t w_) : c(c_), h(h_), w(w_), data(size_t(c_ * h_ * w_), 0.0f) {}
};

// An 8-bit PNG (gray, gray+alpha, RGB, RGBA; non-interlaced) as [3][h][w]/255,
// gray expanded to RGB (`read_png_stream`, src/image.rs:40-70).
Image read_png_bytes(const uint8_t* bytes, size_t n, const std::string& what);
// The same PNG's 8-bit samples as decoded, interleaved RGB (gray expanded),
// h x w x 3 bytes: what the device-side pipeline takes.
struct Rgb8 {
  int64_t h = 0, w = 0;
  std::vector<uint8_t> data;
};
Rgb8 decode_png_rgb8(const uint8_t* bytes, size_t n, const std::string& what);
// Width and height from the IHDR chunk alone (no decompression).
std::pair<int64_t, int64_t> png_size(const uint8_t* bytes, size_t n, const std::string& what);
Image read_png(const std::string& path);
// RGB 8-bit, clamp then round half up (src/image.rs:82-104).
std::vector<uint8_t> encode_png(const Image& img);
// An RGB 8-bit PNG from interleaved h x w x 3 samples, as they are; `level`
// is zlib's compression level (the pixels do not depend on it).
std::vector<uint8_t> encode_png_rgb8(const uint8_t* rgb, int64_t h, int64_t w, int level = 6);
void write_png(const std::string& path, const Image& img);

// Flax SAME padding for one axis (src/image.rs:108-112).
std::pair<int64_t, int64_t> same_pad(int64_t size, int64_t stride, int64_t k);

struct Padded {
  Image img;
  int64_t orig_h, orig_w, even_h, even_w;
};
// Even reflect (bottom/right by one), then centred reflect to a multiple of
// `factor`; refuses a pad that is not smaller than the dimension it mirrors
// (src/image.rs:171-207).
Padded preprocess(const Image& img, int64_t factor);
// The shapes preprocess produces for an h x w image, without the pixels: the
// even shape, the centred pad before each axis (top / left) and the padded
// shape (even + twice that pad). Throws the same refusal as preprocess.
struct PadGeometry {
  int64_t even_h, even_w, top, left, h, w;
};
PadGeometry pad_geometry(int64_t h, int64_t w, int64_t factor);
// Centred on the even shape, then cropped to the original size
// (src/image.rs:233-246).
Image crop_out(const Image& img, int64_t orig_h, int64_t orig_w, int64_t even_h, int64_t even_w);

}  // namespace mx
