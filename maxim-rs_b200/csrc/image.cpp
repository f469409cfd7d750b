#include "image.h"

#include <zlib.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <iterator>

#include "common.h"

namespace mx {

namespace {

uint32_t be32(const uint8_t* p) { return uint32_t(p[0]) << 24 | uint32_t(p[1]) << 16 | uint32_t(p[2]) << 8 | p[3]; }
void put32(std::vector<uint8_t>& v, uint32_t x) {
  v.push_back(uint8_t(x >> 24));
  v.push_back(uint8_t(x >> 16));
  v.push_back(uint8_t(x >> 8));
  v.push_back(uint8_t(x));
}

int paeth(int a, int b, int c) {
  int p = a + b - c, pa = std::abs(p - a), pb = std::abs(p - b), pc = std::abs(p - c);
  if (pa <= pb && pa <= pc) return a;
  if (pb <= pc) return b;
  return c;
}

// torch's / jax's reflect: mirror about the edge without repeating it.
int64_t reflect_index(int64_t i, int64_t n) {
  if (i < 0) return -i;
  if (i >= n) return 2 * n - 2 - i;
  return i;
}

Image reflect_pad2(const Image& img, int64_t top, int64_t bottom, int64_t left, int64_t right) {
  int64_t nh = img.h + top + bottom, nw = img.w + left + right;
  Image out(img.c, nh, nw);
  for (int64_t y = 0; y < nh; ++y) {
    int64_t sy = reflect_index(y - top, img.h);
    for (int64_t x = 0; x < nw; ++x) {
      int64_t sx = reflect_index(x - left, img.w);
      for (int64_t c = 0; c < img.c; ++c)
        out.data[size_t(c * nh * nw + y * nw + x)] = img.data[size_t(c * img.h * img.w + sy * img.w + sx)];
    }
  }
  return out;
}

// The smallest dimension the pad-to-`factor` reflection accepts, for the
// refusal message (src/image.rs:217-228).
int64_t min_dimension(int64_t factor) {
  for (int64_t d = 2; d < factor; d += 2) {
    int64_t up = ((d + factor) / factor) * factor;
    if ((up - d) / 2 < d) return d;
  }
  return factor;
}

// The refusal of an image too small to reflect out to a multiple of
// `factor` (src/image.rs:185-199).
[[noreturn]] void refuse_small(int64_t factor, const char* axis, int64_t dim, int64_t pad) {
  throw Error(fmt("this image is too small for MAXIM's %lld-multiple padding: the %s is %lld pixels and the "
                  "pipeline reflects it out to the next multiple of %lld, which is %lld pixels of padding a side - "
                  "a reflection needs less padding than the dimension it mirrors. The reference pipeline refuses "
                  "this input for the same reason (torch's reflect pad: `Padding size should be less than the "
                  "corresponding input dimension`). Give it an image at least %lld pixels on its %s.",
                  (long long)factor, axis, (long long)dim, (long long)factor, (long long)pad,
                  (long long)min_dimension(factor), axis));
}

}  // namespace

std::pair<int64_t, int64_t> same_pad(int64_t size, int64_t stride, int64_t k) {
  int64_t out = (size + stride - 1) / stride;
  int64_t total = std::max<int64_t>((out - 1) * stride + k - size, 0);
  return {total / 2, total - total / 2};
}

std::pair<int64_t, int64_t> png_size(const uint8_t* b, size_t n, const std::string& what) {
  static const uint8_t sig[8] = {137, 80, 78, 71, 13, 10, 26, 10};
  if (n < 8 || memcmp(b, sig, 8) != 0) throw Error(what + ": not a PNG file", MX_E_IO);
  // The IHDR chunk comes first: 8-byte signature, 4-byte length, "IHDR".
  if (n < 8 + 8 + 13 || memcmp(b + 12, "IHDR", 4) != 0) throw Error(what + ": PNG has no IHDR", MX_E_IO);
  const int64_t W = be32(b + 16), H = be32(b + 20);
  if (W == 0 || H == 0) throw Error(what + ": empty PNG", MX_E_IO);
  return {H, W};
}

Rgb8 decode_png_rgb8(const uint8_t* b, size_t n, const std::string& what) {
  static const uint8_t sig[8] = {137, 80, 78, 71, 13, 10, 26, 10};
  if (n < 8 || memcmp(b, sig, 8) != 0) throw Error(what + ": not a PNG file", MX_E_IO);
  size_t p = 8;
  uint32_t W = 0, H = 0;
  int depth = 0, ctype = -1, interlace = 0;
  std::vector<uint8_t> idat;
  bool seen_ihdr = false;
  while (p + 8 <= n) {
    uint32_t len = be32(b + p);
    const uint8_t* type = b + p + 4;
    if (p + 12 + size_t(len) > n) throw Error(what + ": truncated PNG chunk", MX_E_IO);
    const uint8_t* d = b + p + 8;
    if (!memcmp(type, "IHDR", 4)) {
      if (len < 13) throw Error(what + ": bad IHDR", MX_E_IO);
      W = be32(d);
      H = be32(d + 4);
      depth = d[8];
      ctype = d[9];
      interlace = d[12];
      seen_ihdr = true;
    } else if (!memcmp(type, "IDAT", 4)) {
      idat.insert(idat.end(), d, d + len);
    } else if (!memcmp(type, "IEND", 4)) {
      break;
    }
    p += 12 + size_t(len);
  }
  if (!seen_ihdr) throw Error(what + ": PNG has no IHDR", MX_E_IO);
  if (ctype == 3) throw Error(what + ": indexed PNG; re-save it as RGB", MX_E_IO);
  if (depth != 8) throw Error(fmt("%s: %d-bit PNG; only 8-bit samples are supported", what.c_str(), depth), MX_E_IO);
  if (interlace != 0) throw Error(what + ": interlaced PNG; re-save it without interlacing", MX_E_IO);
  int ch;
  switch (ctype) {
    case 0: ch = 1; break;
    case 2: ch = 3; break;
    case 4: ch = 2; break;
    case 6: ch = 4; break;
    default: throw Error(fmt("%s: unsupported PNG color type %d", what.c_str(), ctype), MX_E_IO);
  }
  if (W == 0 || H == 0) throw Error(what + ": empty PNG", MX_E_IO);
  size_t stride = size_t(W) * ch;
  std::vector<uint8_t> raw((stride + 1) * H);
  z_stream zs{};
  if (inflateInit(&zs) != Z_OK) throw Error(what + ": zlib init failed", MX_E_IO);
  zs.next_in = idat.data();
  zs.avail_in = uInt(idat.size());
  zs.next_out = raw.data();
  zs.avail_out = uInt(raw.size());
  int rc = inflate(&zs, Z_FINISH);
  size_t got = raw.size() - zs.avail_out;
  inflateEnd(&zs);
  if ((rc != Z_STREAM_END && rc != Z_OK && rc != Z_BUF_ERROR) || got != raw.size())
    throw Error(what + ": corrupt PNG image data", MX_E_IO);
  // Undo the per-row filters in place.
  std::vector<uint8_t> pix(stride * H);
  for (uint32_t y = 0; y < H; ++y) {
    uint8_t f = raw[y * (stride + 1)];
    const uint8_t* src = &raw[y * (stride + 1) + 1];
    uint8_t* cur = &pix[y * stride];
    const uint8_t* prev = y ? &pix[(y - 1) * stride] : nullptr;
    for (size_t i = 0; i < stride; ++i) {
      int a = i >= size_t(ch) ? cur[i - ch] : 0;
      int up = prev ? prev[i] : 0;
      int c = (prev && i >= size_t(ch)) ? prev[i - ch] : 0;
      int v = src[i];
      switch (f) {
        case 0: break;
        case 1: v += a; break;
        case 2: v += up; break;
        case 3: v += (a + up) / 2; break;
        case 4: v += paeth(a, up, c); break;
        default: throw Error(what + ": bad PNG filter type", MX_E_IO);
      }
      cur[i] = uint8_t(v);
    }
  }
  Rgb8 out;
  out.h = H, out.w = W;
  const size_t plane = size_t(H) * W;
  if (ch == 3) {
    out.data = std::move(pix);
    return out;
  }
  out.data.resize(plane * 3);
  for (size_t i = 0; i < plane; ++i) {
    const uint8_t* s = &pix[i * ch];
    uint8_t* d = &out.data[i * 3];
    if (ch <= 2) d[0] = d[1] = d[2] = s[0];
    else d[0] = s[0], d[1] = s[1], d[2] = s[2];
  }
  return out;
}

Image read_png_bytes(const uint8_t* b, size_t n, const std::string& what) {
  const Rgb8 px = decode_png_rgb8(b, n, what);
  Image img(3, px.h, px.w);
  const size_t plane = size_t(px.h) * px.w;
  for (size_t i = 0; i < plane; ++i) {
    const uint8_t* s = &px.data[i * 3];
    img.data[i] = s[0] / 255.0f;
    img.data[plane + i] = s[1] / 255.0f;
    img.data[2 * plane + i] = s[2] / 255.0f;
  }
  return img;
}

Image read_png(const std::string& path) {
  std::ifstream f(path, std::ios::binary);
  if (!f) throw Error(path + ": " + strerror(errno), MX_E_IO);
  std::vector<uint8_t> bytes((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
  return read_png_bytes(bytes.data(), bytes.size(), path);
}

std::vector<uint8_t> encode_png(const Image& img) {
  if (img.c != 3) throw Error("write_png: the image must have 3 channels");
  const int64_t H = img.h, W = img.w;
  std::vector<uint8_t> rgb(size_t(H * W * 3));
  size_t plane = size_t(H * W);
  for (int64_t y = 0; y < H; ++y)
    for (int64_t x = 0; x < W; ++x)
      for (int c = 0; c < 3; ++c) {
        float v = std::min(std::max(img.data[c * plane + size_t(y * W + x)], 0.0f), 1.0f);
        rgb[size_t((y * W + x) * 3 + c)] = uint8_t(v * 255.0f + 0.5f);
      }
  return encode_png_rgb8(rgb.data(), H, W);
}

std::vector<uint8_t> encode_png_rgb8(const uint8_t* rgb, int64_t H, int64_t W, int level) {
  if (H <= 0 || W <= 0) throw Error("write_png: empty image");
  std::vector<uint8_t> raw(size_t(H * (W * 3 + 1)));
  for (int64_t y = 0; y < H; ++y) {
    uint8_t* row = &raw[size_t(y * (W * 3 + 1))];
    row[0] = 0;
    memcpy(row + 1, rgb + size_t(y * W * 3), size_t(W * 3));
  }
  uLongf zlen = compressBound(uLong(raw.size()));
  std::vector<uint8_t> z(zlen);
  if (compress2(z.data(), &zlen, raw.data(), uLong(raw.size()), level) != Z_OK)
    throw Error("PNG compression failed");
  z.resize(zlen);
  std::vector<uint8_t> out = {137, 80, 78, 71, 13, 10, 26, 10};
  auto chunk = [&](const char* type, const std::vector<uint8_t>& data) {
    put32(out, uint32_t(data.size()));
    size_t at = out.size();
    out.insert(out.end(), type, type + 4);
    out.insert(out.end(), data.begin(), data.end());
    uint32_t crc = uint32_t(crc32(0, &out[at], uInt(out.size() - at)));
    put32(out, crc);
  };
  std::vector<uint8_t> ihdr;
  put32(ihdr, uint32_t(W));
  put32(ihdr, uint32_t(H));
  ihdr.insert(ihdr.end(), {8, 2, 0, 0, 0});
  chunk("IHDR", ihdr);
  chunk("IDAT", z);
  chunk("IEND", {});
  return out;
}

void write_png(const std::string& path, const Image& img) {
  auto bytes = encode_png(img);
  FILE* f = fopen(path.c_str(), "wb");
  if (!f) throw Error(path + ": " + strerror(errno), MX_E_IO);
  size_t wr = fwrite(bytes.data(), 1, bytes.size(), f);
  int rc = fclose(f);
  if (wr != bytes.size() || rc != 0) throw Error(path + ": write failed", MX_E_IO);
}

PadGeometry pad_geometry(int64_t h, int64_t w, int64_t factor) {
  if (h <= 0 || w <= 0 || factor <= 0) throw Error("pad_geometry: bad argument");
  const int64_t eh = h + h % 2, ew = w + w % 2;
  const int64_t hp = eh % factor ? ((eh + factor) / factor) * factor : eh;
  const int64_t wp = ew % factor ? ((ew + factor) / factor) * factor : ew;
  const int64_t padh = hp - eh, padw = wp - ew;
  struct Ax {
    const char* name;
    int64_t dim, pad;
  } axes[2] = {{"height", eh, padh / 2}, {"width", ew, padw / 2}};
  for (auto& a : axes)
    if (a.pad != 0 && a.pad >= a.dim) refuse_small(factor, a.name, a.dim, a.pad);
  PadGeometry g;
  g.even_h = eh, g.even_w = ew, g.top = padh / 2, g.left = padw / 2;
  g.h = eh + 2 * (padh / 2), g.w = ew + 2 * (padw / 2);
  return g;
}

Padded preprocess(const Image& img, int64_t factor) {
  int64_t h = img.h, w = img.w;
  int64_t ph = h % 2, pw = w % 2;
  Image even = (ph || pw) ? reflect_pad2(img, 0, ph, 0, pw) : img;
  int64_t eh = even.h, ew = even.w;
  int64_t hp = eh % factor ? ((eh + factor) / factor) * factor : eh;
  int64_t wp = ew % factor ? ((ew + factor) / factor) * factor : ew;
  int64_t padh = hp - eh, padw = wp - ew;
  struct Ax {
    const char* name;
    int64_t dim, pad;
  } axes[2] = {{"height", eh, padh / 2}, {"width", ew, padw / 2}};
  for (auto& a : axes)
    if (a.pad != 0 && a.pad >= a.dim) refuse_small(factor, a.name, a.dim, a.pad);
  Padded p;
  p.img = (padh || padw) ? reflect_pad2(even, padh / 2, padh / 2, padw / 2, padw / 2) : even;
  p.orig_h = h, p.orig_w = w, p.even_h = eh, p.even_w = ew;
  return p;
}

Image crop_out(const Image& img, int64_t orig_h, int64_t orig_w, int64_t even_h, int64_t even_w) {
  int64_t hs = img.h / 2 - even_h / 2, ws = img.w / 2 - even_w / 2;
  if (hs < 0 || ws < 0 || hs + orig_h > img.h || ws + orig_w > img.w)
    throw Error("crop_out: the crop does not fit inside the prediction");
  Image out(img.c, orig_h, orig_w);
  for (int64_t c = 0; c < img.c; ++c)
    for (int64_t y = 0; y < orig_h; ++y)
      for (int64_t x = 0; x < orig_w; ++x)
        out.data[size_t(c * orig_h * orig_w + y * orig_w + x)] =
            img.data[size_t(c * img.h * img.w + (hs + y) * img.w + (ws + x))];
  return out;
}

}  // namespace mx
