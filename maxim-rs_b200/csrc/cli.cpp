// `maxim`: restore one image with a MAXIM checkpoint on a B200
// (the reference's CLI, src/main.rs:17-156, over this library's C ABI).
//
//     maxim -m maxim-s3.safetensors -i in.png -o out.png
//     maxim -m maxim-s3.safetensors --batch in_dir out_dir [--devices 0,1,..|all]
//
// The plan is built for the padded input shape (reflect pad to a multiple of
// 64, src/image.rs:171-207), run on the GPU executor, and the result is
// cropped back the way the reference eval script does. There is no CPU
// backend here: a missing driver is an error, never a silent fallback.
#include <dirent.h>

#include <cerrno>

#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <unistd.h>
#include <map>
#include <string>
#include <thread>
#include <vector>

#include "maxim_b200.h"

namespace {

const char* kVersion = "0.1.0";

[[noreturn]] void usage() {
  fprintf(stderr,
          "maxim %s - MAXIM image restoration on B200 (sm_100a)\n\n"
          "USAGE:\n    maxim --model <weights.safetensors> -i <in.png> -o <out.png> [options]\n\n"
          "OPTIONS:\n"
          "    -m, --model <path>    converted .safetensors checkpoint\n"
          "    -i, --input <path>    input PNG, or - for stdin (default: stdin)\n"
          "    -o, --output <path>   output PNG, or - for stdout (default: stdout)\n"
          "        --device <dev>    gpu (the only backend of this build)\n"
          "        --gpu             same as --device gpu\n"
          "        --gpu-index <n>   which CUDA device (default 0)\n"
          "        --profile         per-op-kind device time of the pass\n"
          "        --factor <n>      pad to a multiple of n (default 64, as the reference)\n"
          "        --batch <in> <out>  restore every .png of directory <in> into <out>, images\n"
          "                          round-robin over the devices (one worker per GPU)\n"
          "        --devices <list>  the batch's CUDA devices: comma-separated, or all (default)\n"
          "    -q, --quiet           no progress output\n"
          "    -h, --help            this text\n"
          "    -V, --version         print the version\n",
          kVersion);
  exit(2);
}

std::string last_error() {
  char buf[4096];
  mx_last_error(buf, sizeof(buf));
  return buf;
}

int fail(const std::string& what) {
  fprintf(stderr, "maxim: %s%s\n", what.empty() ? "" : (what + ": ").c_str(), last_error().c_str());
  return 1;
}

std::vector<uint8_t> read_all(FILE* f) {
  std::vector<uint8_t> v;
  uint8_t buf[1 << 16];
  size_t n;
  while ((n = fread(buf, 1, sizeof(buf), f)) > 0) v.insert(v.end(), buf, buf + n);
  return v;
}

// `--batch`: every PNG of a directory, grouped by padded shape (one plan per
// shape, the shape read from each PNG's header), each group through the batch
// runner's PNG path over the chosen devices: the workers decode and encode
// the PNGs while the GPUs run, and pad, crop and round on the device. A file
// whose header cannot be read or that is too small to pad is reported and
// skipped; an image the runner could not restore is reported; the others are
// written. Exit status 1 if anything failed.
int run_batch(mx_weights* w, const std::string& in_dir, const std::string& out_dir, std::vector<int32_t> devices,
              int factor, bool quiet) {
  std::vector<std::string> names;
  if (DIR* d = opendir(in_dir.c_str())) {
    while (dirent* e = readdir(d)) {
      std::string n = e->d_name;
      if (n.size() > 4 && n.compare(n.size() - 4, 4, ".png") == 0) names.push_back(n);
    }
    closedir(d);
  } else {
    fprintf(stderr, "maxim: cannot read directory %s\n", in_dir.c_str());
    return 1;
  }
  std::sort(names.begin(), names.end());
  if (devices.empty()) {
    int n = 0;
    if (mx_device_count(&n) != MX_OK || n == 0) return fail("cuda");
    for (int i = 0; i < n; ++i) devices.push_back(i);
  }
  std::map<std::pair<int32_t, int32_t>, std::vector<std::string>> groups;
  int failed = 0, written = 0;
  for (const auto& n : names) {
    const std::string path = in_dir + "/" + n;
    uint8_t head[64];
    size_t got = 0;
    if (FILE* f = fopen(path.c_str(), "rb")) {
      got = fread(head, 1, sizeof(head), f);
      fclose(f);
    }
    int32_t h = 0, wd = 0, ph = 0, pw = 0;
    if (mx_png_size_mem(head, got, &h, &wd) != MX_OK || mx_pad_geometry(h, wd, factor, &ph, &pw, nullptr, nullptr) != MX_OK) {
      fprintf(stderr, "maxim: %s: %s (skipped)\n", n.c_str(), last_error().c_str());
      ++failed;
      continue;
    }
    groups[{ph, pw}].push_back(n);
  }
  for (auto& kv : groups) {
    auto& items = kv.second;
    mx_plan_handle* plan = nullptr;
    if (mx_plan_build(w, kv.first.first, kv.first.second, 0, &plan) != MX_OK) {
      fprintf(stderr, "maxim: plan for %dx%d: %s\n", kv.first.second, kv.first.first, last_error().c_str());
      failed += int(items.size());
      continue;
    }
    const mx_plan* pv = mx_plan_view(plan);
    mx_batch_config cfg{pv, 0};
    mx_batch* b = nullptr;
    auto t0 = std::chrono::steady_clock::now();
    if (mx_batch_new(&cfg, devices.data(), int32_t(devices.size()), nullptr, &b) != MX_OK) {
      fprintf(stderr, "maxim: %dx%d: %s\n", kv.first.second, kv.first.first, last_error().c_str());
      failed += int(items.size());
      mx_plan_free(plan);
      continue;
    }
    std::vector<std::string> ins, outs;
    for (const auto& n : items) ins.push_back(in_dir + "/" + n), outs.push_back(out_dir + "/" + n);
    std::vector<const char*> ip, op;
    for (size_t i = 0; i < items.size(); ++i) ip.push_back(ins[i].c_str()), op.push_back(outs[i].c_str());
    std::vector<int32_t> st(items.size(), 0);
    auto t1 = std::chrono::steady_clock::now();
    const int rc = mx_batch_run_png(b, int32_t(items.size()), ip.data(), op.data(), factor, st.data());
    auto t2 = std::chrono::steady_clock::now();
    if (rc != MX_OK) fprintf(stderr, "maxim: %s\n", last_error().c_str());
    std::vector<mx_batch_worker> ws(size_t(mx_batch_worker_count(b)));
    mx_batch_workers(b, ws.data(), int32_t(ws.size()));
    if (!quiet) {
      fprintf(stderr, "maxim: %zu image(s) at %dx%d on %zu device(s): setup %.2fs, run %.2fs\n", items.size(),
              kv.first.second, kv.first.first, ws.size(), std::chrono::duration<double>(t1 - t0).count(),
              std::chrono::duration<double>(t2 - t1).count());
      for (const auto& x : ws)
        fprintf(stderr, "maxim:   device %d: %s, %d image(s)%s%s\n", x.device,
                x.state == MX_WORKER_READY ? "ready" : "failed", x.images_done, x.error[0] ? " - " : "", x.error);
    }
    for (size_t i = 0; i < items.size(); ++i) {
      if (st[i] != MX_OK) {
        fprintf(stderr, "maxim: %s: not restored (status %d)\n", items[i].c_str(), st[i]);
        ++failed;
      } else {
        ++written;
      }
    }
    mx_batch_free(b);
    mx_plan_free(plan);
  }
  if (!quiet) fprintf(stderr, "maxim: wrote %d image(s) to %s, %d failed\n", written, out_dir.c_str(), failed);
  return failed ? 1 : 0;
}

const char* kKind[] = {"copy", "add", "mul", "gate", "gelu", "lrelu", "sigmoid", "chanln", "chanmean",
                       "chanscale", "conv1x1", "conv3x3", "convdown", "convt", "gatemm", "blockperm",
                       "resize", "down"};

}  // namespace

int main(int argc, char** argv) {
  if (argc < 2) usage();
  std::string model, input = "-", output = "-", device = "gpu", batch_in, batch_out, devices_arg = "all";
  int gpu_index = 0, factor = 64;
  bool quiet = false, profile = false;
  for (int i = 1; i < argc; ++i) {
    std::string a = argv[i];
    auto next = [&]() -> std::string {
      if (i + 1 >= argc) usage();
      return argv[++i];
    };
    if (a == "-m" || a == "--model") model = next();
    else if (a == "-i" || a == "--input") input = next();
    else if (a == "-o" || a == "--output") output = next();
    else if (a == "--device") device = next();
    else if (a == "--gpu") device = "gpu";
    else if (a == "--cpu") device = "cpu";
    else if (a == "--gpu-index") gpu_index = atoi(next().c_str());
    else if (a == "--factor") factor = atoi(next().c_str());
    else if (a == "--batch") batch_in = next(), batch_out = next();
    else if (a == "--devices") devices_arg = next();
    else if (a == "--profile" || a == "--timeline") profile = true;
    else if (a == "-q" || a == "--quiet") quiet = true;
    else if (a == "-h" || a == "--help") usage();
    else if (a == "-V" || a == "--version") {
      printf("maxim %s\n", kVersion);
      return 0;
    } else {
      fprintf(stderr, "maxim: unknown argument `%s`\n", a.c_str());
      usage();
    }
  }
  if (model.empty()) {
    fprintf(stderr, "maxim: --model is required\n");
    usage();
  }
  if (device != "gpu") {
    fprintf(stderr, "maxim: this build runs on the GPU only (there is no CPU backend); got --device %s\n",
            device.c_str());
    return 1;
  }
  if (factor <= 0) factor = 64;

  mx_weights* w = nullptr;
  if (mx_weights_open(model.c_str(), &w) != MX_OK) return fail("");
  char variant[16];
  mx_weights_variant(w, variant, sizeof(variant));

  if (!batch_in.empty()) {
    std::vector<int32_t> devs;
    if (devices_arg != "all") {
      size_t p = 0;
      while (p <= devices_arg.size()) {
        size_t q = devices_arg.find(',', p);
        if (q == std::string::npos) q = devices_arg.size();
        if (q > p) devs.push_back(int32_t(atoi(devices_arg.substr(p, q - p).c_str())));
        p = q + 1;
      }
    }
    if (mx_driver_ready() != MX_OK) return fail("cuda");
    const int rc = run_batch(w, batch_in, batch_out, devs, factor, quiet);
    mx_weights_free(w);
    return rc;
  }

  // The PNG's size comes from its header, so the plan can be built and the
  // executor brought up (weights converted and uploaded) while a second
  // thread decodes the pixels. The per-pixel steps either side of the pass
  // (divide by 255, reflect pad, crop, 8-bit rounding) run on the device, and
  // only 8-bit images cross PCIe.
  std::vector<uint8_t> bytes;
  const std::string src_name = input == "-" ? "stdin" : input;
  if (input == "-") {
    bytes = read_all(stdin);
  } else {
    FILE* f = fopen(input.c_str(), "rb");
    if (!f) {
      fprintf(stderr, "maxim: %s: %s\n", input.c_str(), strerror(errno));
      return 1;
    }
    bytes = read_all(f);
    fclose(f);
  }
  int32_t img_h = 0, img_w = 0, pad_h = 0, pad_w = 0, even_h = 0, even_w = 0;
  if (mx_png_size_mem(bytes.data(), bytes.size(), &img_h, &img_w) != MX_OK) return fail(src_name);
  if (mx_pad_geometry(img_h, img_w, factor, &pad_h, &pad_w, &even_h, &even_w) != MX_OK) return fail("");
  if (!quiet)
    fprintf(stderr, "maxim %s: %dx%d -> padded %dx%d (even %dx%d), variant %s\n", kVersion, img_w, img_h, pad_w,
            pad_h, even_w, even_h, variant);
  mx_image8 img{};
  int dec_rc = MX_OK;
  std::string dec_err;
  std::thread decoder([&] {
    dec_rc = mx_png_read_rgb8_mem(bytes.data(), bytes.size(), &img);
    if (dec_rc != MX_OK) dec_err = last_error();  // the message slot is per thread
  });
  struct Joiner {
    std::thread& t;
    ~Joiner() {
      if (t.joinable()) t.join();
    }
  } joiner{decoder};

  auto t0 = std::chrono::steady_clock::now();
  mx_plan_handle* plan = nullptr;
  if (mx_plan_build(w, pad_h, pad_w, 0, &plan) != MX_OK) return fail("");
  const mx_plan* pv = mx_plan_view(plan);
  if (!quiet)
    fprintf(stderr, "maxim: plan %d ops, %d buffers, arena %.1f MiB\n", pv->n_ops, pv->n_bufs,
            pv->arena_len * 4.0 / 1048576.0);

  if (mx_driver_ready() != MX_OK) return fail("cuda");
  mx_gpu* gpu = nullptr;
  if (mx_gpu_new(gpu_index, pv, &gpu) != MX_OK) return fail("");
  mx_gpu_stats st{};
  mx_gpu_get_stats(gpu, &st);
  if (!quiet)
    fprintf(stderr, "maxim: device %s, %lld kernel launches per pass, weights %.1f MiB\n", st.device_name,
            (long long)st.kernels, st.weight_bytes / 1048576.0);
  if (profile) mx_gpu_set_timeline(gpu, 1);
  decoder.join();
  if (dec_rc != MX_OK) {
    fprintf(stderr, "maxim: %s: %s\n", src_name.c_str(), dec_err.c_str());
    return 1;
  }
  std::vector<uint8_t> out(size_t(img_h) * size_t(img_w) * 3);
  auto t1 = std::chrono::steady_clock::now();
  if (mx_gpu_run_rgb8(gpu, img.data, img_h, img_w, factor, out.data()) != MX_OK) return fail("");
  auto t2 = std::chrono::steady_clock::now();
  if (!quiet)
    fprintf(stderr, "maxim: setup %.2fs, pass %.1f ms\n", std::chrono::duration<double>(t1 - t0).count(),
            std::chrono::duration<double, std::milli>(t2 - t1).count());
  if (profile) {
    std::vector<float> per(size_t(pv->n_ops));
    float total = 0.0f;
    if (mx_gpu_timeline(gpu, per.data(), pv->n_ops, &total) == MX_OK) {
      std::map<std::string, std::pair<double, int>> by;
      for (int32_t i = 0; i < pv->n_ops; ++i) {
        auto& e = by[kKind[pv->ops[i].kind]];
        e.first += per[size_t(i)];
        e.second += 1;
      }
      printf("timeline: %.2f ms total, %d ops\n%-10s %7s %9s %7s\n", total, pv->n_ops, "op", "count", "total ms",
             "share");
      for (auto& kv : by)
        printf("%-10s %7d %9.2f %6.1f%%\n", kv.first.c_str(), kv.second.second, kv.second.first,
               100.0 * kv.second.first / (total > 0 ? total : 1));
    }
  }
  mx_image8 restored{3, img_h, img_w, out.data()};
  if (output == "-") {
    // The library writes files; stream through a temporary for stdout.
    char tmpl[] = "/tmp/maxim_out_XXXXXX";
    int fd = mkstemp(tmpl);
    if (fd < 0) {
      fprintf(stderr, "maxim: cannot create a temporary file for stdout\n");
      return 1;
    }
    close(fd);
    if (mx_png_write_rgb8(tmpl, &restored) != MX_OK) return fail("stdout");
    FILE* f = fopen(tmpl, "rb");
    auto obytes = read_all(f);
    fclose(f);
    unlink(tmpl);
    fwrite(obytes.data(), 1, obytes.size(), stdout);
  } else {
    if (mx_png_write_rgb8(output.c_str(), &restored) != MX_OK) return fail("");
    if (!quiet) fprintf(stderr, "maxim: wrote %s\n", output.c_str());
  }
  mx_image8_free(&img);
  mx_gpu_free(gpu);
  mx_plan_free(plan);
  mx_weights_free(w);
  return 0;
}
