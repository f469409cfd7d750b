// The batch runner: independent images sharded round-robin over GPUs, one
// worker thread and one executor handle (its own arena, weights, stream and
// CUDA graph) per device, no collective.
//
// The reference restores one image per process (src/main.rs:173-458) and
// stops at the first error. A batch over several GPUs needs more than that,
// so the runner adds host-side failure handling:
//   * each worker reports a status (ready / failed, the error that took it
//     out, the images it restored);
//   * a device whose executor cannot be built (say, the pass does not fit
//     its memory budget) is left out, and the batch runs on the others;
//   * a worker that fails on an image is retired, and the images it had not
//     finished - the failing one included - go round-robin to the workers
//     still standing; an image that no worker could restore keeps the error
//     code of its last attempt, and the call returns instead of hanging.
// Device-side waits are bounded in time by the kernels themselves, so every
// executor call returns.
//
// The executor is pluggable (mx_batch_executor): by default the GPU executor
// of this library; a caller may supply its own (a CPU path, or a fake that
// fails on purpose to exercise the handling above without a GPU).
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cerrno>
#include <chrono>
#include <condition_variable>
#include <cstdio>
#include <deque>
#include <cstring>
#include <exception>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "common.h"
#include "gpu_common.cuh"
#include "image.h"
#include "maxim_b200.h"

namespace mx {
namespace {

std::string last_message() {
  char buf[1024];
  mx_last_error(buf, sizeof(buf));
  return buf;
}

// The built-in executor: mx_gpu_* with pinned staging, so the caller's
// pageable images are copied once on the host and cross PCIe asynchronously.
// Two staging slots let a worker copy image j+1 in (and image j-1 out) on
// the host while the GPU runs image j.
struct GpuWorker {
  mx_gpu* g = nullptr;
  int device = 0;
  float* pin_in[2] = {nullptr, nullptr};
  float* pin_out[2] = {nullptr, nullptr};
  cudaEvent_t done[2] = {nullptr, nullptr};
  size_t in_len = 0, out_len = 0;
};

int gpu_open(void* ctx, int32_t device, void** handle) {
  const mx_batch_config* cfg = static_cast<const mx_batch_config*>(ctx);
  auto w = std::make_unique<GpuWorker>();
  w->device = device;
  int rc = mx_gpu_new_budget(device, cfg->plan, cfg->device_mem_budget, &w->g);
  if (rc != MX_OK) return rc;
  return guard([&] {
    const mx_buf& bi = cfg->plan->bufs[cfg->plan->input];
    const mx_buf& bo = cfg->plan->bufs[cfg->plan->output];
    w->in_len = size_t(bi.c * bi.h * bi.w);
    w->out_len = size_t(bo.c * bo.h * bo.w);
    MX_CUDA(cudaSetDevice(device));
    for (int k = 0; k < 2; ++k) {
      MX_CUDA(cudaMallocHost(&w->pin_in[k], w->in_len * 4));
      MX_CUDA(cudaMallocHost(&w->pin_out[k], w->out_len * 4));
      MX_CUDA(cudaEventCreateWithFlags(&w->done[k], cudaEventDisableTiming));
    }
    *handle = w.release();
  });
}

void gpu_close(void* ctx, void* handle) {
  GpuWorker* w = static_cast<GpuWorker*>(handle);
  if (!w) return;
  cudaSetDevice(w->device);
  mx_gpu_free(w->g);
  for (int k = 0; k < 2; ++k) {
    cudaFreeHost(w->pin_in[k]);
    cudaFreeHost(w->pin_out[k]);
    if (w->done[k]) cudaEventDestroy(w->done[k]);
  }
  delete w;
}

int gpu_run(void* ctx, void* handle, const float* input, float* output) {
  GpuWorker* w = static_cast<GpuWorker*>(handle);
  memcpy(w->pin_in[0], input, w->in_len * 4);
  int rc = mx_gpu_upload_input(w->g, w->pin_in[0]);
  if (rc == MX_OK) rc = mx_gpu_enqueue(w->g);
  if (rc == MX_OK) rc = mx_gpu_download_output(w->g, w->pin_out[0]);
  if (rc == MX_OK) rc = mx_gpu_sync(w->g);
  if (rc == MX_OK) memcpy(output, w->pin_out[0], w->out_len * 4);
  return rc;
}

// A worker's list of images on the GPU executor, two in flight: image j is
// enqueued (upload, pass, download into slot j % 2) before image j-1 is
// collected. Returns how many images from the front of the list completed;
// on a failure *rc and *msg say why, and the images from that index on are
// the caller's to hand to other workers (the one in flight behind the
// failing pass included: it ran on a pipeline that had given up).
size_t gpu_run_list(GpuWorker* w, const std::vector<int32_t>& list, const float* const* inputs,
                    float* const* outputs, int* rc, std::string* msg) {
  *rc = MX_OK;
  void* sp = nullptr;
  if ((*rc = mx_gpu_stream(w->g, &sp)) != MX_OK || (*rc = guard([&] { MX_CUDA(cudaSetDevice(w->device)); })) != MX_OK) {
    *msg = last_message();
    return 0;
  }
  cudaStream_t stream = static_cast<cudaStream_t>(sp);
  size_t done = 0;
  auto collect = [&](size_t j) -> bool {  // finish image j: wait, check, copy out
    const int k = int(j & 1);
    int r = guard([&] { MX_CUDA(cudaEventSynchronize(w->done[k])); });
    if (r == MX_OK) r = mx_gpu_poll(w->g);  // the pipelines' status word; image j+1 keeps running
    if (r != MX_OK) {
      *rc = r, *msg = last_message();
      return false;
    }
    memcpy(outputs[list[j]], w->pin_out[k], w->out_len * 4);
    done = j + 1;
    return true;
  };
  for (size_t j = 0; j < list.size(); ++j) {
    const int k = int(j & 1);
    if (j >= 2 && !collect(j - 2)) return done;
    memcpy(w->pin_in[k], inputs[list[j]], w->in_len * 4);
    int r = mx_gpu_upload_input(w->g, w->pin_in[k]);
    if (r == MX_OK) r = mx_gpu_enqueue(w->g);
    if (r == MX_OK) r = mx_gpu_download_output(w->g, w->pin_out[k]);
    if (r == MX_OK) r = guard([&] { MX_CUDA(cudaEventRecord(w->done[k], stream)); });
    if (r != MX_OK) {
      *rc = r, *msg = last_message();
      if (j >= 1) collect(j - 1);
      return done;
    }
  }
  for (size_t j = list.size() >= 2 ? list.size() - 2 : 0; j < list.size(); ++j)
    if (j >= done && !collect(j)) return done;
  return done;
}

// ---- PNG files in, PNG files out, through the device-side image path
//
// Per worker: this thread reads and decodes image j+1 and copies it into a
// pinned 8-bit slot while the GPU runs image j (two in flight, as above);
// finished images go to the worker's encoder thread, which compresses and
// writes them while the next ones run. Only 8-bit images cross PCIe. An
// image that cannot be read, decoded or written fails alone; a device
// failure retires the worker as above.
struct PngItem {
  int32_t img = -1;
  int64_t h = 0, w = 0;
  std::vector<uint8_t> rgb;
};

struct Encoder {
  std::mutex mu;
  std::condition_variable cv;       // an item was queued, or the queue was closed
  std::condition_variable room;     // an item was taken off the queue
  std::deque<PngItem> q;
  size_t limit = 4;                 // queued images a worker may run ahead of its encoders
  bool closed = false;
  std::vector<std::thread> th;
  // Closing drains the queue: the encoders finish what is queued, then exit.
  void close_and_join() {
    {
      std::lock_guard<std::mutex> l(mu);
      closed = true;
    }
    cv.notify_all();
    for (auto& t : th)
      if (t.joinable()) t.join();
  }
  ~Encoder() { close_and_join(); }
};

// zlib level of the batch's PNG writer. Deflate's cost depends on the data:
// at level 6 a noisy image with few distinct values (the output of an
// untrained checkpoint, say) took 340-420 ms to compress against 40 ms at
// level 1, for 40% more bytes; level 1 keeps the writer behind the GPU. The
// pixels are the same at every level.
constexpr int kBatchPngLevel = 1;

// Encoder threads per worker: the host threads left over after one per
// worker, shared out, at least one and at most four.
int encoder_threads(size_t workers) {
  const int hw = int(std::thread::hardware_concurrency());
  const int w = int(std::max<size_t>(workers, 1));
  return std::max(1, std::min(4, (hw - w) / w));
}

struct PngSlots {
  uint8_t* in[2] = {nullptr, nullptr};
  uint8_t* out[2] = {nullptr, nullptr};
  size_t cap = 0;
  ~PngSlots() {
    for (int k = 0; k < 2; ++k) {
      cudaFreeHost(in[k]);
      cudaFreeHost(out[k]);
    }
  }
};

// Returns how many images of `list` were dealt with (restored and handed to
// the encoder, or failed on their own); the rest, from the returned index
// on, are the caller's to hand to other workers after a device failure
// (*rc, *msg).
size_t png_run_list(GpuWorker* w, const std::vector<int32_t>& list, const char* const* in_paths,
                    const char* const* out_paths, int32_t factor, int n_encoders, std::vector<int32_t>& status,
                    std::vector<std::string>& why, int* rc, std::string* msg) {
  *rc = MX_OK;
  void* sp = nullptr;
  if ((*rc = mx_gpu_stream(w->g, &sp)) != MX_OK || (*rc = guard([&] { MX_CUDA(cudaSetDevice(w->device)); })) != MX_OK) {
    *msg = last_message();
    return 0;
  }
  cudaStream_t stream = static_cast<cudaStream_t>(sp);
  const size_t cap = w->in_len;  // floats of the padded [3][H][W] input = bytes of an H x W x 3 image
  PngSlots slots;
  int r0 = guard([&] {
    for (int k = 0; k < 2; ++k) {
      MX_CUDA(cudaMallocHost(&slots.in[k], cap));
      MX_CUDA(cudaMallocHost(&slots.out[k], cap));
    }
  });
  if (r0 != MX_OK) {
    *rc = r0, *msg = last_message();
    return 0;
  }
  Encoder enc;
  enc.limit = size_t(2 * n_encoders);
  for (int t = 0; t < n_encoders; ++t) enc.th.emplace_back([&] {
    for (;;) {
      PngItem it;
      {
        std::unique_lock<std::mutex> l(enc.mu);
        enc.cv.wait(l, [&] { return enc.closed || !enc.q.empty(); });
        if (enc.q.empty()) return;
        it = std::move(enc.q.front());
        enc.q.pop_front();
      }
      enc.room.notify_one();
      try {
        const std::vector<uint8_t> png = encode_png_rgb8(it.rgb.data(), it.h, it.w, kBatchPngLevel);
        FILE* f = fopen(out_paths[it.img], "wb");
        if (!f) throw Error(std::string(out_paths[it.img]) + ": " + strerror(errno), MX_E_IO);
        const bool ok = fwrite(png.data(), 1, png.size(), f) == png.size();
        if (fclose(f) != 0 || !ok) throw Error(std::string(out_paths[it.img]) + ": write failed", MX_E_IO);
        status[size_t(it.img)] = MX_OK;
      } catch (const Error& e) {
        status[size_t(it.img)] = e.code, why[size_t(it.img)] = e.what();
      } catch (const std::exception& e) {
        status[size_t(it.img)] = MX_E_IO, why[size_t(it.img)] = e.what();
      }
    }
  });
  struct InFlight {
    size_t j;  // index into list
    int k;     // slot
    int64_t h, w;
  };
  std::deque<InFlight> fl;
  int free_slots[2] = {1, 1};
  auto collect = [&]() -> bool {  // finish the oldest image in flight
    const InFlight f = fl.front();
    int r = guard([&] { MX_CUDA(cudaEventSynchronize(w->done[f.k])); });
    if (r == MX_OK) r = mx_gpu_poll(w->g);
    if (r != MX_OK) {
      *rc = r, *msg = last_message();
      return false;
    }
    PngItem it;
    it.img = list[f.j], it.h = f.h, it.w = f.w;
    it.rgb.assign(slots.out[f.k], slots.out[f.k] + size_t(f.h * f.w * 3));
    {
      // Hold the GPU back rather than queue without bound when the encoders
      // fall behind.
      std::unique_lock<std::mutex> l(enc.mu);
      enc.room.wait(l, [&] { return enc.q.size() < enc.limit; });
      enc.q.push_back(std::move(it));
    }
    enc.cv.notify_one();
    free_slots[f.k] = 1;
    fl.pop_front();
    return true;
  };
  bool failed = false;
  size_t j = 0;
  for (; j < list.size() && !failed; ++j) {
    const int32_t img = list[j];
    if (fl.size() == 2 && !collect()) {
      failed = true;
      break;
    }
    // Read and decode on this thread, while the GPU runs what is in flight.
    Rgb8 px;
    try {
      FILE* f = fopen(in_paths[img], "rb");
      if (!f) throw Error(std::string(in_paths[img]) + ": " + strerror(errno), MX_E_IO);
      std::vector<uint8_t> bytes;
      uint8_t buf[1 << 16];
      size_t got;
      while ((got = fread(buf, 1, sizeof(buf), f)) > 0) bytes.insert(bytes.end(), buf, buf + got);
      fclose(f);
      px = decode_png_rgb8(bytes.data(), bytes.size(), in_paths[img]);
      if (size_t(px.h * px.w * 3) > cap) throw Error(std::string(in_paths[img]) + ": larger than the batch's plan");
    } catch (const Error& e) {
      status[size_t(img)] = e.code, why[size_t(img)] = e.what();
      continue;
    } catch (const std::exception& e) {
      status[size_t(img)] = MX_E_IO, why[size_t(img)] = std::string(in_paths[img]) + ": " + e.what();
      continue;
    }
    int k = free_slots[0] ? 0 : 1;
    memcpy(slots.in[k], px.data.data(), px.data.size());
    int r = mx_gpu_upload_rgb8(w->g, slots.in[k], int32_t(px.h), int32_t(px.w), factor);
    if (r != MX_OK) {
      // The image's own problem (too small, pads to another shape): it fails
      // alone, nothing was enqueued for it.
      status[size_t(img)] = r, why[size_t(img)] = last_message();
      continue;
    }
    r = mx_gpu_enqueue(w->g);
    if (r == MX_OK) r = mx_gpu_download_rgb8(w->g, slots.out[k]);
    if (r == MX_OK) r = guard([&] { MX_CUDA(cudaEventRecord(w->done[k], stream)); });
    if (r != MX_OK) {
      *rc = r, *msg = last_message();
      failed = true;
      break;
    }
    free_slots[k] = 0;
    fl.push_back({j, k, px.h, px.w});
  }
  while (!failed && !fl.empty())
    if (!collect()) failed = true;
  // After a device failure the first image not dealt with is the oldest one
  // still in flight, or else the one this thread was on.
  const size_t dealt = !failed ? list.size() : !fl.empty() ? fl.front().j : j;
  enc.close_and_join();
  return dealt;
}

}  // namespace
}  // namespace mx

struct mx_batch {
  mx_batch_executor ex{};
  mx_batch_config cfg{};
  std::vector<mx_batch_worker> workers;
  std::vector<void*> handles;
};

using namespace mx;

namespace {

void set_worker_error(mx_batch_worker& w, int code, const std::string& msg) {
  w.state = MX_WORKER_FAILED;
  w.error_code = code;
  snprintf(w.error, sizeof(w.error), "%s", msg.c_str());
}

}  // namespace

extern "C" {

int mx_batch_new(const mx_batch_config* cfg, const int32_t* devices, int32_t n_devices,
                 const mx_batch_executor* executor, mx_batch** out) {
  std::unique_ptr<mx_batch> b;
  int rc = guard([&] {
    if (!cfg || !out || (n_devices > 0 && !devices)) throw Error("mx_batch_new: null argument");
    if (n_devices <= 0) throw Error("mx_batch_new: no devices");
    if (!executor && !cfg->plan) throw Error("mx_batch_new: the GPU executor needs a plan");
    if (cfg->device_mem_budget < 0) throw Error("mx_batch_new: negative memory budget");
    b = std::make_unique<mx_batch>();
    b->cfg = *cfg;
    if (executor) {
      if (!executor->open || !executor->run || !executor->close) throw Error("mx_batch_new: incomplete executor");
      b->ex = *executor;
    } else {
      b->ex.ctx = &b->cfg;
      b->ex.open = gpu_open;
      b->ex.run = gpu_run;
      b->ex.close = gpu_close;
    }
    b->workers.resize(size_t(n_devices));
    b->handles.assign(size_t(n_devices), nullptr);
    // Bring the executors up side by side: weight conversion and upload are
    // per device and take a while.
    std::vector<std::thread> th;
    for (int32_t i = 0; i < n_devices; ++i) {
      mx_batch_worker& w = b->workers[size_t(i)];
      memset(&w, 0, sizeof(w));
      w.device = devices[i];
      th.emplace_back([&b, i] {
        mx_batch_worker& w = b->workers[size_t(i)];
        int r = MX_E_INVALID;
        std::string msg;
        try {
          r = b->ex.open(b->ex.ctx, w.device, &b->handles[size_t(i)]);
          if (r != MX_OK) msg = b->ex.open == gpu_open ? last_message() : fmt("the executor returned %d", r);
        } catch (const std::exception& e) {
          r = MX_E_INVALID, msg = e.what();
        } catch (...) {
          r = MX_E_INVALID, msg = "unknown exception";
        }
        if (r != MX_OK) {
          b->handles[size_t(i)] = nullptr;
          set_worker_error(w, r, fmt("device %d: %s", w.device, msg.c_str()));
        } else {
          w.state = MX_WORKER_READY;
        }
      });
    }
    for (auto& t : th) t.join();
    int ready = 0;
    for (const auto& w : b->workers) ready += w.state == MX_WORKER_READY;
    if (ready == 0) {
      const mx_batch_worker& w0 = b->workers[0];
      throw Error(fmt("no device could take the batch; first: %s", w0.error), w0.error_code);
    }
    *out = b.release();
  });
  if (rc != MX_OK && b) mx_batch_free(b.release());
  return rc;
}

void mx_batch_free(mx_batch* b) {
  if (!b) return;
  for (size_t i = 0; i < b->handles.size(); ++i)
    if (b->handles[i]) b->ex.close(b->ex.ctx, b->handles[i]);
  delete b;
}

int mx_batch_run(mx_batch* b, int32_t n_images, const float* const* inputs, float* const* outputs,
                 int32_t* image_status) {
  return guard([&] {
    if (!b || n_images < 0 || (n_images > 0 && (!inputs || !outputs))) throw Error("mx_batch_run: bad argument");
    for (auto& w : b->workers) w.images_done = 0, w.seconds = 0.0;
    std::vector<int32_t> status(size_t(n_images), MX_E_INVALID);
    std::vector<std::string> why(size_t(n_images), "no device was left to restore it");
    std::vector<int32_t> todo(static_cast<size_t>(n_images));
    for (int32_t i = 0; i < n_images; ++i) todo[size_t(i)] = i;
    // Rounds: the pending images go round-robin to the workers still ready;
    // a worker that fails hands back what it had not finished.
    while (!todo.empty()) {
      std::vector<size_t> ready;
      for (size_t k = 0; k < b->workers.size(); ++k)
        if (b->workers[k].state == MX_WORKER_READY) ready.push_back(k);
      if (ready.empty()) break;
      std::vector<std::vector<int32_t>> share(ready.size());
      for (size_t j = 0; j < todo.size(); ++j) share[j % ready.size()].push_back(todo[j]);
      std::mutex mu;
      std::vector<int32_t> left;
      std::vector<std::thread> th;
      for (size_t r = 0; r < ready.size(); ++r) {
        th.emplace_back([&, r] {
          const size_t k = ready[r];
          mx_batch_worker& w = b->workers[k];
          void* h = b->handles[k];
          const auto t0 = std::chrono::steady_clock::now();
          size_t j = 0;
          if (b->ex.run == gpu_run) {
            // The built-in executor keeps two images in flight.
            int rc = MX_OK;
            std::string msg;
            j = gpu_run_list(static_cast<GpuWorker*>(h), share[r], inputs, outputs, &rc, &msg);
            for (size_t q = 0; q < j; ++q) status[size_t(share[r][q])] = MX_OK;
            w.images_done += int32_t(j);
            if (j < share[r].size()) {
              const int32_t img = share[r][j];
              status[size_t(img)] = rc;
              why[size_t(img)] = fmt("device %d: %s", w.device, msg.c_str());
              set_worker_error(w, rc, fmt("device %d failed on image %d: %s", w.device, img, msg.c_str()));
            }
          } else
          for (; j < share[r].size(); ++j) {
            const int32_t img = share[r][j];
            int rc = MX_E_INVALID;
            std::string msg;
            try {
              rc = b->ex.run(b->ex.ctx, h, inputs[img], outputs[img]);
              if (rc != MX_OK) msg = b->ex.run == gpu_run ? last_message() : fmt("the executor returned %d", rc);
            } catch (const std::exception& e) {
              rc = MX_E_INVALID, msg = e.what();
            } catch (...) {
              rc = MX_E_INVALID, msg = "unknown exception";
            }
            if (rc == MX_OK) {
              status[size_t(img)] = MX_OK;
              ++w.images_done;
              continue;
            }
            status[size_t(img)] = rc;
            why[size_t(img)] = fmt("device %d: %s", w.device, msg.c_str());
            set_worker_error(w, rc, fmt("device %d failed on image %d: %s", w.device, img, msg.c_str()));
            break;
          }
          w.seconds += std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
          if (j < share[r].size()) {
            std::lock_guard<std::mutex> l(mu);
            left.insert(left.end(), share[r].begin() + long(j), share[r].end());
          }
        });
      }
      for (auto& t : th) t.join();
      std::sort(left.begin(), left.end());
      todo.swap(left);
    }
    int failed = 0, first = -1;
    for (int32_t i = 0; i < n_images; ++i) {
      if (image_status) image_status[i] = status[size_t(i)];
      if (status[size_t(i)] != MX_OK) {
        ++failed;
        if (first < 0) first = i;
      }
    }
    if (failed)
      throw Error(fmt("%d of %d images were not restored; image %d: %s", failed, n_images, first,
                      why[size_t(first)].c_str()),
                  status[size_t(first)]);
  });
}

int mx_batch_run_png(mx_batch* b, int32_t n_images, const char* const* in_paths, const char* const* out_paths,
                     int32_t factor, int32_t* image_status) {
  return guard([&] {
    if (!b || n_images < 0 || (n_images > 0 && (!in_paths || !out_paths)) || factor <= 0)
      throw Error("mx_batch_run_png: bad argument");
    if (b->ex.run != gpu_run) throw Error("mx_batch_run_png: needs the built-in GPU executor");
    for (auto& w : b->workers) w.images_done = 0, w.seconds = 0.0;
    std::vector<int32_t> status(size_t(n_images), MX_E_INVALID);
    std::vector<std::string> why(size_t(n_images), "no device was left to restore it");
    std::vector<int32_t> todo(static_cast<size_t>(n_images));
    for (int32_t i = 0; i < n_images; ++i) todo[size_t(i)] = i;
    while (!todo.empty()) {
      std::vector<size_t> ready;
      for (size_t k = 0; k < b->workers.size(); ++k)
        if (b->workers[k].state == MX_WORKER_READY) ready.push_back(k);
      if (ready.empty()) break;
      std::vector<std::vector<int32_t>> share(ready.size());
      for (size_t j = 0; j < todo.size(); ++j) share[j % ready.size()].push_back(todo[j]);
      std::mutex mu;
      std::vector<int32_t> left;
      std::vector<std::thread> th;
      for (size_t r = 0; r < ready.size(); ++r) {
        th.emplace_back([&, r] {
          const size_t k = ready[r];
          mx_batch_worker& w = b->workers[k];
          const auto t0 = std::chrono::steady_clock::now();
          int rc = MX_OK;
          std::string msg;
          size_t j = 0;
          try {
            j = png_run_list(static_cast<GpuWorker*>(b->handles[k]), share[r], in_paths, out_paths, factor,
                             encoder_threads(ready.size()), status, why, &rc, &msg);
          } catch (const std::exception& e) {  // host resources (threads, memory): the worker stops here
            j = 0, rc = MX_E_INVALID, msg = e.what();
          }
          for (size_t q = 0; q < j; ++q) w.images_done += status[size_t(share[r][q])] == MX_OK;
          if (j < share[r].size()) {
            const int32_t img = share[r][j];
            status[size_t(img)] = rc;
            why[size_t(img)] = fmt("device %d: %s", w.device, msg.c_str());
            set_worker_error(w, rc, fmt("device %d failed on image %d: %s", w.device, img, msg.c_str()));
            std::lock_guard<std::mutex> l(mu);
            left.insert(left.end(), share[r].begin() + long(j), share[r].end());
          }
          w.seconds += std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        });
      }
      for (auto& t : th) t.join();
      std::sort(left.begin(), left.end());
      todo.swap(left);
    }
    int failed = 0, first = -1;
    for (int32_t i = 0; i < n_images; ++i) {
      if (image_status) image_status[i] = status[size_t(i)];
      if (status[size_t(i)] != MX_OK) {
        ++failed;
        if (first < 0) first = i;
      }
    }
    if (failed)
      throw Error(fmt("%d of %d images were not restored; image %d: %s", failed, n_images, first,
                      why[size_t(first)].c_str()),
                  status[size_t(first)]);
  });
}

int mx_batch_workers(const mx_batch* b, mx_batch_worker* out, int32_t n) {
  return guard([&] {
    if (!b || (n > 0 && !out)) throw Error("mx_batch_workers: null argument");
    if (size_t(n) != b->workers.size()) throw Error("mx_batch_workers: n must be the worker count");
    for (int32_t i = 0; i < n; ++i) out[i] = b->workers[size_t(i)];
  });
}

int32_t mx_batch_worker_count(const mx_batch* b) { return b ? int32_t(b->workers.size()) : 0; }

}  // extern "C"
