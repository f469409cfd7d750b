// The GPU executor: the B200 replacement for the reference's `exec_gpu::Gpu`
// (src/exec_gpu.rs:48-357) behind the C ABI in include/maxim_b200.h.
//
// What differs from the reference, by design:
//   * Activations live in ONE device arena, each storage-owning buffer laid
//     out NHWC - pixel-major, channels contiguous - instead of NCHW. A channel
//     view of a wider buffer becomes a strided view (same pixel stride as its
//     parent), so the model's splits and concatenations still cost nothing.
//     Host images stay NCHW; the boundary transposes on device.
//   * A pass runs the executor's own schedule of the plan (schedule.h): GEMM
//     epilogues absorb the elementwise op after them, copies are forwarded
//     into their producers, block permutations are dropped in favour of
//     gating through 5-D tensor maps, and the arena is re-packed by live
//     range for that shorter op list (still one allocation).
//   * Every weight is converted to its kernel's layout and uploaded once, at
//     construction (resident, not lazy per op).
//   * The whole scheduled stream - input transpose, every step, output
//     transpose - is captured once into a CUDA graph and replayed per image.
// The per-op walk (begin / step_op / read_buf / read_arena) keeps the plan's
// own op list and offsets: every op runs eagerly and unfused, and every
// buffer is where the plan put it.
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <climits>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <map>
#include <memory>
#include <mutex>
#include <set>
#include <string>
#include <utility>
#include <vector>

#include <cudaTypedefs.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <cstdio>

#include "common.h"
#include "gpu_common.cuh"
#include "kernels_simt.cuh"
#include "kernels_conv3.cuh"
#include "kernels_mem.cuh"
#include "kernels_umma.cuh"
#include "kernels_conv3f.cuh"
#include "kernels_image.cuh"
#include "image.h"
#include "maxim_b200.h"
#include "schedule.h"

namespace mx {

const char* describe_kind(int k);

namespace {

constexpr float kLnEps = 1e-6f;  // src/model.rs:35
constexpr int TPB = 256;

// Tap table of one resize axis, built exactly as the reference's `ResizeTaps`
// (src/exec_cpu.rs:1224-1282) so the device kernels apply the same weights.
struct HostTaps {
  std::vector<int> j0, w0, cnt;
  std::vector<float> w, wsum;
  std::vector<float> wrcp;  // 1 / wsum where wsum is an exact power of two, else 0
};
HostTaps make_taps(int n_in, int n_out, int max_taps) {
  HostTaps t;
  float inv = float(n_in) / float(n_out);
  float kscale = inv > 1.0f ? inv : 1.0f;
  for (int o = 0; o < n_out; ++o) {
    float sample = (float(o) + 0.5f) * inv - 0.5f;
    long a = long(std::ceil(sample - kscale));
    long b = long(std::floor(sample + kscale));
    if (a < 0) a = 0;
    if (b > n_in - 1) b = n_in - 1;
    int first = int(t.w.size());
    float s = 0.0f;
    for (long j = a; j <= b; ++j) {
      float d = std::fabs(sample - float(j)) / kscale;
      if (d < 1.0f) {
        float wv = 1.0f - d;
        t.w.push_back(wv);
        s += wv;
      }
    }
    t.j0.push_back(int(a));
    t.w0.push_back(first);
    t.wsum.push_back(s);
  }
  for (int o = 0; o < n_out; ++o) {
    int end = o + 1 < n_out ? t.w0[o + 1] : int(t.w.size());
    t.cnt.push_back(std::min(end - t.w0[o], max_taps));
    int e = 0;
    const float m = std::frexp(t.wsum[size_t(o)], &e);
    const float ws = t.wsum[size_t(o)];
    t.wrcp.push_back(std::isnormal(ws) && ws > 0.0f && m == 0.5f && e > -120 && e < 120 ? 1.0f / ws : 0.0f);
  }
  return t;
}

// One converted layout read back from a converted-weights cache file: the
// source blob's length and hash it was made from, and the layout itself.
struct WcEntry {
  uint64_t src_hash = 0;
  int64_t src_len = 0;
  const float* data = nullptr;  // into the file's bytes, held by the handle while it is built
  int64_t len = 0;              // floats
};

// A read-only mapping of a whole file (the converted-weights cache), pages
// populated up front.
struct FileMap {
  const char* p = nullptr;
  size_t n = 0;
  FileMap() = default;
  FileMap(const FileMap&) = delete;
  FileMap& operator=(const FileMap&) = delete;
  ~FileMap() { reset(); }
  void reset() {
    if (p) munmap(const_cast<char*>(p), n);
    p = nullptr;
    n = 0;
  }
};

// A bump allocator over one device allocation: weights and tables, each
// 256-byte aligned. The host image grows by realloc (which moves large
// blocks by remapping pages, not copying) and is never zero-filled beyond
// the alignment gaps: a std::vector's resize cleared and re-copied the whole
// image at every doubling, most of an executor's construction time.
struct DevicePool {
  char* host = nullptr;
  size_t len = 0, cap = 0;
  char* dev = nullptr;
  DevicePool() = default;
  DevicePool(const DevicePool&) = delete;
  DevicePool& operator=(const DevicePool&) = delete;
  ~DevicePool() { free(host); }
  size_t size() const { return len; }
  size_t put(const void* data, size_t bytes) {
    const size_t off = (len + 255) & ~size_t(255), need = off + bytes;
    if (need > cap) {
      size_t nc = cap ? cap : (size_t(1) << 20);
      while (nc < need) nc *= 2;
      char* q = static_cast<char*>(realloc(host, nc));
      if (!q) throw std::bad_alloc();
      host = q, cap = nc;
    }
    if (off > len) memset(host + len, 0, off - len);
    if (bytes) memcpy(host + off, data, bytes);
    len = need;
    return off;
  }
  template <class T>
  size_t put(const std::vector<T>& v) {
    return put(v.data(), v.size() * sizeof(T));
  }
  void drop_host() {
    free(host);
    host = nullptr;
    cap = 0;
  }
};

struct Step {
  int op;       // plan op index, -1 for the boundary transposes
  int kernels;  // launches it makes
  std::function<void(cudaStream_t)> run;
  // Runs once after the arena and the weight pool exist (tensor maps need
  // final device addresses).
  std::function<void()> prepare;
};

// w rounded to the nearest TF32 value (ties to even), as fp32 with the low
// 13 mantissa bits clear; values whose rounding would overflow stay as they are.
float round_tf32(float w) {
  uint32_t b;
  memcpy(&b, &w, 4);
  uint32_t r = (b + 0xFFFu + ((b >> 13) & 1u)) & 0xFFFFE000u;
  float h;
  memcpy(&h, &r, 4);
  return std::isfinite(h) ? h : w;
}

// Weights split for the 3-pass TF32 products: hi = w rounded to TF32, lo =
// the remainder w - hi (exact in fp32) rounded to TF32 in turn, so the tensor
// core reads both exactly.
void split_tf32(const std::vector<float>& w, std::vector<float>& hi, std::vector<float>& lo) {
  hi.resize(w.size());
  lo.resize(w.size());
  for (size_t i = 0; i < w.size(); ++i) {
    const float h = round_tf32(w[i]);
    hi[i] = h;
    lo[i] = round_tf32(w[i] - h);
  }
}

// The driver's tensor-map encoder, looked up once per process (batch
// workers build executors on several threads at once).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static std::mutex mu;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::lock_guard<std::mutex> l(mu);
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    MX_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
    if (q != cudaDriverEntryPointSuccess || !p) throw Error("cuTensorMapEncodeTiled is unavailable", MX_E_CUDA);
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// A tiled fp32 tensor map with 128-byte swizzle (the UMMA canonical layout).
// dims / box innermost first; strides in bytes for dims 1..rank-1. Every box
// row is 128 bytes (32 channels), and many views are channel ranges of wider
// buffers, so L2 fetches are promoted to 128 bytes only: a 256-byte promotion
// would also pull in the neighbouring channels of a strided view, doubling
// the DRAM reads of a 32-channel half of a 64-channel buffer.
CUtensorMap make_tensor_map(const void* base, int rank, const uint64_t* dims, const uint64_t* strides,
                            const uint32_t* box, CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B,
                            const uint32_t* elem_strides = nullptr) {
  CUtensorMap m;
  uint32_t es[5] = {1, 1, 1, 1, 1};
  if (elem_strides)
    for (int i = 0; i < rank; ++i) es[i] = elem_strides[i];
  CUresult r = tensor_map_encoder()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, cuuint32_t(rank), const_cast<void*>(base),
                                    dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                                    CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw Error(fmt("cuTensorMapEncodeTiled failed (%d)", int(r)), MX_E_CUDA);
  return m;
}

// The tensor maps and the launch parameters of one tensor-core conv: A, B
// (hi, lo) and the output D.
struct UmmaOp {
  CUtensorMap a, b, blo, d, l;  // l: the LayerNorm output of a CONV1 epilogue (else a copy of d)
  UmmaConvParams p{};
  int n = 0, taps = 1, mode = 0, grid = 0, smem = 0;
};

}  // namespace
}  // namespace mx

struct mx_gpu {
  int device = 0;
  cudaStream_t stream = nullptr;
  std::vector<mx_buf> bufs;
  std::vector<int64_t> offs;
  std::vector<int32_t> alias_parent;
  std::vector<mx_op> ops;
  int32_t input = -1, output = -1;
  int64_t arena_len = 0;
  mx_buf shape{};
  float* arena = nullptr;
  float* io_in = nullptr;   // NCHW staging of the input image
  float* io_out = nullptr;  // NCHW staging of the output image
  mx::DevicePool pool;
  int64_t weight_bytes = 0;
  std::vector<mx::Step> steps;  // op-by-op walk at the plan's offsets: [in-transpose, ops..., out-transpose]
  std::vector<int> step_of_op;  // op index -> step index
  std::vector<int64_t> roffs;   // each buffer's offset relative to its root (alignment checks)
  std::vector<int64_t> foffs;   // the scheduled pass's offsets
  std::vector<int32_t> merged_into;  // per plan root: the root it is placed inside in the pass (-1: none)
  std::vector<mx::Step> fsteps; // the scheduled pass: [in-transpose, steps..., out-transpose]
  std::vector<int32_t> primary_of;  // plan op -> the op whose step carries it out (-1: dropped)
  std::vector<int32_t> sched_flags; // plan op -> MX_SCHED_* flags
  int64_t farena_len = 0;
  int perms_dropped = 0, ops_fused = 0;
  std::map<std::pair<int32_t, int>, int64_t> wcache;  // (weight id, layout tag) -> pool offset
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t graph_exec = nullptr;
  bool timeline_on = false;
  std::vector<float> timeline_ms;
  std::vector<int32_t> timeline_kernels;
  float timeline_total = 0.0f;
  // What the arena holds: nothing yet, the scheduled pass's state (at foffs),
  // or the op-by-op walk's (at the plan's offsets).
  enum { HOLDS_NOTHING, HOLDS_PASS, HOLDS_WALK } holds = HOLDS_NOTHING;
  std::vector<int32_t> write_order;  // storage roots by their last write in the plan (input first)
  float* readback = nullptr;         // device staging for plan-layout read-back (largest root)
  int64_t readback_len = 0;
  int64_t kernels = 0;
  int64_t umma_ops = 0;
  std::string name;
  int* status = nullptr;  // device status word the tensor-core kernels write
  int sms = 148;
  bool use_umma = true;
  float* scratch = nullptr;  // per-op scratch (the channel-mean partial sums)
  int64_t scratch_len = 0;   // floats
  // The device-side image pipeline (mx_gpu_upload_rgb8 / download_rgb8):
  // 8-bit staging, allocated at its first use, and the geometry of the image
  // last uploaded through it.
  uint8_t* rgb_in = nullptr;
  uint8_t* rgb_out = nullptr;
  int32_t rgb_h = 0, rgb_w = 0, rgb_even_h = 0, rgb_even_w = 0;
  // The converted-weights cache (mx_gpu_new_cached, mx_gpu_save_weight_cache).
  const mx_plan* building = nullptr;  // the caller's plan, while the steps are made
  bool wc_track = false;              // hash source weights (a cache file is in use)
  mx::FileMap wc_file;                // the cache file, mapped while the steps are made
  std::map<std::pair<int32_t, int>, mx::WcEntry> wc_loaded;  // layouts read from the file, not yet used
  std::map<int32_t, uint64_t> wc_hash;                       // weight id -> hash of its plan blob
  std::map<int32_t, int64_t> wsrc_len;                       // weight id -> its plan blob's length
  std::map<std::pair<int32_t, int>, int64_t> wbytes;        // (weight id, layout) -> bytes in the pool
  int64_t wc_hits = 0, wc_converted = 0;
  int wc_saved = 0;
  double t_cache_read = 0, t_steps = 0, t_device = 0, t_cache_write = 0;  // construction phases, seconds
};

namespace mx {
namespace {

struct DevicePin {
  explicit DevicePin(int dev) { MX_CUDA(cudaSetDevice(dev)); }
};

int32_t root_of(const mx_gpu& g, int32_t id) {
  while (g.alias_parent[size_t(id)] >= 0) id = g.alias_parent[size_t(id)];
  return id;
}

// A buffer's NHWC view in a given layout (per-buffer float offsets: the
// plan's, or the scheduled pass's).
using Layout = std::vector<int64_t>;

// The root whose pixel stride a buffer's view has in layout L: its plan
// root, or in the scheduled pass the root that root is placed inside.
int32_t base_of(const mx_gpu& g, const Layout& L, int32_t id) {
  int32_t base = root_of(g, id);
  if (&L == &g.foffs && size_t(base) < g.merged_into.size() && g.merged_into[size_t(base)] >= 0)
    base = g.merged_into[size_t(base)];
  return base;
}

View view_of(const mx_gpu& g, const Layout& L, int32_t id) {
  int32_t base = base_of(g, L, id);
  const mx_buf& b = g.bufs[size_t(id)];
  int64_t hw = b.h * b.w;
  int64_t ch0 = hw ? (L[size_t(id)] - L[size_t(base)]) / hw : 0;
  View v;
  v.ptr = g.arena + L[size_t(base)] + ch0;
  v.stride = g.bufs[size_t(base)].c;
  v.c = b.c;
  v.npix = hw;
  return v;
}

bool aligned4(const View& v) {
  return (reinterpret_cast<uintptr_t>(v.ptr) % 16 == 0) && v.stride % 4 == 0 && v.c % 4 == 0;
}

template <int KIND>
void launch_ew(cudaStream_t s, View d, View a, View b, float slope) {
  int64_t npix = d.npix;
  if (aligned4(d) && aligned4(a) && (b.ptr == nullptr || aligned4(b))) {
    int c4 = int(d.c / 4);
    ew_kernel4<KIND><<<blocks_for(npix * c4, TPB), TPB, 0, s>>>(npix, c4, a.ptr, a.stride, b.ptr, b.stride, d.ptr,
                                                                  d.stride, slope);
  } else {
    ew_kernel1<KIND><<<blocks_for(npix * d.c, TPB), TPB, 0, s>>>(npix, int(d.c), a.ptr, a.stride, b.ptr, b.stride,
                                                                   d.ptr, d.stride, slope);
  }
}

template <int BM, int BN, class P>
void launch_gemm(cudaStream_t s, const P& p, int batch) {
  dim3 grid(unsigned((p.M + BM - 1) / BM), unsigned((p.N + BN - 1) / BN), unsigned(batch));
  simt_gemm_kernel<BM, BN, 4, 4, P><<<grid, (BM / 4) * (BN / 4), 0, s>>>(p);
}

void check_launch() {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw Error(std::string("kernel launch: ") + cudaGetErrorString(e), MX_E_CUDA);
}

// Element offset (into the arena), pixel stride and channel count of a
// buffer's NHWC view, known before any device memory exists.
struct ViewMeta {
  int64_t off, stride, c, npix;
};
ViewMeta meta_of(const mx_gpu& g, const Layout& L, int32_t id) {
  int32_t base = base_of(g, L, id);
  const mx_buf& b = g.bufs[size_t(id)];
  int64_t hw = b.h * b.w;
  int64_t ch0 = hw ? (L[size_t(id)] - L[size_t(base)]) / hw : 0;
  return {L[size_t(base)] + ch0, g.bufs[size_t(base)].c, b.c, hw};
}

// Whether a buffer can be read or written by TMA as n channels: 16-byte
// aligned start and pixel stride.
bool tma_view(const mx_gpu& g, const Layout& L, int32_t id, int n) {
  if (id < 0) return false;
  ViewMeta m = meta_of(g, L, id);
  return m.c == n && m.off % 4 == 0 && m.stride % 4 == 0;
}

// Whether a conv runs on the tensor-core kernel: TMA needs 16-byte aligned
// rows and strides; the kernel takes K in blocks of 32 channels and
// N = c_out in {32, 64, 128, 256}.
// A 1x1 conv over fewer pixels than one tensor-core tile (the channel
// attention's convs on the 1x1 squeeze) runs on the small-conv kernel: the
// persistent tensor-core kernel would launch 148 CTAs for one tile.
constexpr int64_t kSmallConvPixels = 128;
bool small_conv(const mx_op& o) { return o.kind == MX_OP_CONV1X1 && int64_t(o.h) * o.wd < kSmallConvPixels; }

bool umma_eligible(const mx_gpu& g, const Layout& L, const mx_op& o) {
  if (!g.use_umma) return false;
  if (o.kind != MX_OP_CONV1X1 && o.kind != MX_OP_CONV3X3 && o.kind != MX_OP_CONV4X4S2) return false;
  if (small_conv(o)) return false;
  if (o.c_in % 32 != 0) return false;
  if (o.c_out != 32 && o.c_out != 64 && o.c_out != 128 && o.c_out != 256) return false;
  ViewMeta x = meta_of(g, L, o.src), d = meta_of(g, L, o.dst);
  if (x.off % 4 || x.stride % 4 || d.off % 4 || d.stride % 4) return false;
  if (x.c != o.c_in || d.c != o.c_out || x.npix != int64_t(o.h) * o.wd) return false;
  return true;
}

// Whether a 2x2 transposed conv runs on the tensor-core kernel: the GEMM's
// N = 4 c_out comes in 128-column slices, and each epilogue warp's 32 input
// pixels must be one row segment (width a multiple of 32).
bool umma_convt_eligible(const mx_gpu& g, const Layout& L, const mx_op& o) {
  if (!g.use_umma || o.kind != MX_OP_CONVT2X2) return false;
  if (o.c_in % 32 != 0 || (o.c_out != 32 && o.c_out != 64 && o.c_out != 128)) return false;
  if (o.wd % 32 != 0) return false;
  ViewMeta x = meta_of(g, L, o.src), d = meta_of(g, L, o.dst);
  if (x.off % 4 || x.stride % 4 || d.off % 4 || d.stride % 4) return false;
  if (x.c != o.c_in || d.c != o.c_out || x.npix != int64_t(o.h) * o.wd || d.npix != 4 * x.npix) return false;
  return true;
}

// Whether a gating matmul runs on the tensor-core kernel.
bool umma_gate_eligible(const mx_gpu& g, const Layout& L, const mx_op& o) {
  if (!g.use_umma || o.kind != MX_OP_GATE_MM) return false;
  const int n = o.mode == 0 ? o.outer : o.inner;
  if (n != 32 && n != 64 && n != 128 && n != 256) return false;
  if (o.c % 32 != 0) return false;
  ViewMeta x = meta_of(g, L, o.src), d = meta_of(g, L, o.dst);
  if (x.off % 4 || x.stride % 4 || d.off % 4 || d.stride % 4) return false;
  if (x.c != o.c || d.c != o.c || x.npix != int64_t(o.outer) * o.inner) return false;
  return true;
}

// Whether a gating matmul can read spatial-order data blocked as `perm`
// describes (MODE_GATE_SP): one box per group must cover 32 consecutive
// contracted indices as whole rows, so the row length (cells per grid row
// for grid gating, pixels per block row for block gating) must divide 32.
bool umma_gate_spatial_ok(const mx_gpu& g, const Layout& L, const mx_op& gate, const mx_op& perm) {
  if (!umma_gate_eligible(g, L, gate)) return false;
  const int row = gate.mode == 0 ? perm.gw : perm.fw;
  if (row <= 0 || row > 32 || 32 % row != 0) return false;
  return tma_view(g, L, perm.src, gate.c) && perm.c == gate.c;
}

// Kernel instances: N (columns per tile; 256 output columns run as two
// 128-column slices) x MODE.
#define MX_UMMA_INSTANCES(X)                                                                        \
  X(32, 0) X(64, 0) X(128, 0) X(32, 1) X(64, 1) X(128, 1) X(32, 2) X(64, 2) X(128, 2) X(32, 3) X(64, 3) \
  X(128, 3) X(32, 4) X(64, 4) X(128, 4) X(32, 5) X(64, 5) X(128, 5) X(128, 6) X(32, 7) X(64, 7)

// The tensor-core kernels' shared-memory opt-in. A function attribute is
// per device, so it is set once for each device an executor is built on
// (the current one), under a lock: batch workers build executors for
// several devices on several threads at once.
void umma_attrs_once() {
  static std::mutex mu;
  static std::set<int> done;
  int dev = -1;
  MX_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> l(mu);
  if (done.count(dev)) return;
#define MX_UMMA_ATTR(NN, MM)                                                                              \
  MX_CUDA(cudaFuncSetAttribute(umma_conv_kernel<NN, MM, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                               UmmaCfg<NN, MM>::SMEM_BYTES));                                                \
  MX_CUDA(cudaFuncSetAttribute(umma_conv_kernel<NN, MM, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,  \
                               UmmaCfg<NN, MM>::SMEM_BYTES));
  MX_UMMA_INSTANCES(MX_UMMA_ATTR)
#undef MX_UMMA_ATTR
  MX_CUDA(cudaFuncSetAttribute(umma_conv3f_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               Conv3fCfg::SMEM_BYTES));
  done.insert(dev);
}
int umma_smem(int n, int mode) {
#define MX_UMMA_SMEM(NN, MM) \
  if (n == NN && mode == MM) return UmmaCfg<NN, MM>::SMEM_BYTES;
  MX_UMMA_INSTANCES(MX_UMMA_SMEM)
#undef MX_UMMA_SMEM
  throw Error(fmt("no tensor-core kernel for N=%d mode=%d", n, mode));
}

// Columns per tile for an output of n columns (32..256), and the slices.
int umma_tile_n(int n) { return n > 128 ? 128 : n; }
void launch_umma(cudaStream_t s, const UmmaOp& u) {
#define MX_UMMA_CASE(NN, MM)                                                                              \
  if (u.n == NN && u.mode == MM) {                                                                        \
    if (u.p.epi >= UEPI_ADD)                                                                              \
      umma_conv_kernel<NN, MM, true>                                                                      \
          <<<unsigned(u.grid), UmmaCfg<NN, MM>::THREADS, u.smem, s>>>(u.a, u.b, u.blo, u.d, u.l, u.p);    \
    else                                                                                                  \
      umma_conv_kernel<NN, MM, false>                                                                     \
          <<<unsigned(u.grid), UmmaCfg<NN, MM>::THREADS, u.smem, s>>>(u.a, u.b, u.blo, u.d, u.l, u.p);    \
    return;                                                                                               \
  }
  MX_UMMA_INSTANCES(MX_UMMA_CASE)
#undef MX_UMMA_CASE
  throw Error(fmt("no tensor-core kernel for N=%d mode=%d", u.n, u.mode));
}

// Weights in a kernel's layout, uploaded once per (weight, layout) however
// many steps use them; -1 for an absent weight.
enum WeightTag : int {
  WT_RAW = 0,
  WT_KTAP = 1,
  WT_HI = 2,
  WT_LO = 3,
  WT_KTAP_HI = 4,
  WT_KTAP_LO = 5,
  WT_CONVT = 6,
  WT_CONVT_HI = 7,
  WT_CONVT_LO = 8,
  WT_BIAS4 = 9,  // a bias repeated once per transposed-conv tap
  WT_T = 10,     // a 1x1 kernel transposed to [c_in][c_out] (the small-conv kernel)
  WT_CONV3F = 11,  // a 32-to-32 3x3 kernel for umma_conv3f_kernel: [ky][hi, lo][kx][c_out][c_in]
};
// 64-bit hash of a weight blob's bytes (multiply-rotate over 8-byte words,
// then a final avalanche): what ties a cached layout to the weights it was
// made from.
uint64_t blob_hash(const float* p, int64_t n) {
  const uint64_t k1 = 0x9E3779B97F4A7C15ull, k2 = 0xC2B2AE3D27D4EB4Full;
  auto mix = [&](uint64_t h, uint64_t x) {
    h ^= x * k2;
    return ((h << 31) | (h >> 33)) * k1;
  };
  const unsigned char* b = reinterpret_cast<const unsigned char*>(p);
  const size_t bytes = size_t(n) * 4;
  // Four independent lanes over 32-byte blocks, so the multiplies overlap.
  uint64_t h[4] = {uint64_t(n) * k1, k2, k1 ^ k2, uint64_t(n) ^ k2};
  size_t i = 0;
  for (; i + 32 <= bytes; i += 32) {
    uint64_t x[4];
    memcpy(x, b + i, 32);
    for (int l = 0; l < 4; ++l) h[l] = mix(h[l], x[l]);
  }
  uint64_t r = mix(mix(mix(h[0], h[1]), h[2]), h[3]);
  for (; i < bytes; i += 8) {
    uint64_t x = 0;
    memcpy(&x, b + i, std::min<size_t>(8, bytes - i));
    r = mix(r, x);
  }
  r ^= r >> 33;
  r *= k2;
  r ^= r >> 29;
  return r;
}

uint64_t src_hash(mx_gpu& g, int32_t id) {
  auto it = g.wc_hash.find(id);
  if (it != g.wc_hash.end()) return it->second;
  if (!g.building) throw Error("weight cache: no plan to hash");
  const uint64_t h = blob_hash(g.building->weights[id], g.building->weight_lens[id]);
  g.wc_hash[id] = h;
  g.wsrc_len[id] = g.building->weight_lens[id];
  return h;
}

// Whether the cache file held this layout, made from the weight blob the plan
// holds now (same length and hash).
bool cache_has(mx_gpu& g, const std::pair<int32_t, int>& key) {
  if (g.wc_loaded.empty()) return false;
  auto it = g.wc_loaded.find(key);
  return it != g.wc_loaded.end() && it->second.src_len == g.building->weight_lens[key.first] &&
         it->second.src_hash == src_hash(g, key.first);
}

WcEntry cache_take(mx_gpu& g, const std::pair<int32_t, int>& key) {
  auto it = g.wc_loaded.find(key);
  const WcEntry e = it->second;
  g.wc_loaded.erase(it);
  ++g.wc_hits;
  return e;
}

int64_t cached(mx_gpu& g, int32_t id, int tag, const std::function<std::vector<float>()>& make) {
  if (id < 0) return -1;
  const auto key = std::make_pair(id, tag);
  auto it = g.wcache.find(key);
  if (it != g.wcache.end()) return it->second;
  std::vector<float> v;
  const float* data = nullptr;
  int64_t len = 0;
  if (tag == WT_RAW && g.building) {
    data = g.building->weights[id], len = g.building->weight_lens[id];  // as the plan holds it
  } else if (tag != WT_RAW && cache_has(g, key)) {
    const WcEntry e = cache_take(g, key);
    data = e.data, len = e.len;
  } else {
    v = make();
    data = v.data(), len = int64_t(v.size());
    if (tag != WT_RAW) {
      ++g.wc_converted;
      if (g.wc_track) src_hash(g, id);  // known for a later save
    }
  }
  int64_t off = -1;
  if (len > 0) {
    off = int64_t(g.pool.put(data, size_t(len) * 4));
    g.weight_bytes += len * 4;
    if (tag != WT_RAW) g.wbytes[key] = len * 4;
  }
  g.wcache[key] = off;
  return off;
}

// What a scheduled step adds to its tensor-core op: the elementwise tail and,
// for a gating matmul over spatial-order data, the blocking it reads through.
struct UmmaEpi {
  int epi = EPI_NONE;
  int32_t src = -1;
  int32_t src2 = -1;  // a channel scale's second residual
  float slope = 0.0f;
  bool spatial = false;
  mx_op perm{};
  int32_t ln_stats = -1;                 // LayerNorm on load: statistics buffer
  int64_t ln_scale = -1, ln_bias = -1;  // and the pool offsets of its weights
  int32_t lo_dst = -1, lo_c0 = 0;       // LayerNorm of output columns [lo_c0, +32) written to lo_dst
  bool lo_only = false;                 // ...and those columns themselves not stored
  int64_t lo_scale = -1, lo_bias = -1;
  int32_t st_out[2] = {-1, -1};          // LayerNorm statistics the epilogue writes
  int32_t st_c0[2] = {0, 0};
  int32_t st_c = 0;
};

// The tensor-core step of a gating matmul. Over a blocked buffer (pixels in
// block order g * pp + q, NHWC): block gating (mode 1) contracts q inside a
// block, grid gating (mode 0) contracts the cell g. Over a spatial buffer
// (E.spatial) the same contraction reads the blocks in place through 5-D
// tensor maps. A is the activation (MN-major), B = W[a][t] (K-major), D and
// the epilogue operand are activation-shaped.
Step umma_gate_step(mx_gpu& g, int32_t oi, const mx_op& o, const Layout* L, int64_t ho, int64_t lo_off, int64_t bo,
                    const UmmaEpi& E) {
  auto u = std::make_shared<UmmaOp>();
  mx_gpu* G = &g;
  const mx_op op = o;
  ++g.umma_ops;
  Step st{oi, 1, nullptr, nullptr};
  st.prepare = [G, L, u, op, ho, lo_off, bo, E]() {
    View x = view_of(*G, *L, op.src), d = view_of(*G, *L, op.dst);
    View e = E.epi >= EPI_ADD ? view_of(*G, *L, E.src) : d;
    const uint64_t gg = uint64_t(op.outer), pp = uint64_t(op.inner), c = uint64_t(op.c);
    const int n = op.mode == 0 ? op.outer : op.inner;  // the contracted (and produced) axis
    const int tn = umma_tile_n(n);
    const float* whi = reinterpret_cast<const float*>(G->pool.dev + ho);
    const float* wlo = reinterpret_cast<const float*>(G->pool.dev + lo_off);
    {
      uint64_t dims[2] = {uint64_t(n), uint64_t(n)}, str[1] = {uint64_t(n) * 4};
      uint32_t box[2] = {32, uint32_t(tn)};
      u->b = make_tensor_map(whi, 2, dims, str, box);
      u->blo = make_tensor_map(wlo, 2, dims, str, box);
    }
    u->p.eptr = E.epi >= EPI_ADD ? e.ptr : nullptr;
    u->p.estride = int(e.stride);
    u->p.e_pp = int(pp);
    u->p.sp_shift = 0;
    if (E.spatial) {
      // dims (channel, fx, gx, fy, gy), strides ascending; pixel
      // (gy * fh + fy, gx * fw + fx).
      const mx_op& P = E.perm;
      const uint64_t fw = uint64_t(P.fw), gw = uint64_t(P.gw), fh = uint64_t(P.fh), gh = uint64_t(P.gh);
      uint64_t dims[5] = {c, fw, gw, fh, gh};
      auto strides = [&](const View& v, uint64_t* sv) {
        const uint64_t px = uint64_t(v.stride) * 4;
        sv[0] = px, sv[1] = fw * px, sv[2] = fw * gw * px, sv[3] = fh * fw * gw * px;
      };
      uint64_t sa[4], sd[4], se[4];
      strides(x, sa), strides(d, sd), strides(e, se);
      uint32_t box[5];
      if (op.mode == 0) {  // grid gating: t = cell, a group = a position in the cell
        box[0] = 32, box[1] = 1, box[2] = uint32_t(gw), box[3] = 1, box[4] = uint32_t(32 / gw);
        u->p.groups = int(pp);
      } else {  // block gating: t = position in the block, a group = a block
        box[0] = 32, box[1] = uint32_t(fw), box[2] = 1, box[3] = uint32_t(32 / fw), box[4] = 1;
        u->p.groups = int(gg);
      }
      u->a = make_tensor_map(x.ptr, 5, dims, sa, box, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
      u->d = make_tensor_map(d.ptr, 5, dims, sd, box);
      // The gate operand, read by the epilogue in the output's boxes.
      u->l = E.epi >= EPI_ADD ? make_tensor_map(e.ptr, 5, dims, se, box) : u->d;
      u->mode = MODE_GATE_SP;
      u->p.sp_mode = op.mode == 0 ? 0 : 1;
      u->p.fw = P.fw;
      u->p.gw = P.gw;
      u->p.fh = P.fh;
      u->p.e_w = P.gw * P.fw;
      const int rowlen = op.mode == 0 ? P.gw : P.fw;
      while ((1 << u->p.sp_shift) < rowlen) ++u->p.sp_shift;
    } else {
      // dims (channel, q, g), strides ascending: q steps one pixel, g one block.
      uint64_t dims[3] = {c, pp, gg};
      uint64_t sa[2] = {uint64_t(x.stride) * 4, pp * uint64_t(x.stride) * 4};
      uint64_t sd[2] = {uint64_t(d.stride) * 4, pp * uint64_t(d.stride) * 4};
      uint32_t box[3];
      if (op.mode == 1) {  // block gating: box (32 channels, 32 q, 4 blocks)
        box[0] = 32, box[1] = 32, box[2] = 4;
        u->mode = MODE_GATE;
        u->p.groups = int(gg);
      } else {  // grid gating: per-position box (32 channels, 1 q, 32 cells)
        box[0] = 32, box[1] = 1, box[2] = 32;
        u->mode = MODE_GATE_GRID;
        u->p.groups = int(pp);
      }
      // The activation is the MN-major operand: 32-byte-atom swizzle (see
      // desc_mnmajor_sw128_32b). The output staging is plain 128-byte swizzle.
      u->a = make_tensor_map(x.ptr, 3, dims, sa, box, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
      // The output goes out per epilogue warp, one group at a time.
      uint32_t bd[3] = {box[0], box[1], 1};
      if (op.mode == 0) bd[1] = 1, bd[2] = 32;
      u->d = make_tensor_map(d.ptr, 3, dims, sd, bd);
      const uint64_t se[2] = {uint64_t(e.stride) * 4, pp * uint64_t(e.stride) * 4};
      u->l = E.epi >= EPI_ADD ? make_tensor_map(e.ptr, 3, dims, se, bd) : u->d;
    }
    u->p.n_slices = n / tn;
    u->p.tiles_x = (u->p.groups + 3) / 4;
    u->p.tiles = u->p.tiles_x * int(c / 32) * u->p.n_slices;
    u->p.kb_per_tap = n / 32;
    u->p.c_in = n;
    u->p.epi = E.epi;
    u->p.slope = E.slope;
    u->p.bias = bo < 0 ? nullptr : reinterpret_cast<const float*>(G->pool.dev + bo);
    u->p.status = G->status;
    u->n = tn;
    u->taps = 1;
    u->grid = std::min(u->p.tiles, G->sms);
    u->smem = umma_smem(tn, u->mode);
  };
  st.run = [u](cudaStream_t s) { launch_umma(s, *u); };
  return st;
}

// The tensor-core step of a 1x1, 3x3 or 4x4 stride-2 conv over weights split
// into TF32 hi/lo in [c_out][tap][c_in] order; the tensor maps are built once
// the arena and the pool have their final addresses.
Step umma_conv_step(mx_gpu& g, int32_t oi, const mx_op& o, const Layout* L, int64_t ho, int64_t lo_off, int64_t bo,
                    const UmmaEpi& E) {
  const int taps = o.kind == MX_OP_CONV3X3 ? 9 : (o.kind == MX_OP_CONV4X4S2 ? 16 : 1);
  auto u = std::make_shared<UmmaOp>();
  mx_gpu* G = &g;
  const mx_op op = o;
  ++g.umma_ops;
  Step st{oi, 1, nullptr, nullptr};
  st.prepare = [G, L, u, op, taps, ho, lo_off, bo, E]() {
    View x = view_of(*G, *L, op.src), d = view_of(*G, *L, op.dst);
    View e = E.epi >= EPI_ADD ? view_of(*G, *L, E.src) : d;
    const int n = op.c_out, ci = op.c_in, H = op.h, W = op.wd;
    const int tn = umma_tile_n(n);
    const uint64_t K = uint64_t(taps) * ci;
    const float* whi = reinterpret_cast<const float*>(G->pool.dev + ho);
    const float* wlo = reinterpret_cast<const float*>(G->pool.dev + lo_off);
    {
      uint64_t dims[2] = {K, uint64_t(n)}, str[1] = {K * 4};
      uint32_t box[2] = {32, uint32_t(tn)};
      u->b = make_tensor_map(whi, 2, dims, str, box);
      u->blo = make_tensor_map(wlo, 2, dims, str, box);
    }
    u->p.eptr = E.epi >= EPI_ADD ? e.ptr : nullptr;
    u->p.estride = int(e.stride);
    for (int g2 = 0; g2 < 2; ++g2)
      if (E.st_out[g2] >= 0) {
        u->p.st_out[g2] = reinterpret_cast<float2*>(view_of(*G, *L, E.st_out[g2]).ptr);
        u->p.st_c0[g2] = E.st_c0[g2];
      }
    u->p.st_c = E.st_c;
    u->p.st_eps = kLnEps;
    if (E.ln_stats >= 0) {
      u->p.ln_stats = reinterpret_cast<const float2*>(view_of(*G, *L, E.ln_stats).ptr);
      u->p.ln_scale = reinterpret_cast<const float*>(G->pool.dev + E.ln_scale);
      u->p.ln_bias = reinterpret_cast<const float*>(G->pool.dev + E.ln_bias);
      u->p.in_w = taps == 1 ? int(x.npix) : W;
      u->p.in_h = H;
    }
    if (taps == 1) {
      uint64_t da[2] = {uint64_t(ci), uint64_t(x.npix)}, sa[1] = {uint64_t(x.stride) * 4};
      uint32_t ba[2] = {32, 128};
      u->a = make_tensor_map(x.ptr, 2, da, sa, ba);
      // The output goes out per epilogue warp: 32 pixels x 32 channels.
      uint64_t dd[2] = {uint64_t(n), uint64_t(d.npix)}, sd[1] = {uint64_t(d.stride) * 4};
      uint32_t bd[2] = {32, 32};
      u->d = make_tensor_map(d.ptr, 2, dd, sd, bd);
      u->l = u->d;
      if (E.lo_dst >= 0) {
        // The LayerNorm of 32 output channels goes to its own buffer, in
        // the same 32-pixel boxes.
        View y = view_of(*G, *L, E.lo_dst);
        uint64_t dy[2] = {32, uint64_t(y.npix)}, sy[1] = {uint64_t(y.stride) * 4};
        u->l = make_tensor_map(y.ptr, 2, dy, sy, bd);
        u->p.lo_col = E.lo_c0;
        u->p.lo_only = E.lo_only ? 1 : 0;
        u->p.lo_scale = reinterpret_cast<const float*>(G->pool.dev + E.lo_scale);
        u->p.lo_bias = reinterpret_cast<const float*>(G->pool.dev + E.lo_bias);
      }
      if (E.src2 >= 0) {
        // The second addend of a binary tail, in the output's boxes (the
        // schedule gives no LayerNorm output to such a step).
        if (E.lo_dst >= 0 || E.epi != EPI_ADD) throw Error("schedule: a second addend beside a LayerNorm output");
        View e2 = view_of(*G, *L, E.src2);
        uint64_t de[2] = {uint64_t(n), uint64_t(d.npix)}, se[1] = {uint64_t(e2.stride) * 4};
        u->l = make_tensor_map(e2.ptr, 2, de, se, bd);
        u->p.e2 = 1;
      }
      u->p.tiles = int((x.npix + 127) / 128);
      u->p.tiles_x = 0;
      u->p.e_npix = int(d.npix);
    } else {
      // 8x16 output-pixel tiles. The 3x3 conv's A box is the same 8x16
      // window shifted per tap; the stride-2 conv's box spans 16x32 input
      // pixels read every second pixel in both dimensions.
      const int OH = taps == 16 ? op.oh : H, OW = taps == 16 ? op.ow : W;
      uint64_t da[3] = {uint64_t(ci), uint64_t(W), uint64_t(H)};
      uint64_t sa[2] = {uint64_t(x.stride) * 4, uint64_t(W) * uint64_t(x.stride) * 4};
      // The 3x3 conv with at most 64 output columns per tile stages one
      // 16 x 10 box per column shift instead (MODE_CONV3H).
      const bool halo = taps == 9 && tn <= 64;
      uint32_t ba[3] = {32, 16, uint32_t(halo ? 10 : 8)};
      if (taps == 16) {
        uint32_t ba2[3] = {32, 32, 16}, es[3] = {1, 2, 2};
        u->a = make_tensor_map(x.ptr, 3, da, sa, ba2, CU_TENSOR_MAP_SWIZZLE_128B, es);
      } else {
        u->a = make_tensor_map(x.ptr, 3, da, sa, ba);
      }
      uint64_t dd[3] = {uint64_t(n), uint64_t(OW), uint64_t(OH)};
      uint64_t sd[2] = {uint64_t(d.stride) * 4, uint64_t(OW) * uint64_t(d.stride) * 4};
      uint32_t bd[3] = {32, 16, 2};  // per epilogue warp: two rows of the 8x16 tile
      u->d = make_tensor_map(d.ptr, 3, dd, sd, bd);
      u->l = u->d;
      u->p.e_w = OW;
      u->p.e_h = OH;
      u->p.tiles_x = (OW + 15) / 16;
      u->p.tiles = u->p.tiles_x * ((OH + 7) / 8);
      u->p.pad_t = op.pad_top;
      u->p.pad_l = op.pad_left;
    }
    u->p.n_slices = n / tn;
    u->p.tiles *= u->p.n_slices;
    u->p.kb_per_tap = ci / 32;
    u->p.c_in = ci;
    u->p.epi = E.epi;
    u->p.slope = E.slope;
    u->p.bias = bo < 0 ? nullptr : reinterpret_cast<const float*>(G->pool.dev + bo);
    u->p.status = G->status;
    u->n = tn;
    u->taps = taps;
    u->mode = taps == 9 ? (tn <= 64 ? MODE_CONV3H : MODE_CONV3) : (taps == 16 ? MODE_CONV4 : MODE_CONV1);
    u->grid = std::min(u->p.tiles, G->sms);
    u->smem = umma_smem(tn, u->mode);
  };
  st.run = [u](cudaStream_t s) { launch_umma(s, *u); };
  return st;
}

// The 32-to-32 3x3 conv on umma_conv3f_kernel (MAXIM_NO_CONV3F=1 keeps it
// on umma_conv_kernel): 4 x 30 output-pixel tiles, the A box 32 x 6 input
// pixels around each, the weights (WT_CONV3F layout) resident in shared
// memory. Its epilogue takes every tail a schedule gives a 3x3 conv (unary,
// add, multiply) but no LayerNorm statistics, which the schedule therefore
// never assigns it, so the scheduled pass and the op-by-op walk run every
// such conv on this kernel alike.
bool conv3f_shape(const mx_gpu& g, const Layout& L, const mx_op& o) {
  if (o.kind != MX_OP_CONV3X3 || o.c_in != 32 || o.c_out != 32 || !umma_eligible(g, L, o)) return false;
  const char* off = std::getenv("MAXIM_NO_CONV3F");
  return !(off && *off && std::strcmp(off, "0") != 0);
}
bool conv3f_eligible(const mx_gpu& g, const Layout& L, const mx_op& o, const UmmaEpi& E) {
  if (!conv3f_shape(g, L, o) || E.epi == EPI_GATE) return false;
  return E.ln_stats < 0 && E.st_out[0] < 0 && E.st_out[1] < 0 && E.lo_dst < 0 && !E.spatial;
}
struct Conv3fOp {
  CUtensorMap a, w, d, e;
  UmmaConvParams p{};
  int grid = 0;
};
Step umma_conv3f_step(mx_gpu& g, int32_t oi, const mx_op& o, const Layout* L, int64_t wf, int64_t bo,
                      const UmmaEpi& E) {
  auto u = std::make_shared<Conv3fOp>();
  mx_gpu* G = &g;
  const mx_op op = o;
  ++g.umma_ops;
  Step st{oi, 1, nullptr, nullptr};
  st.prepare = [G, L, u, op, wf, bo, E]() {
    View x = view_of(*G, *L, op.src), d = view_of(*G, *L, op.dst);
    const int H = op.h, W = op.wd;
    {
      uint64_t dims[2] = {32, 3 * 2 * 96}, str[1] = {32 * 4};
      uint32_t box[2] = {32, 2 * 96};
      u->w = make_tensor_map(reinterpret_cast<const float*>(G->pool.dev + wf), 2, dims, str, box);
    }
    uint64_t da[3] = {32, uint64_t(W), uint64_t(H)};
    uint64_t sa[2] = {uint64_t(x.stride) * 4, uint64_t(W) * uint64_t(x.stride) * 4};
    uint32_t ba[3] = {32, Conv3fCfg::BOX_W, Conv3fCfg::BOX_H};
    u->a = make_tensor_map(x.ptr, 3, da, sa, ba);
    uint64_t dd[3] = {32, uint64_t(W), uint64_t(H)};
    uint64_t sd[2] = {uint64_t(d.stride) * 4, uint64_t(W) * uint64_t(d.stride) * 4};
    uint32_t bd[3] = {32, Conv3fCfg::OUT_W, 1};  // per epilogue warp: one output row of the tile
    u->d = make_tensor_map(d.ptr, 3, dd, sd, bd);
    u->e = u->d;
    if (E.epi >= EPI_ADD) {
      // The binary tail's operand, read in the output's boxes.
      View e = view_of(*G, *L, E.src);
      uint64_t se[2] = {uint64_t(e.stride) * 4, uint64_t(W) * uint64_t(e.stride) * 4};
      u->e = make_tensor_map(e.ptr, 3, dd, se, bd);
    }
    u->p.e_w = W;
    u->p.e_h = H;
    u->p.tiles_x = (W + Conv3fCfg::OUT_W - 1) / Conv3fCfg::OUT_W;
    u->p.tiles = u->p.tiles_x * ((H + Conv3fCfg::OUT_H - 1) / Conv3fCfg::OUT_H);
    u->p.n_slices = 1;
    u->p.kb_per_tap = 1;
    u->p.c_in = 32;
    u->p.epi = E.epi;
    u->p.slope = E.slope;
    u->p.bias = bo < 0 ? nullptr : reinterpret_cast<const float*>(G->pool.dev + bo);
    u->p.status = G->status;
    u->grid = std::min(u->p.tiles, G->sms);
  };
  st.run = [u](cudaStream_t s) {
    umma_conv3f_kernel<<<unsigned(u->grid), Conv3fCfg::THREADS, Conv3fCfg::SMEM_BYTES, s>>>(u->a, u->w, u->d,
                                                                                           u->e, u->p);
  };
  return st;
}

// The TF32 hi/lo halves of a weight in a given layout, uploaded once.
std::pair<int64_t, int64_t> cached_split(mx_gpu& g, int32_t id, int tag_hi, int tag_lo,
                                         const std::function<std::vector<float>()>& make) {
  const auto kh = std::make_pair(id, tag_hi), kl = std::make_pair(id, tag_lo);
  auto ih = g.wcache.find(kh), il = g.wcache.find(kl);
  if (ih != g.wcache.end() && il != g.wcache.end()) return {ih->second, il->second};
  std::vector<float> hi, lo;
  WcEntry eh, el;
  if (cache_has(g, kh) && cache_has(g, kl)) {
    eh = cache_take(g, kh);
    el = cache_take(g, kl);
  } else {
    split_tf32(make(), hi, lo);
    eh.data = hi.data(), eh.len = int64_t(hi.size());
    el.data = lo.data(), el.len = int64_t(lo.size());
    g.wc_converted += 2;
    if (g.wc_track) src_hash(g, id);
  }
  const int64_t oh = int64_t(g.pool.put(eh.data, size_t(eh.len) * 4));
  const int64_t ol = int64_t(g.pool.put(el.data, size_t(el.len) * 4));
  g.weight_bytes += (eh.len + el.len) * 4;
  g.wcache[kh] = oh;
  g.wcache[kl] = ol;
  g.wbytes[kh] = eh.len * 4;
  g.wbytes[kl] = el.len * 4;
  return {oh, ol};
}

// The tensor-core step of a 2x2 stride-2 transposed conv: a 1x1 GEMM over the
// input pixels with N = 4 c_out columns (tap major), stored through a 5-D
// map onto the output pixels (2y + dy, 2x + dx).
Step umma_convt_step(mx_gpu& g, int32_t oi, const mx_op& o, const Layout* L, int64_t ho, int64_t lo_off, int64_t bo) {
  auto u = std::make_shared<UmmaOp>();
  mx_gpu* G = &g;
  const mx_op op = o;
  ++g.umma_ops;
  Step st{oi, 1, nullptr, nullptr};
  st.prepare = [G, L, u, op, ho, lo_off, bo]() {
    View x = view_of(*G, *L, op.src), d = view_of(*G, *L, op.dst);
    const int co = op.c_out, ci = op.c_in, n = 4 * co, tn = 128, W = op.wd, H = op.h;
    const float* whi = reinterpret_cast<const float*>(G->pool.dev + ho);
    const float* wlo = reinterpret_cast<const float*>(G->pool.dev + lo_off);
    {
      uint64_t dims[2] = {uint64_t(ci), uint64_t(n)}, str[1] = {uint64_t(ci) * 4};
      uint32_t box[2] = {32, uint32_t(tn)};
      u->b = make_tensor_map(whi, 2, dims, str, box);
      u->blo = make_tensor_map(wlo, 2, dims, str, box);
    }
    uint64_t da[2] = {uint64_t(ci), uint64_t(x.npix)}, sa[1] = {uint64_t(x.stride) * 4};
    uint32_t ba[2] = {32, 128};
    u->a = make_tensor_map(x.ptr, 2, da, sa, ba);
    // Output pixel (2y + dy, 2x + dx) of a 2W-wide image: dims (c, dx, x, dy, y).
    const uint64_t px = uint64_t(d.stride) * 4;
    uint64_t dd[5] = {uint64_t(co), 2, uint64_t(W), 2, uint64_t(H)};
    uint64_t sd[4] = {px, 2 * px, 2 * uint64_t(W) * px, 4 * uint64_t(W) * px};
    uint32_t bd[5] = {32, 1, 32, 1, 1};
    u->d = make_tensor_map(d.ptr, 5, dd, sd, bd);
    u->l = u->d;
    u->p.tiles = int((x.npix + 127) / 128);
    u->p.tiles_x = 0;
    u->p.e_npix = int(x.npix);
    u->p.e_w = W;
    u->p.co = co;
    u->p.n_slices = n / tn;
    u->p.tiles *= u->p.n_slices;
    u->p.kb_per_tap = ci / 32;
    u->p.c_in = ci;
    u->p.epi = EPI_NONE;
    u->p.bias = bo < 0 ? nullptr : reinterpret_cast<const float*>(G->pool.dev + bo);
    u->p.status = G->status;
    u->n = tn;
    u->taps = 1;
    u->mode = MODE_CONVT;
    u->grid = std::min(u->p.tiles, G->sms);
    u->smem = umma_smem(tn, u->mode);
  };
  st.run = [u](cudaStream_t s) { launch_umma(s, *u); };
  return st;
}

// Build the step that runs op `o` (plan op oi, as the plan has it or as the
// schedule rewrote it, `fs` non-null) over layout L. Weight layouts are
// converted here and recorded in the pool (once per weight and layout);
// pointers are resolved after the pool is uploaded, so each step captures the
// pool offset and reads the base at run time.
Step make_step(mx_gpu& g, const mx_plan& plan, const mx_op& o, int32_t oi, const Layout* L, const SchedStep* fs) {
  auto W = [&](int32_t id) -> std::vector<float> {
    if (id < 0) return {};
    return std::vector<float>(plan.weights[id], plan.weights[id] + plan.weight_lens[id]);
  };
  auto raw = [&](int32_t id) { return cached(g, id, WT_RAW, [&] { return W(id); }); };
  UmmaEpi E;
  if (fs) {
    E.epi = fs->epi;
    E.src = fs->epi_src;
    E.src2 = fs->epi_src2;
    E.slope = fs->epi_slope;
    if (fs->gate_perm >= 0) {
      E.spatial = true;
      E.perm = plan.ops[fs->gate_perm];
    }
    if (fs->ln_stats >= 0) {
      E.ln_stats = fs->ln_stats;
      E.ln_scale = raw(fs->ln_scale);
      E.ln_bias = raw(fs->ln_bias);
    }
    if (fs->ln_out >= 0) {
      E.lo_dst = fs->ln_out;
      E.lo_c0 = fs->ln_out_c0;
      E.lo_only = fs->ln_out_only;
      E.lo_scale = raw(fs->ln_out_scale);
      E.lo_bias = raw(fs->ln_out_bias);
    }
    for (int g2 = 0; g2 < 2; ++g2) {
      E.st_out[g2] = fs->stats_out[g2];
      E.st_c0[g2] = fs->stats_c0[g2];
    }
    E.st_c = fs->stats_c;
  }
  bool needs_umma = (E.epi != EPI_NONE && o.kind != MX_OP_CHAN_SCALE) || E.spatial || E.ln_stats >= 0 ||
                    E.st_out[0] >= 0 || E.lo_dst >= 0;
  bool on_umma = false;
  mx_gpu* G = &g;
  auto P = [G](int64_t off) -> const float* {
    return off < 0 ? nullptr : reinterpret_cast<const float*>(G->pool.dev + off);
  };
  Step st{oi, 1, nullptr};
  const int32_t dst = o.dst, src = o.src, src2 = o.src2;
  switch (o.kind) {
    case MX_OP_COPY:
    case MX_OP_ADD:
    case MX_OP_MUL:
    case MX_OP_GATE_APPLY:
    case MX_OP_GELU:
    case MX_OP_LRELU:
    case MX_OP_SIGMOID: {
      const mx_buf& db = g.bufs[size_t(dst)];
      if (db.c * db.h * db.w != o.n)
        throw Error(fmt("op %d: an elementwise op over %lld values on a %lldx%lldx%lld buffer is not supported", oi,
                        (long long)o.n, (long long)db.c, (long long)db.h, (long long)db.w));
      int kind = o.kind;
      float slope = o.slope;
      st.run = [G, L, kind, dst, src, src2, slope](cudaStream_t s) {
        View d = view_of(*G, *L, dst), a = view_of(*G, *L, src);
        View b{nullptr, 0, 0, 0};
        if (src2 >= 0) b = view_of(*G, *L, src2);
        switch (kind) {
          case MX_OP_COPY: launch_ew<EW_COPY>(s, d, a, b, slope); break;
          case MX_OP_ADD: launch_ew<EW_ADD>(s, d, a, b, slope); break;
          case MX_OP_MUL: launch_ew<EW_MUL>(s, d, a, b, slope); break;
          case MX_OP_GATE_APPLY: launch_ew<EW_GATE>(s, d, a, b, slope); break;
          case MX_OP_GELU: launch_ew<EW_GELU>(s, d, a, b, slope); break;
          case MX_OP_LRELU: launch_ew<EW_LRELU>(s, d, a, b, slope); break;
          default: launch_ew<EW_SIGMOID>(s, d, a, b, slope); break;
        }
      };
      break;
    }
    case MX_OP_CHAN_LN: {
      if (fs && fs->stats_only) {
        // The statistics half only (its consumer normalises on load).
        st.run = [G, L, dst, src](cudaStream_t s) {
          View d = view_of(*G, *L, dst), x = view_of(*G, *L, src);
          const int c = int(x.c), np = int(x.npix);
          const int pb = c <= 64 ? 128 : (c == 128 ? 64 : 32);
          const unsigned grid = unsigned((np + pb - 1) / pb);
          const size_t smem = size_t(pb) * (c + 1) * sizeof(float);
          float2* sp = reinterpret_cast<float2*>(d.ptr);
          const int sx = int(x.stride);
          if (c == 32) chan_stats_tile_kernel<32><<<grid, 128, smem, s>>>(np, x.ptr, sx, sp, kLnEps);
          else if (c == 64) chan_stats_tile_kernel<64><<<grid, 128, smem, s>>>(np, x.ptr, sx, sp, kLnEps);
          else if (c == 128) chan_stats_tile_kernel<128><<<grid, 128, smem, s>>>(np, x.ptr, sx, sp, kLnEps);
          else chan_stats_tile_kernel<256><<<grid, 128, smem, s>>>(np, x.ptr, sx, sp, kLnEps);
        };
        break;
      }
      int64_t ws = raw(o.scale), wb = raw(o.bias);
      st.run = [G, L, P, dst, src, ws, wb](cudaStream_t s) {
        View d = view_of(*G, *L, dst), x = view_of(*G, *L, src);
        const int c = int(x.c), np = int(x.npix);
        if (aligned4(d) && aligned4(x) && (c == 32 || c == 64 || c == 128 || c == 256)) {
          const int pb = c <= 64 ? 128 : (c == 128 ? 64 : 32);
          const unsigned grid = unsigned((np + pb - 1) / pb);
          // the tile (rows of c + 1 floats, rounded to an even count), then
          // pb (mean, rstd) pairs
          const size_t smem = ((size_t(pb) * (c + 1) + 1) & ~size_t(1)) * sizeof(float) + size_t(pb) * 8;
          const int sx = int(x.stride), sy = int(d.stride);
          if (c == 32) chan_ln_tile_kernel<32><<<grid, 128, smem, s>>>(np, x.ptr, sx, P(ws), P(wb), d.ptr, sy, kLnEps);
          else if (c == 64) chan_ln_tile_kernel<64><<<grid, 128, smem, s>>>(np, x.ptr, sx, P(ws), P(wb), d.ptr, sy, kLnEps);
          else if (c == 128) chan_ln_tile_kernel<128><<<grid, 128, smem, s>>>(np, x.ptr, sx, P(ws), P(wb), d.ptr, sy, kLnEps);
          else chan_ln_tile_kernel<256><<<grid, 128, smem, s>>>(np, x.ptr, sx, P(ws), P(wb), d.ptr, sy, kLnEps);
        } else if (aligned4(d) && aligned4(x)) {
          chan_ln_kernel4<<<blocks_for(x.npix, 128), 128, 0, s>>>(x.npix, c, x.ptr, x.stride, P(ws), P(wb), d.ptr,
                                                                  d.stride, kLnEps);
        } else {
          chan_ln_kernel1<<<blocks_for(x.npix, 128), 128, 0, s>>>(x.npix, c, x.ptr, x.stride, P(ws), P(wb), d.ptr,
                                                                  d.stride, kLnEps);
        }
      };
      break;
    }
    case MX_OP_CHAN_MEAN: {
      // Two phases over a scratch of per-block partial sums (deterministic).
      const int64_t npix = int64_t(o.hw);
      const int nb = int(std::max<int64_t>(1, std::min<int64_t>((npix + 511) / 512, 1024)));
      const int per = int((npix + nb - 1) / nb);
      g.scratch_len = std::max<int64_t>(g.scratch_len, int64_t(nb) * o.c);
      st.kernels = 2;
      st.run = [G, L, dst, src, nb, per](cudaStream_t s) {
        View d = view_of(*G, *L, dst), x = view_of(*G, *L, src);
        if (aligned4(x) && x.c <= 1024) {
          const int c4 = int(x.c / 4);
          chan_mean_partial_kernel<<<unsigned(nb), 256, 0, s>>>(int(x.npix), c4, per, x.ptr, int(x.stride),
                                                                G->scratch);
          chan_mean_final_tree_kernel<<<unsigned(x.c), 256, 0, s>>>(nb, int(x.c), int(x.npix), G->scratch, d.ptr);
        } else {
          chan_mean_kernel<<<unsigned(x.c), 512, 0, s>>>(x.npix, x.ptr, x.stride, d.ptr);
        }
      };
      break;
    }
    case MX_OP_CHAN_SCALE: {
      if (E.epi == EPI_ADD && E.src2 >= 0) {
        // ((x * s) + residual) + residual 2 in one pass (views 4-channel
        // aligned, checked by the schedule).
        const int32_t res = E.src, res2 = E.src2;
        st.run = [G, L, dst, src, src2, res, res2](cudaStream_t s) {
          View d = view_of(*G, *L, dst), x = view_of(*G, *L, src), sc = view_of(*G, *L, src2),
               r = view_of(*G, *L, res), r2 = view_of(*G, *L, res2);
          const int c4 = int(x.c / 4), total4 = int(x.npix) * c4;
          chan_scale_add2_4_kernel<<<blocks_for(total4, TPB), TPB, 0, s>>>(
              total4, c4, x.ptr, int(x.stride), sc.ptr, r.ptr, int(r.stride), r2.ptr, int(r2.stride), d.ptr,
              int(d.stride));
        };
        on_umma = needs_umma = false;
        break;
      }
      if (E.epi == EPI_ADD) {
        // x * s + residual in one pass (the schedule checked the views are
        // 4-channel aligned).
        const int32_t res = E.src;
        st.run = [G, L, dst, src, src2, res](cudaStream_t s) {
          View d = view_of(*G, *L, dst), x = view_of(*G, *L, src), sc = view_of(*G, *L, src2),
               r = view_of(*G, *L, res);
          const int c4 = int(x.c / 4), total4 = int(x.npix) * c4;
          chan_scale_add4_kernel<<<blocks_for(total4, TPB), TPB, 0, s>>>(total4, c4, x.ptr, int(x.stride), sc.ptr,
                                                                         r.ptr, int(r.stride), d.ptr, int(d.stride));
        };
        on_umma = needs_umma = false;
        break;
      }
      st.run = [G, L, dst, src, src2](cudaStream_t s) {
        View d = view_of(*G, *L, dst), x = view_of(*G, *L, src), sc = view_of(*G, *L, src2);
        if (aligned4(d) && aligned4(x) && aligned4(sc)) {
          const int c4 = int(x.c / 4), total4 = int(x.npix) * c4;
          chan_scale4_kernel<<<blocks_for(total4, TPB), TPB, 0, s>>>(total4, c4, x.ptr, int(x.stride), sc.ptr, d.ptr,
                                                                     int(d.stride));
        } else {
          chan_scale_kernel<<<blocks_for(x.npix * x.c, TPB), TPB, 0, s>>>(x.npix, int(x.c), x.ptr, x.stride, sc.ptr,
                                                                          d.ptr, d.stride);
        }
      };
      break;
    }
    case MX_OP_CONV1X1: {
      if (umma_eligible(g, *L, o)) {
        const auto hl = cached_split(g, o.w, WT_HI, WT_LO, [&] { return W(o.w); });
        st = umma_conv_step(g, oi, o, L, hl.first, hl.second, raw(o.bias), E);
        on_umma = true;
        break;
      }
      if (small_conv(o)) {
        // [c_out][c_in] -> [c_in][c_out]
        const int ci = o.c_in, co = o.c_out;
        const int64_t wt = cached(g, o.w, WT_T, [&] {
          auto w = W(o.w);
          std::vector<float> t(w.size());
          for (int n = 0; n < co; ++n)
            for (int k = 0; k < ci; ++k) t[size_t(k) * co + n] = w[size_t(n) * ci + k];
          return t;
        });
        const int64_t bo = raw(o.bias);
        const int tail = E.epi == EPI_GELU ? EW_GELU : E.epi == EPI_LRELU ? EW_LRELU : E.epi == EPI_SIGMOID ? EW_SIGMOID : -1;
        if (E.epi != EPI_NONE && tail < 0) throw Error(fmt("op %d: a small 1x1 conv takes only a unary tail", oi));
        const float slope = E.slope;
        needs_umma = false;
        st.run = [G, L, P, dst, src, wt, bo, ci, co, tail, slope](cudaStream_t s) {
          View d = view_of(*G, *L, dst), x = view_of(*G, *L, src);
          const dim3 grid(unsigned(x.npix), unsigned((co + 127) / 128));
          const size_t ws = size_t(ci) * size_t(std::min(co, 128)) * sizeof(float);
          const int stage_w = ws + size_t(ci) * sizeof(float) <= 48 * 1024;
          const size_t smem = size_t(ci) * sizeof(float) + (stage_w ? ws : 0);
          conv1x1_small_kernel<<<grid, 128, smem, s>>>(ci, co, x.ptr, x.stride, P(wt), P(bo), d.ptr, d.stride, tail,
                                                       slope, stage_w);
        };
        break;
      }
      int64_t wo = raw(o.w), bo = raw(o.bias);  // [c_out][c_in]
      int ci = o.c_in, co = o.c_out;
      st.run = [G, L, P, dst, src, wo, bo, ci, co](cudaStream_t s) {
        View d = view_of(*G, *L, dst), x = view_of(*G, *L, src);
        ProbConv1x1 p{x.ptr, x.stride, P(wo), P(bo), d.ptr, d.stride, x.npix, co, ci};
        if (co <= 32) launch_gemm<64, 32>(s, p, 1);
        else launch_gemm<64, 64>(s, p, 1);
      };
      break;
    }
    case MX_OP_CONV3X3:
    case MX_OP_CONV4X4S2: {
      int ks = o.kind == MX_OP_CONV3X3 ? 3 : 4;
      int ci = o.c_in, co = o.c_out;
      // [co][ci][k][k] -> [co][tap][ci]
      auto ktap = [&] {
        auto w = W(o.w);
        std::vector<float> wt(w.size());
        for (int oc = 0; oc < co; ++oc)
          for (int ic = 0; ic < ci; ++ic)
            for (int t = 0; t < ks * ks; ++t)
              wt[(size_t(oc) * ks * ks + t) * ci + ic] = w[(size_t(oc) * ci + ic) * ks * ks + t];
        return wt;
      };
      if (ks == 3 && conv3f_eligible(g, *L, o, E)) {
        // [co][tap][ci] split into TF32 halves, then [ky][hi, lo][kx][co][ci].
        const int64_t wf = cached(g, o.w, WT_CONV3F, [&] {
          std::vector<float> hi, lo;
          split_tf32(ktap(), hi, lo);
          std::vector<float> f(size_t(3 * 2 * 3 * 32 * 32));
          for (int ky = 0; ky < 3; ++ky)
            for (int part = 0; part < 2; ++part)
              for (int kx = 0; kx < 3; ++kx)
                for (int oc = 0; oc < 32; ++oc)
                  for (int ic = 0; ic < 32; ++ic)
                    f[((((size_t(ky) * 2 + part) * 3 + kx) * 32 + oc) * 32) + ic] =
                        (part ? lo : hi)[(size_t(oc) * 9 + ky * 3 + kx) * 32 + ic];
          return f;
        });
        st = umma_conv3f_step(g, oi, o, L, wf, raw(o.bias), E);
        on_umma = true;
        break;
      }
      if (umma_eligible(g, *L, o)) {
        const auto hl = cached_split(g, o.w, WT_KTAP_HI, WT_KTAP_LO, ktap);
        st = umma_conv_step(g, oi, o, L, hl.first, hl.second, raw(o.bias), E);
        on_umma = true;
        break;
      }
      int64_t wo = cached(g, o.w, WT_KTAP, ktap), bo = raw(o.bias);
      int h = o.h, wd = o.wd;
      if (ks == 3 && (ci == 3 || co == 3)) {
        // The image-facing convs (3 input or 3 output channels). Their
        // weights travel as a kernel parameter (a constant bank): per
        // 32-output-channel chunk for c_in = 3, whole for c_out = 3 with
        // c_in in {32, 64, 128}.
        const std::vector<float> wk = ktap(), bk = W(o.bias);
        const bool cout_c = co == 3 && ci == 32 || co == 3 && ci == 64 || co == 3 && ci == 128;
        if (ci == 3) {
          std::vector<Cin3Weights> chunks(size_t((co + 31) / 32));
          for (size_t k = 0; k < chunks.size(); ++k) {
            Cin3Weights& c = chunks[k];
            memset(&c, 0, sizeof(c));
            for (int oo = 0; oo < 32 && int(k) * 32 + oo < co; ++oo) {
              const int oc = int(k) * 32 + oo;
              for (int t = 0; t < 27; ++t) c.w[t * 32 + oo] = wk[size_t(oc) * 27 + t];
              c.b[oo] = bk.empty() ? 0.0f : bk[size_t(oc)];
            }
          }
          st.kernels = int(chunks.size());
          st.run = [G, L, dst, src, co, h, wd, chunks](cudaStream_t s) {
            View d = view_of(*G, *L, dst), x = view_of(*G, *L, src);
            for (size_t k = 0; k < chunks.size(); ++k)
              conv3x3_cin3c_kernel<<<unsigned((h * wd + 127) / 128), 128, 0, s>>>(
                  h, wd, std::min(32, co - int(k) * 32), x.ptr, int(x.stride), d.ptr + 32 * k, int(d.stride),
                  chunks[k]);
          };
          break;
        }
        if (cout_c) {
          auto fill = [&](auto& c) {
            memset(&c, 0, sizeof(c));
            for (size_t i = 0; i < wk.size(); ++i) c.w[i] = wk[i];
            for (int oc = 0; oc < 3; ++oc) c.b[oc] = bk.empty() ? 0.0f : bk[size_t(oc)];
          };
          auto c32 = std::make_shared<Cout3Weights<32>>();
          auto c64 = std::make_shared<Cout3Weights<64>>();
          auto c128 = std::make_shared<Cout3Weights<128>>();
          if (ci == 32) fill(*c32);
          if (ci == 64) fill(*c64);
          if (ci == 128) fill(*c128);
          st.run = [G, L, P, dst, src, wo, bo, ci, h, wd, c32, c64, c128](cudaStream_t s) {
            View d = view_of(*G, *L, dst), x = view_of(*G, *L, src);
            dim3 grid(unsigned((wd + 15) / 16), unsigned((h + 15) / 16));
            if (!aligned4(x)) {
              conv3x3_cout3_kernel<<<grid, 256, 0, s>>>(h, wd, ci, x.ptr, int(x.stride), P(wo), P(bo), d.ptr,
                                                        int(d.stride));
            } else if (ci == 32) {
              conv3x3_cout3c_kernel<32><<<grid, 256, 0, s>>>(h, wd, x.ptr, int(x.stride), d.ptr, int(d.stride), *c32);
            } else if (ci == 64) {
              conv3x3_cout3c_kernel<64><<<grid, 256, 0, s>>>(h, wd, x.ptr, int(x.stride), d.ptr, int(d.stride), *c64);
            } else {
              conv3x3_cout3c_kernel<128><<<grid, 256, 0, s>>>(h, wd, x.ptr, int(x.stride), d.ptr, int(d.stride),
                                                              *c128);
            }
          };
          break;
        }
        st.run = [G, L, P, dst, src, wo, bo, ci, co, h, wd](cudaStream_t s) {
          View d = view_of(*G, *L, dst), x = view_of(*G, *L, src);
          if (ci == 3) {
            dim3 grid(unsigned((h * wd + 127) / 128), unsigned((co + 31) / 32));
            conv3x3_cin3_kernel<<<grid, 128, 0, s>>>(h, wd, co, x.ptr, int(x.stride), P(wo), P(bo), d.ptr,
                                                     int(d.stride));
          } else {
            dim3 grid(unsigned((wd + 15) / 16), unsigned((h + 15) / 16));
            conv3x3_cout3_kernel<<<grid, 256, 0, s>>>(h, wd, ci, x.ptr, int(x.stride), P(wo), P(bo), d.ptr,
                                                      int(d.stride));
          }
        };
        break;
      }
      int oh = ks == 3 ? h : o.oh, ow = ks == 3 ? wd : o.ow;
      int stride = ks == 3 ? 1 : 2, pt = ks == 3 ? 1 : o.pad_top, pl = ks == 3 ? 1 : o.pad_left;
      st.run = [G, L, P, dst, src, wo, bo, ci, co, h, wd, oh, ow, ks, stride, pt, pl](cudaStream_t s) {
        View d = view_of(*G, *L, dst), x = view_of(*G, *L, src);
        ProbConvKxK p{x.ptr, x.stride, P(wo), P(bo), d.ptr, d.stride, int64_t(oh) * ow, co, ks * ks * ci,
                      ci, h, wd, oh, ow, ks, stride, pt, pl};
        if (co <= 32) launch_gemm<64, 32>(s, p, 1);
        else launch_gemm<64, 64>(s, p, 1);
      };
      break;
    }
    case MX_OP_CONVT2X2: {
      int ci = o.c_in, co = o.c_out;
      // [ci][co][2][2] (flipped) -> [tap*co + o][ci]
      auto tapmajor = [&] {
        auto w = W(o.w);
        std::vector<float> wt(w.size());
        for (int ic = 0; ic < ci; ++ic)
          for (int oc = 0; oc < co; ++oc)
            for (int t = 0; t < 4; ++t) wt[(size_t(t) * co + oc) * ci + ic] = w[(size_t(ic) * co + oc) * 4 + t];
        return wt;
      };
      if (umma_convt_eligible(g, *L, o)) {
        const auto hl = cached_split(g, o.w, WT_CONVT_HI, WT_CONVT_LO, tapmajor);
        const int64_t b4 = cached(g, o.bias, WT_BIAS4, [&] {
          auto b = W(o.bias);
          std::vector<float> r(4 * b.size());
          for (size_t t = 0; t < 4; ++t) std::copy(b.begin(), b.end(), r.begin() + long(t * b.size()));
          return r;
        });
        st = umma_convt_step(g, oi, o, L, hl.first, hl.second, b4);
        on_umma = true;
        break;
      }
      int64_t wo = cached(g, o.w, WT_CONVT, tapmajor);
      int64_t bo = raw(o.bias);
      int wd = o.wd;
      st.run = [G, L, P, dst, src, wo, bo, ci, co, wd](cudaStream_t s) {
        View d = view_of(*G, *L, dst), x = view_of(*G, *L, src);
        ProbConvT p{x.ptr, x.stride, P(wo), P(bo), d.ptr, d.stride, x.npix, 4 * co, ci, co, wd};
        launch_gemm<64, 64>(s, p, 1);
      };
      break;
    }
    case MX_OP_GATE_MM: {
      if (umma_gate_eligible(g, *L, o) || E.spatial) {
        const auto hl = cached_split(g, o.w, WT_HI, WT_LO, [&] { return W(o.w); });
        st = umma_gate_step(g, oi, o, L, hl.first, hl.second, raw(o.bias), E);
        on_umma = true;
        break;
      }
      int64_t wo = raw(o.w), bo = raw(o.bias);  // [out][in]
      int c = o.c, outer = o.outer, inner = o.inner, mode = o.mode;
      st.run = [G, L, P, dst, src, wo, bo, c, outer, inner, mode](cudaStream_t s) {
        View d = view_of(*G, *L, dst), x = view_of(*G, *L, src);
        if (mode == 0) {
          ProbGate0 p{x.ptr, x.stride, P(wo), P(bo), d.ptr, d.stride, outer, inner * c, outer, c, inner};
          launch_gemm<64, 64>(s, p, 1);
        } else {
          ProbGate1 p{x.ptr, x.stride, P(wo), P(bo), d.ptr, d.stride, inner, c, inner, inner};
          if (c <= 32) launch_gemm<64, 32>(s, p, outer);
          else launch_gemm<64, 64>(s, p, outer);
        }
      };
      break;
    }
    case MX_OP_BLOCK_PERM: {
      const mx_op op = o;
      if (int64_t(o.gh) * o.fh != o.h || int64_t(o.gw) * o.fw != o.wd)
        throw Error(fmt("op %d: a %dx%d blocking of a %dx%d plane drops pixels; the executor needs plans whose "
                        "planes the blocks tile exactly (the pad-to-64 pipeline always does)",
                        oi, o.gh * o.fh, o.gw * o.fw, o.h, o.wd));
      st.run = [G, L, op](cudaStream_t s) {
        View d = view_of(*G, *L, op.dst), x = view_of(*G, *L, op.src);
        if (aligned4(d) && aligned4(x)) {
          const int c4 = op.c / 4, total4 = op.h * op.wd * c4;
          block_perm4_kernel<<<blocks_for(total4, TPB), TPB, 0, s>>>(total4, c4, op.wd, op.gw, op.fh, op.fw,
                                                                     op.gh * op.gw, op.fh * op.fw, op.swap, op.forward,
                                                                     x.ptr, int(x.stride), d.ptr, int(d.stride));
          return;
        }
        int64_t total = int64_t(op.h) * op.wd * op.c;
        block_perm_kernel<<<blocks_for(total, TPB), TPB, 0, s>>>(total, op.c, op.wd, op.gw, op.fh, op.fw,
                                                                 op.gh * op.gw, op.fh * op.fw, op.swap, op.forward,
                                                                 x.ptr, x.stride, d.ptr, d.stride);
      };
      break;
    }
    case MX_OP_DOWN_S: {
      const mx_op op = o;
      st.run = [G, L, op](cudaStream_t s) {
        View d = view_of(*G, *L, op.dst), x = view_of(*G, *L, op.src);
        int64_t total = int64_t(op.oh) * op.ow * op.c;
        down_s_kernel<<<blocks_for(total, TPB), TPB, 0, s>>>(total, op.c, op.wd, op.ow, op.stride, op.off, x.ptr,
                                                             x.stride, d.ptr, d.stride);
      };
      break;
    }
    case MX_OP_RESIZE: {
      const mx_op op = o;
      HostTaps tx = make_taps(o.win, o.wout, 1 << 30), ty = make_taps(o.hin, o.hout, 64);
      int64_t tx_j0 = int64_t(g.pool.put(tx.j0)), tx_w0 = int64_t(g.pool.put(tx.w0)),
              tx_c = int64_t(g.pool.put(tx.cnt)), tx_w = int64_t(g.pool.put(tx.w)),
              tx_s = int64_t(g.pool.put(tx.wsum)), tx_r = int64_t(g.pool.put(tx.wrcp));
      int64_t ty_j0 = int64_t(g.pool.put(ty.j0)), ty_w0 = int64_t(g.pool.put(ty.w0)),
              ty_c = int64_t(g.pool.put(ty.cnt)), ty_w = int64_t(g.pool.put(ty.w)),
              ty_s = int64_t(g.pool.put(ty.wsum)), ty_r = int64_t(g.pool.put(ty.wrcp));
      // Upsampling whose every tile of kRzTY output rows reads at most kRzRows
      // input rows runs both passes in one launch (resize_hv4_kernel).
      const int c4 = o.c / 4;
      bool hv = o.win <= o.wout && o.hin <= o.hout && o.c % 4 == 0 && c4 > 0 && (c4 & (c4 - 1)) == 0 && c4 <= 256;
      for (int y0 = 0; hv && y0 < o.hout; y0 += kRzTY) {
        int r_lo = 1 << 30, r_hi = -1;
        for (int yo = y0; yo < std::min(y0 + kRzTY, o.hout); ++yo) {
          r_lo = std::min(r_lo, ty.j0[size_t(yo)]);
          r_hi = std::max(r_hi, ty.j0[size_t(yo)] + ty.cnt[size_t(yo)] - 1);
        }
        hv = r_hi - r_lo + 1 <= kRzRows;
      }
      for (size_t i = 0; hv && i < ty.cnt.size(); ++i) hv = ty.cnt[i] <= kRzTaps;
      for (size_t i = 0; hv && i < tx.cnt.size(); ++i) hv = tx.cnt[i] <= kRzTaps;
      st.kernels = hv ? 1 : 2;
      st.run = [G, L, op, hv, tx_j0, tx_w0, tx_c, tx_w, tx_s, tx_r, ty_j0, ty_w0, ty_c, ty_w, ty_s,
                ty_r](cudaStream_t s) {
        auto I = [G](int64_t off) { return reinterpret_cast<const int*>(G->pool.dev + off); };
        auto F = [G](int64_t off) { return reinterpret_cast<const float*>(G->pool.dev + off); };
        View d = view_of(*G, *L, op.dst), x = view_of(*G, *L, op.src), t = view_of(*G, *L, op.tmp);
        const int c4 = op.c / 4;
        if (aligned4(d) && aligned4(x) && aligned4(t) && op.c % 4 == 0 && (c4 & (c4 - 1)) == 0 && op.hin < 65536 &&
            op.hout < 65536) {
          TapTable4 TX{I(tx_j0), I(tx_w0), I(tx_c), F(tx_w), F(tx_s), F(tx_r)};
          TapTable4 TY{I(ty_j0), I(ty_w0), I(ty_c), F(ty_w), F(ty_s), F(ty_r)};
          int lg4 = 0;
          while ((1 << lg4) < c4) ++lg4;
          if (hv) {
            const int cols = (kRzTile / 4) >> lg4;
            const dim3 g((unsigned(op.wout) + cols - 1) / cols, (unsigned(op.hout) + kRzTY - 1) / kRzTY);
            resize_hv4_kernel<<<g, kRzTile / 4, 0, s>>>(lg4, op.win, op.wout, op.hout, TX, TY, x.ptr, int(x.stride),
                                                        d.ptr, int(d.stride));
            return;
          }
          const int row = op.wout * c4;
          const dim3 g1(unsigned(blocks_for(row, TPB)), unsigned(op.hin)), g2(unsigned(blocks_for(row, TPB)),
                                                                              unsigned(op.hout));
          resize_h4_kernel<<<g1, TPB, 0, s>>>(lg4, op.win, op.wout, TX, x.ptr, int(x.stride), t.ptr, int(t.stride));
          resize_v4_kernel<<<g2, TPB, 0, s>>>(lg4, op.wout, TY, t.ptr, int(t.stride), d.ptr, int(d.stride));
          return;
        }
        TapTable TX{I(tx_j0), I(tx_w0), I(tx_c), F(tx_w), F(tx_s)};
        TapTable TY{I(ty_j0), I(ty_w0), I(ty_c), F(ty_w), F(ty_s)};
        int64_t t1 = int64_t(op.hin) * op.wout * op.c;
        resize_h_kernel<<<blocks_for(t1, TPB), TPB, 0, s>>>(t1, op.c, op.win, op.wout, TX, x.ptr, x.stride, t.ptr,
                                                            t.stride);
        int64_t t2 = int64_t(op.hout) * op.wout * op.c;
        resize_v_kernel<<<blocks_for(t2, TPB), TPB, 0, s>>>(t2, op.c, op.hin, op.hout, op.wout, TY, t.ptr, t.stride,
                                                            d.ptr, d.stride);
      };
      break;
    }
    default:
      throw Error(fmt("op %d: unknown op kind %d", oi, o.kind));
  }
  if (needs_umma && !on_umma)
    throw Error(fmt("op %d: the schedule fused work into an op that does not run on the tensor-core kernel", oi));
  return st;
}

// Bracket a step list with the boundary transposes (host NCHW <-> arena NHWC).
void add_boundary_steps(mx_gpu& g, std::vector<Step>& steps, const Layout* L) {
  mx_gpu* G = &g;
  int32_t in = g.input, out = g.output;
  Step a{-1, 1, [G, L, in](cudaStream_t s) {
           View d = view_of(*G, *L, in);
           nchw_to_nhwc_kernel<<<blocks_for(d.npix * d.c, TPB), TPB, 0, s>>>(d.npix, int(d.c), G->io_in, d.ptr,
                                                                             d.stride);
         }};
  Step b{-1, 1, [G, L, out](cudaStream_t s) {
           View x = view_of(*G, *L, out);
           nhwc_to_nchw_kernel<<<blocks_for(x.npix * x.c, TPB), TPB, 0, s>>>(x.npix, int(x.c), x.ptr, x.stride,
                                                                             G->io_out);
         }};
  steps.insert(steps.begin(), std::move(a));
  steps.push_back(std::move(b));
}

void capture_graph(mx_gpu& g) {
  if (g.graph_exec) return;
  MX_CUDA(cudaStreamBeginCapture(g.stream, cudaStreamCaptureModeThreadLocal));
  try {
    for (auto& st : g.fsteps) st.run(g.stream);
  } catch (...) {
    cudaGraph_t tmp;
    cudaStreamEndCapture(g.stream, &tmp);
    if (tmp) cudaGraphDestroy(tmp);
    throw;
  }
  MX_CUDA(cudaStreamEndCapture(g.stream, &g.graph));
  MX_CUDA(cudaGraphInstantiate(&g.graph_exec, g.graph, 0));
}

// The schedule's questions about a plan, answered for layouts whose roots
// are 256-byte aligned (the schedule's own packing): only a view's channel
// offset and its root's width decide alignment.
ScheduleHooks schedule_hooks(const mx_gpu& g) {
  const mx_gpu* G = &g;
  ScheduleHooks h;
  h.umma = [G](const mx_op& o) {
    if (o.kind == MX_OP_CONVT2X2) return umma_convt_eligible(*G, G->roffs, o);
    return o.kind == MX_OP_GATE_MM ? umma_gate_eligible(*G, G->roffs, o) : umma_eligible(*G, G->roffs, o);
  };
  h.gate_spatial = [G](const mx_op& gate, const mx_op& perm) {
    return umma_gate_spatial_ok(*G, G->roffs, gate, perm) && tma_view(*G, G->roffs, gate.dst, gate.c);
  };
  h.tma_view = [G](int32_t b, int n) { return tma_view(*G, G->roffs, b, n); };
  h.small_conv = [](const mx_op& o) { return small_conv(o); };
  // The split stage normalises A for 1x1 convs whose input has a channel
  // count the statistics kernel takes (32..256, aligned rows). A 3x3 conv
  // could too, but it would normalise every input pixel once per tap (nine
  // times), which measured slower than the separate LayerNorm.
  h.ln_on_load = [G](const mx_op& o) {
    if (o.kind != MX_OP_CONV1X1 || small_conv(o)) return false;
    const int c = o.c_in;
    return (c == 32 || c == 64 || c == 128 || c == 256) && tma_view(*G, G->roffs, o.src, c);
  };
  // A 1x1 / 3x3 / 4x4 conv on the tensor-core kernel writes whole pixel rows
  // per epilogue thread, one output slice at a time.
  h.stats_slice = [G](const mx_op& o) {
    if (o.kind != MX_OP_CONV1X1 && o.kind != MX_OP_CONV3X3 && o.kind != MX_OP_CONV4X4S2) return 0;
    if (conv3f_shape(*G, G->roffs, o)) return 0;
    return umma_eligible(*G, G->roffs, o) ? umma_tile_n(o.c_out) : 0;
  };
  return h;
}

// Host-side set-up shared by mx_gpu_new and the schedule inspector: copy the
// plan's tables and work out the scheduled pass.
Schedule plan_schedule(mx_gpu& g, const mx_plan& plan) {
  g.bufs.assign(plan.bufs, plan.bufs + plan.n_bufs);
  g.offs.assign(plan.offs, plan.offs + plan.n_bufs);
  g.alias_parent.assign(plan.alias_parent, plan.alias_parent + plan.n_bufs);
  g.ops.assign(plan.ops, plan.ops + plan.n_ops);
  g.input = plan.input;
  g.output = plan.output;
  g.arena_len = plan.arena_len;
  g.shape = plan.shape;
  g.roffs.resize(size_t(plan.n_bufs));
  for (int32_t b = 0; b < plan.n_bufs; ++b) g.roffs[size_t(b)] = plan.offs[b] - plan.offs[root_of(g, b)];
  return build_schedule(plan, schedule_hooks(g), std::getenv("MAXIM_NO_FUSE") == nullptr);
}

int64_t len_of(const mx_buf& b) { return b.c * b.h * b.w; }

// After a synchronisation: a tensor-core kernel that gave up waiting on its
// own pipeline leaves a nonzero code in the status word. Report and clear it.
void check_status(mx_gpu& g) {
  int code = 0;
  MX_CUDA(cudaMemcpy(&code, g.status, sizeof(int), cudaMemcpyDeviceToHost));
  if (code) {
    MX_CUDA(cudaMemset(g.status, 0, sizeof(int)));
    throw Error(fmt("a tensor-core kernel gave up waiting on its pipeline (code 0x%x); its output is invalid", code),
                MX_E_DEVICE);
  }
}

// Every weight an op names must be present with exactly the length the op's
// layout needs; a plan built without a checkpoint (empty blobs) is refused
// here rather than read out of bounds.
// The converted-weights cache file: every layout the executor derived from
// the plan's weights (tensor-core tap-major orders, TF32 hi/lo halves,
// transposes), so a later executor for the same checkpoint, at any image
// size, uploads them instead of deriving them again. Little-endian:
//   "MXWCACHE", u32 format version, u32 entry count, then per entry
//   i32 weight id, i32 layout tag, u64 source-blob hash, i64 source length
//   (floats), i64 layout length (floats), the layout's floats.
// An entry is used only when the plan's blob for that weight id has the
// recorded length and hash; anything else is derived afresh. The version
// changes whenever a layout's definition changes, and a file of another
// version is ignored as a whole.
constexpr char kWcMagic[8] = {'M', 'X', 'W', 'C', 'A', 'C', 'H', 'E'};
constexpr uint32_t kWcVersion = 1;

// Maps the whole file into `map` and indexes it; the entries point into the
// mapping.
std::map<std::pair<int32_t, int>, WcEntry> load_weight_cache(const std::string& path, FileMap& map) {
  std::map<std::pair<int32_t, int>, WcEntry> m;
  const int fd = open(path.c_str(), O_RDONLY | O_CLOEXEC);
  if (fd < 0) {
    if (errno == ENOENT) return m;  // no cache yet: everything is derived, then saved
    throw Error(path + ": " + strerror(errno), MX_E_IO);
  }
  struct stat st;
  if (fstat(fd, &st) != 0) {
    close(fd);
    throw Error(path + ": " + strerror(errno), MX_E_IO);
  }
  const size_t size = size_t(st.st_size);
  if (size > 0) {
    void* p = mmap(nullptr, size, PROT_READ, MAP_PRIVATE | MAP_POPULATE, fd, 0);
    if (p == MAP_FAILED) {
      close(fd);
      throw Error(path + ": " + strerror(errno), MX_E_IO);
    }
    map.p = static_cast<const char*>(p);
    map.n = size;
  }
  close(fd);
  size_t at = 0;
  auto rd = [&](void* p, size_t n) {
    if (n > size - at) throw Error(path + ": truncated converted-weights cache", MX_E_IO);
    memcpy(p, map.p + at, n);
    at += n;
  };
  char magic[8];
  uint32_t version = 0, count = 0;
  rd(magic, 8);
  if (memcmp(magic, kWcMagic, 8) != 0) throw Error(path + ": not a converted-weights cache", MX_E_IO);
  rd(&version, 4);
  if (version != kWcVersion) return m;  // another layout definition: derive everything again
  rd(&count, 4);
  for (uint32_t i = 0; i < count; ++i) {
    int32_t id = 0, tag = 0;
    WcEntry e;
    rd(&id, 4);
    rd(&tag, 4);
    rd(&e.src_hash, 8);
    rd(&e.src_len, 8);
    rd(&e.len, 8);
    if (id < 0 || e.len < 0 || e.len > (int64_t(1) << 31) || e.src_len < 0 || size_t(e.len) * 4 > size - at)
      throw Error(path + ": corrupt converted-weights cache entry", MX_E_IO);
    e.data = reinterpret_cast<const float*>(map.p + at);  // 4-byte aligned: the header and entry heads are
    at += size_t(e.len) * 4;
    m[std::make_pair(id, int(tag))] = e;
  }
  return m;
}

// Every derived layout of this handle, read back from its weight pool, into
// `path` (written beside it under a temporary name, then renamed over it).
void save_weight_cache(mx_gpu& g, const std::string& path) {
  if (g.wbytes.empty()) throw Error("weight cache: this executor derived no weight layouts");
  if (!g.wc_track)
    throw Error("weight cache: build the executor with mx_gpu_new_cached to save its layouts (the source weights' "
                "hashes are taken only then)");
  const std::string tmp = path + fmt(".tmp%d", int(getpid()));
  FILE* f = fopen(tmp.c_str(), "wb");
  if (!f) throw Error(tmp + ": " + strerror(errno), MX_E_IO);
  bool ok = true;
  auto wr = [&](const void* p, size_t n) { ok = ok && fwrite(p, 1, n, f) == n; };
  const uint32_t n = uint32_t(g.wbytes.size());
  wr(kWcMagic, 8);
  wr(&kWcVersion, 4);
  wr(&n, 4);
  std::vector<float> buf;
  try {
    for (const auto& kv : g.wbytes) {
      const int32_t id = kv.first.first, tag = kv.first.second;
      const int64_t off = g.wcache.at(kv.first), len = kv.second / 4;
      auto h = g.wc_hash.find(id);
      if (h == g.wc_hash.end()) throw Error(fmt("weight cache: weight %d was never hashed", id));
      const int64_t src_len = g.wsrc_len.at(id);
      buf.resize(size_t(len));
      MX_CUDA(cudaMemcpy(buf.data(), g.pool.dev + off, size_t(kv.second), cudaMemcpyDeviceToHost));
      wr(&id, 4);
      wr(&tag, 4);
      wr(&h->second, 8);
      wr(&src_len, 8);
      wr(&len, 8);
      wr(buf.data(), size_t(kv.second));
    }
  } catch (...) {
    fclose(f);
    unlink(tmp.c_str());
    throw;
  }
  ok = (fclose(f) == 0) && ok;
  if (!ok || rename(tmp.c_str(), path.c_str()) != 0) {
    unlink(tmp.c_str());
    throw Error(path + ": could not write the converted-weights cache", MX_E_IO);
  }
}

void validate_weights(const mx_plan& plan) {
  auto need = [&](int32_t oi, int32_t id, int64_t n, const char* what) {
    if (id < 0) return;
    if (id >= plan.n_weights)
      throw Error(fmt("op %d: %s names weight %d, past the plan's %d weights", oi, what, id, plan.n_weights));
    if (plan.weight_lens[id] != n || (n > 0 && !plan.weights[id]))
      throw Error(fmt("op %d: %s (weight %d) holds %lld values, the op needs %lld - a plan built without a "
                      "checkpoint cannot run",
                      oi, what, id, (long long)plan.weight_lens[id], (long long)n));
  };
  for (int32_t i = 0; i < plan.n_ops; ++i) {
    const mx_op& o = plan.ops[i];
    switch (o.kind) {
      case MX_OP_CHAN_LN:
        need(i, o.scale, o.c, "LayerNorm scale");
        need(i, o.bias, o.c, "LayerNorm bias");
        break;
      case MX_OP_CONV1X1:
        need(i, o.w, int64_t(o.c_in) * o.c_out, "kernel");
        need(i, o.bias, o.c_out, "bias");
        break;
      case MX_OP_CONV3X3:
        need(i, o.w, int64_t(o.c_in) * o.c_out * 9, "kernel");
        need(i, o.bias, o.c_out, "bias");
        break;
      case MX_OP_CONV4X4S2:
        need(i, o.w, int64_t(o.c_in) * o.c_out * 16, "kernel");
        need(i, o.bias, o.c_out, "bias");
        break;
      case MX_OP_CONVT2X2:
        need(i, o.w, int64_t(o.c_in) * o.c_out * 4, "kernel");
        need(i, o.bias, o.c_out, "bias");
        break;
      case MX_OP_GATE_MM: {
        int64_t n = o.mode == 0 ? o.outer : o.inner;
        need(i, o.w, n * n, "gating kernel");
        need(i, o.bias, n, "gating bias");
        break;
      }
      default:
        break;
    }
  }
}

// ------------------------------------------------- plan-layout read-back
// The reference's executor keeps every buffer at the plan's offset in
// [c][h][w] order, and its callers read that arena back directly
// (`Gpu::read_into` / `read_arena`, src/exec_gpu.rs:284-303; `--dump`,
// src/main.rs:494-499). This executor keeps its buffers NHWC, and a scheduled
// pass packs them at its own offsets. The read-back below rebuilds the
// plan's view: the op-by-op walk (at the plan's offsets) provides the values,
// and every storage root is transposed to [c][h][w] into its plan region,
// later writers over earlier ones.

// Storage roots in the order of their last write by the plan's ops (the
// input, written before the first op, comes first).
const std::vector<int32_t>& write_order(mx_gpu& g) {
  if (!g.write_order.empty()) return g.write_order;
  const size_t nb = g.offs.size();  // the plan's buffers (the schedule's extras are not in the plan's arena)
  std::vector<int64_t> last(nb, INT64_MIN);
  last[size_t(root_of(g, g.input))] = -1;
  for (size_t i = 0; i < g.ops.size(); ++i) {
    const mx_op& o = g.ops[i];
    if (o.dst >= 0) last[size_t(root_of(g, o.dst))] = int64_t(i);
    if (o.kind == MX_OP_RESIZE && o.tmp >= 0) last[size_t(root_of(g, o.tmp))] = int64_t(i);
  }
  std::vector<int32_t> roots;
  for (size_t b = 0; b < nb; ++b)
    if (last[b] != INT64_MIN) roots.push_back(int32_t(b));
  std::stable_sort(roots.begin(), roots.end(), [&](int32_t a, int32_t b) { return last[size_t(a)] < last[size_t(b)]; });
  g.write_order = std::move(roots);
  return g.write_order;
}

// Put the op-by-op walk's state in the arena. After a scheduled pass the
// input is still staged, so the walk is replayed from it (bit-identical to
// the pass: every value is computed by the same operations in the same order).
void hold_walk(mx_gpu& g) {
  if (g.holds == mx_gpu::HOLDS_WALK) return;
  if (g.holds == mx_gpu::HOLDS_NOTHING) throw Error("the arena holds nothing yet: run a pass or begin a walk first");
  for (size_t i = 0; i + 1 < g.steps.size(); ++i) g.steps[i].run(g.stream);  // input transpose, every op
  check_launch();
  MX_CUDA(cudaStreamSynchronize(g.stream));
  check_status(g);
  g.holds = mx_gpu::HOLDS_WALK;
}

// Elements [off, off + len) of the arena in the plan's layout, into host
// memory. Regions no plan buffer wrote read as zero. A buffer still live at
// the end of the plan (its output, and every named activation of a plan built
// with dumps) reads exactly; the stale remains of buffers that died earlier
// are not reproduced (the reference leaves whatever was last written there).
void read_plan_layout(mx_gpu& g, int64_t off, int64_t len, float* out) {
  if (off < 0 || len < 0 || off + len > g.arena_len) throw Error("read: the range runs past the arena");
  if (len == 0) return;
  const int64_t oo = g.offs[size_t(g.output)], on = len_of(g.bufs[size_t(g.output)]);
  if (g.holds == mx_gpu::HOLDS_PASS && off >= oo && off + len <= oo + on) {
    // The pass's output transpose already left the output in [c][h][w].
    MX_CUDA(cudaMemcpyAsync(out, g.io_out + (off - oo), size_t(len) * 4, cudaMemcpyDeviceToHost, g.stream));
    MX_CUDA(cudaStreamSynchronize(g.stream));
    return;
  }
  hold_walk(g);
  memset(out, 0, size_t(len) * 4);
  const std::vector<int32_t>& order = write_order(g);
  std::vector<std::pair<int64_t, int64_t>> covered;  // sorted, disjoint
  for (size_t k = order.size(); k-- > 0;) {
    const int32_t r = order[k];
    const mx_buf& b = g.bufs[size_t(r)];
    const int64_t r0 = g.offs[size_t(r)], rn = len_of(b);
    const int64_t lo = std::max(off, r0), hi = std::min(off + len, r0 + rn);
    if (lo >= hi) continue;
    std::vector<std::pair<int64_t, int64_t>> vis;  // [lo, hi) less what later writers cover
    int64_t a = lo;
    for (const auto& c : covered) {
      if (c.second <= a) continue;
      if (c.first >= hi) break;
      if (c.first > a) vis.push_back({a, c.first});
      a = std::max(a, c.second);
      if (a >= hi) break;
    }
    if (a < hi) vis.push_back({a, hi});
    if (vis.empty()) continue;
    if (g.readback_len < rn) {
      cudaFree(g.readback);
      g.readback = nullptr;
      g.readback_len = 0;
      MX_CUDA(cudaMalloc(&g.readback, size_t(rn) * 4));
      g.readback_len = rn;
    }
    const int64_t npix = b.h * b.w;
    nhwc_to_nchw_kernel<<<blocks_for(npix * b.c, TPB), TPB, 0, g.stream>>>(npix, int(b.c), g.arena + r0, b.c,
                                                                           g.readback);
    check_launch();
    for (const auto& v : vis)
      MX_CUDA(cudaMemcpyAsync(out + (v.first - off), g.readback + (v.first - r0), size_t(v.second - v.first) * 4,
                              cudaMemcpyDeviceToHost, g.stream));
    MX_CUDA(cudaStreamSynchronize(g.stream));
    covered.push_back({lo, hi});
    std::sort(covered.begin(), covered.end());
    std::vector<std::pair<int64_t, int64_t>> merged;
    for (const auto& c : covered) {
      if (!merged.empty() && c.first <= merged.back().second)
        merged.back().second = std::max(merged.back().second, c.second);
      else
        merged.push_back(c);
    }
    covered.swap(merged);
  }
}

}  // namespace

const char* describe_kind(int k) {
  static const char* names[] = {"copy", "add", "mul", "gate", "gelu", "lrelu", "sigmoid", "chanln", "chanmean",
                                "chanscale", "conv1x1", "conv3x3", "convdown", "convt", "gatemm", "blockperm",
                                "resize", "down"};
  return (k >= 0 && k < MX_OP_KINDS) ? names[k] : "?";
}

}  // namespace mx

using namespace mx;

extern "C" {

int mx_driver_ready(void) {
  return guard([&] {
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) throw Error(std::string("cuda: ") + cudaGetErrorString(e), MX_E_NO_DEVICE);
    if (n == 0) throw Error("cuda: no CUDA device is visible", MX_E_NO_DEVICE);
  });
}

int mx_device_count(int* count) {
  return guard([&] {
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) n = 0;
    if (count) *count = n;
    if (e != cudaSuccess) throw Error(std::string("cuda: ") + cudaGetErrorString(e), MX_E_NO_DEVICE);
  });
}

int mx_gpu_new(int device, const mx_plan* plan, mx_gpu** out) { return mx_gpu_new_budget(device, plan, 0, out); }

int mx_gpu_new_budget(int device, const mx_plan* plan, int64_t budget_bytes, mx_gpu** out) {
  return mx_gpu_new_cached(device, plan, budget_bytes, nullptr, out);
}

int mx_gpu_new_cached(int device, const mx_plan* plan, int64_t budget_bytes, const char* cache_path, mx_gpu** out) {
  std::unique_ptr<mx_gpu> g;
  int rc = guard([&] {
    if (budget_bytes < 0) throw Error("mx_gpu_new_budget: negative budget");
    if (!plan || !out) throw Error("mx_gpu_new: null argument");
    if (plan->input < 0 || plan->output < 0 || plan->n_ops <= 0) throw Error("mx_gpu_new: empty plan");
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0)
      throw Error("cuda: no CUDA device is visible", MX_E_NO_DEVICE);
    if (device < 0 || device >= ndev) throw Error(fmt("cuda: device %d does not exist (%d visible)", device, ndev));
    DevicePin pin(device);
    g = std::make_unique<mx_gpu>();
    g->device = device;
    validate_weights(*plan);
    g->use_umma = std::getenv("MAXIM_NO_UMMA") == nullptr;
    g->building = plan;
    g->wc_track = cache_path != nullptr;
    auto now = [] { return std::chrono::steady_clock::now(); };
    auto secs = [](std::chrono::steady_clock::time_point a, std::chrono::steady_clock::time_point b) {
      return std::chrono::duration<double>(b - a).count();
    };
    auto t0 = now();
    if (cache_path) g->wc_loaded = load_weight_cache(cache_path, g->wc_file);
    auto t1 = now();
    g->t_cache_read = secs(t0, t1);
    const Schedule S = plan_schedule(*g, *plan);

    // The op-by-op walk, at the plan's offsets.
    g->step_of_op.assign(size_t(plan->n_ops), -1);
    for (int32_t i = 0; i < plan->n_ops; ++i) {
      g->step_of_op[size_t(i)] = int(g->steps.size()) + 1;  // after the input transpose
      g->steps.push_back(make_step(*g, *plan, plan->ops[i], i, &g->offs, nullptr));
    }
    add_boundary_steps(*g, g->steps, &g->offs);

    // The scheduled pass, at its own offsets, over the plan's buffers and the
    // ones the schedule adds (LayerNorm statistics).
    for (const mx_buf& b : S.extra) {
      g->bufs.push_back(b);
      g->alias_parent.push_back(-1);
      g->roffs.push_back(0);
    }
    g->foffs = S.offs;
    g->merged_into = S.merged_into;
    g->farena_len = S.arena_len;
    g->perms_dropped = S.perms_dropped;
    g->ops_fused = S.ops_fused;
    g->primary_of.assign(size_t(plan->n_ops), -1);
    g->sched_flags.assign(size_t(plan->n_ops), 0);
    for (const SchedStep& ss : S.steps) {
      g->fsteps.push_back(make_step(*g, *plan, ss.o, ss.op, &g->foffs, &ss));
      for (int32_t c : ss.covers) g->primary_of[size_t(c)] = ss.op;
      g->sched_flags[size_t(ss.op)] = (ss.stats_only ? MX_SCHED_STATS_ONLY : 0) |
                                      (ss.ln_stats >= 0 ? MX_SCHED_LN_ON_LOAD : 0);
      if (ss.ln_out_op >= 0)
        g->sched_flags[size_t(ss.ln_out_op)] |= MX_SCHED_LN_IN_EPILOGUE | (ss.ln_out_only ? MX_SCHED_LN_INPUT_UNSTORED : 0);
    }
    add_boundary_steps(*g, g->fsteps, &g->foffs);
    for (auto& st : g->fsteps) g->kernels += st.kernels;
    g->building = nullptr;
    g->wc_loaded.clear();
    g->wc_file.reset();
    auto t2 = now();
    g->t_steps = secs(t1, t2);

    // Size the pass before allocating it, and refuse it with the numbers
    // (src/exec_gpu.rs:96-146). One arena serves both walks.
    size_t free_b = 0, total_b = 0;
    MX_CUDA(cudaMemGetInfo(&free_b, &total_b));
    const bool budgeted = budget_bytes > 0 && size_t(budget_bytes) < free_b;
    if (budgeted) free_b = size_t(budget_bytes);
    int64_t arena_bytes = std::max(plan->arena_len, g->farena_len) * 4;
    int64_t io_bytes = (len_of(g->bufs[size_t(g->input)]) + len_of(g->bufs[size_t(g->output)])) * 4;
    int64_t need = arena_bytes + int64_t(g->pool.size()) + io_bytes + g->scratch_len * 4;
    if (need > int64_t(free_b))
      throw Error(fmt("not enough device memory for a %lldx%lld pass\n"
                      "maxim: the arena needs %lld MiB and the weights %lld MiB; %lld MiB is %s\n"
                      "maxim: the arena is exact - the larger of the plan's own packed size and the executor's "
                      "schedule's, not an estimate - so this is a hard limit, not a guess",
                      (long long)plan->shape.w, (long long)plan->shape.h, (long long)(arena_bytes >> 20),
                      (long long)(g->pool.size() >> 20), (long long)(free_b >> 20),
                      budgeted ? "the budget" : "free"),
                  MX_E_OOM);
    // The vectorised kernels index with 32 bits.
    for (const mx_buf& b : g->bufs)
      if (len_of(b) >= (int64_t(1) << 31))
        throw Error(fmt("a %lldx%lldx%lld activation has 2^31 or more elements; images this large are not supported",
                        (long long)b.c, (long long)b.h, (long long)b.w));
    MX_CUDA(cudaStreamCreateWithFlags(&g->stream, cudaStreamNonBlocking));
    cudaError_t e = cudaMalloc(&g->arena, size_t(arena_bytes > 0 ? arena_bytes : 4));
    if (e != cudaSuccess)
      throw Error(fmt("the arena for %lldx%lld (%lld MiB) did not fit after all, with %lld MiB free: %s",
                      (long long)plan->shape.w, (long long)plan->shape.h, (long long)(arena_bytes >> 20),
                      (long long)(free_b >> 20), cudaGetErrorString(e)),
                  MX_E_OOM);
    MX_CUDA(cudaMalloc(&g->pool.dev, std::max<size_t>(g->pool.size(), 256)));
    MX_CUDA(cudaMemcpy(g->pool.dev, g->pool.host, g->pool.size(), cudaMemcpyHostToDevice));
    g->pool.drop_host();
    MX_CUDA(cudaMalloc(&g->io_in, size_t(len_of(g->bufs[size_t(g->input)]) * 4)));
    MX_CUDA(cudaMalloc(&g->io_out, size_t(len_of(g->bufs[size_t(g->output)]) * 4)));
    if (g->scratch_len > 0) MX_CUDA(cudaMalloc(&g->scratch, size_t(g->scratch_len) * 4));
    MX_CUDA(cudaMalloc(&g->status, sizeof(int)));
    MX_CUDA(cudaMemset(g->status, 0, sizeof(int)));
    cudaDeviceProp prop;
    MX_CUDA(cudaGetDeviceProperties(&prop, device));
    g->name = prop.name;
    g->sms = prop.multiProcessorCount;
    if (g->umma_ops) {
      if (prop.major != 10)
        throw Error(fmt("%s is compute capability %d.%d; this build's tensor-core kernels are sm_100a only",
                        prop.name, prop.major, prop.minor),
                    MX_E_NO_DEVICE);
      umma_attrs_once();
    }
    for (auto& st : g->steps)
      if (st.prepare) st.prepare();
    for (auto& st : g->fsteps)
      if (st.prepare) st.prepare();
    auto t3 = now();
    g->t_device = secs(t2, t3);
    // Save what had to be derived, so the next executor for these weights
    // finds it. A cache that cannot be written does not stop this one.
    if (cache_path && g->wc_converted > 0) {
      try {
        save_weight_cache(*g, cache_path);
        g->wc_saved = 1;
      } catch (const Error&) {
        g->wc_saved = -1;
      }
    }
    g->t_cache_write = secs(t3, now());
    *out = g.release();
  });
  if (rc != MX_OK && g) mx_gpu_free(g.release());
  return rc;
}

int mx_gpu_save_weight_cache(mx_gpu* g, const char* path) {
  return guard([&] {
    if (!g || !path) throw Error("mx_gpu_save_weight_cache: null argument");
    DevicePin pin(g->device);
    save_weight_cache(*g, path);
  });
}

int mx_gpu_build_info(mx_gpu* g, mx_build_info* out) {
  return guard([&] {
    if (!g || !out) throw Error("mx_gpu_build_info: null argument");
    memset(out, 0, sizeof(*out));
    out->layouts_loaded = g->wc_hits;
    out->layouts_derived = g->wc_converted;
    out->cache_saved = g->wc_saved;
    out->seconds_cache_read = g->t_cache_read;
    out->seconds_steps = g->t_steps;
    out->seconds_device = g->t_device;
    out->seconds_cache_write = g->t_cache_write;
  });
}

void mx_gpu_free(mx_gpu* g) {
  if (!g) return;
  cudaSetDevice(g->device);
  if (g->stream) cudaStreamSynchronize(g->stream);
  if (g->graph_exec) cudaGraphExecDestroy(g->graph_exec);
  if (g->graph) cudaGraphDestroy(g->graph);
  cudaFree(g->arena);
  cudaFree(g->pool.dev);
  cudaFree(g->io_in);
  cudaFree(g->io_out);
  cudaFree(g->status);
  cudaFree(g->scratch);
  cudaFree(g->readback);
  cudaFree(g->rgb_in);
  cudaFree(g->rgb_out);
  if (g->stream) cudaStreamDestroy(g->stream);
  delete g;
}

int mx_gpu_upload_input(mx_gpu* g, const float* input) {
  return guard([&] {
    if (!g || !input) throw Error("mx_gpu_upload_input: null argument");
    DevicePin pin(g->device);
    MX_CUDA(cudaMemcpyAsync(g->io_in, input, size_t(len_of(g->bufs[size_t(g->input)]) * 4), cudaMemcpyHostToDevice,
                            g->stream));
  });
}

int mx_gpu_upload_input_device(mx_gpu* g, const float* dev_input) {
  return guard([&] {
    if (!g || !dev_input) throw Error("mx_gpu_upload_input_device: null argument");
    DevicePin pin(g->device);
    MX_CUDA(cudaMemcpyAsync(g->io_in, dev_input, size_t(len_of(g->bufs[size_t(g->input)]) * 4),
                            cudaMemcpyDeviceToDevice, g->stream));
  });
}

int mx_gpu_download_output_device(mx_gpu* g, float* dev_output) {
  return guard([&] {
    if (!g || !dev_output) throw Error("mx_gpu_download_output_device: null argument");
    DevicePin pin(g->device);
    MX_CUDA(cudaMemcpyAsync(dev_output, g->io_out, size_t(len_of(g->bufs[size_t(g->output)]) * 4),
                            cudaMemcpyDeviceToDevice, g->stream));
  });
}

int mx_gpu_stream(mx_gpu* g, void** stream) {
  return guard([&] {
    if (!g || !stream) throw Error("mx_gpu_stream: null argument");
    *stream = static_cast<void*>(g->stream);
  });
}

int mx_gpu_enqueue(mx_gpu* g) {
  return guard([&] {
    if (!g) throw Error("mx_gpu_enqueue: null handle");
    DevicePin pin(g->device);
    if (g->timeline_on) {
      // One event before every step and one after the last, one sync at the
      // end (src/exec_gpu.rs:231-265).
      size_t n = g->fsteps.size();
      std::vector<cudaEvent_t> ev(n + 1);
      for (auto& e : ev) MX_CUDA(cudaEventCreate(&e));
      for (size_t i = 0; i < n; ++i) {
        MX_CUDA(cudaEventRecord(ev[i], g->stream));
        g->fsteps[i].run(g->stream);
      }
      MX_CUDA(cudaEventRecord(ev[n], g->stream));
      check_launch();
      MX_CUDA(cudaEventSynchronize(ev[n]));
      check_status(*g);
      g->timeline_ms.assign(g->ops.size(), 0.0f);
      g->timeline_kernels.assign(g->ops.size(), 0);
      g->timeline_total = 0.0f;
      for (size_t i = 0; i < n; ++i) {
        float ms = 0.0f;
        MX_CUDA(cudaEventElapsedTime(&ms, ev[i], ev[i + 1]));
        g->timeline_total += ms;
        int op = g->fsteps[i].op;  // a fused step's time goes to its primary op
        if (op >= 0) {
          g->timeline_ms[size_t(op)] += ms;
          g->timeline_kernels[size_t(op)] += g->fsteps[i].kernels;
        }
      }
      for (auto& e : ev) cudaEventDestroy(e);
      g->holds = mx_gpu::HOLDS_PASS;
      return;
    }
    capture_graph(*g);
    MX_CUDA(cudaGraphLaunch(g->graph_exec, g->stream));
    g->holds = mx_gpu::HOLDS_PASS;
  });
}

int mx_gpu_download_output(mx_gpu* g, float* output) {
  return guard([&] {
    if (!g || !output) throw Error("mx_gpu_download_output: null argument");
    DevicePin pin(g->device);
    MX_CUDA(cudaMemcpyAsync(output, g->io_out, size_t(len_of(g->bufs[size_t(g->output)]) * 4),
                            cudaMemcpyDeviceToHost, g->stream));
  });
}

int mx_gpu_sync(mx_gpu* g) {
  return guard([&] {
    if (!g) throw Error("mx_gpu_sync: null handle");
    DevicePin pin(g->device);
    MX_CUDA(cudaStreamSynchronize(g->stream));
    check_status(*g);
  });
}

int mx_gpu_poll(mx_gpu* g) {
  return guard([&] {
    if (!g) throw Error("mx_gpu_poll: null handle");
    DevicePin pin(g->device);
    check_status(*g);  // a plain copy: it does not wait for the handle's (non-blocking) stream
  });
}

int mx_gpu_run(mx_gpu* g, const float* input, float* output) {
  int rc = mx_gpu_upload_input(g, input);
  if (rc == MX_OK) rc = mx_gpu_enqueue(g);
  if (rc == MX_OK) rc = mx_gpu_download_output(g, output);
  if (rc == MX_OK) rc = mx_gpu_sync(g);
  return rc;
}

int mx_gpu_upload_rgb8(mx_gpu* g, const uint8_t* rgb, int32_t h, int32_t w, int32_t factor) {
  return guard([&] {
    if (!g || !rgb) throw Error("mx_gpu_upload_rgb8: null argument");
    if (h < 2 || w < 2 || factor <= 0)
      throw Error(fmt("mx_gpu_upload_rgb8: a %dx%d image (factor %d); reflection needs at least 2 pixels a side", w,
                      h, factor));
    const PadGeometry pg = pad_geometry(h, w, factor);
    const mx_buf& in = g->bufs[size_t(g->input)];
    if (in.c != 3 || pg.h != in.h || pg.w != in.w)
      throw Error(fmt("mx_gpu_upload_rgb8: a %dx%d image pads to %lldx%lld, but this executor's plan takes a "
                      "%lldx%lld input",
                      w, h, (long long)pg.w, (long long)pg.h, (long long)in.w, (long long)in.h));
    DevicePin pin(g->device);
    // The original image is never larger than the padded one.
    const size_t cap = size_t(in.h * in.w * 3);
    if (!g->rgb_in) MX_CUDA(cudaMalloc(&g->rgb_in, cap));
    if (!g->rgb_out) MX_CUDA(cudaMalloc(&g->rgb_out, cap));
    MX_CUDA(cudaMemcpyAsync(g->rgb_in, rgb, size_t(h) * size_t(w) * 3, cudaMemcpyHostToDevice, g->stream));
    const int64_t n = in.h * in.w;
    const unsigned grid = std::min<unsigned>(blocks_for(n, 256), unsigned(g->sms) * 8);
    rgb8_to_padded_kernel<<<grid, 256, 0, g->stream>>>(g->rgb_in, h, w, int(pg.even_h), int(pg.even_w),
                                                        int(pg.top), int(pg.left), int(in.h), int(in.w), g->io_in);
    check_launch();
    g->rgb_h = h, g->rgb_w = w, g->rgb_even_h = int32_t(pg.even_h), g->rgb_even_w = int32_t(pg.even_w);
  });
}

int mx_gpu_download_rgb8(mx_gpu* g, uint8_t* out_rgb) {
  return guard([&] {
    if (!g || !out_rgb) throw Error("mx_gpu_download_rgb8: null argument");
    if (!g->rgb_in) throw Error("mx_gpu_download_rgb8: no image was uploaded with mx_gpu_upload_rgb8");
    const mx_buf& ob = g->bufs[size_t(g->output)];
    const int64_t hs = ob.h / 2 - g->rgb_even_h / 2, ws = ob.w / 2 - g->rgb_even_w / 2;
    if (ob.c != 3 || hs < 0 || ws < 0 || hs + g->rgb_h > ob.h || ws + g->rgb_w > ob.w)
      throw Error("mx_gpu_download_rgb8: the crop does not fit inside the prediction");
    DevicePin pin(g->device);
    const int64_t n = int64_t(g->rgb_h) * g->rgb_w;
    const unsigned grid = std::min<unsigned>(blocks_for(n, 256), unsigned(g->sms) * 8);
    crop_to_rgb8_kernel<<<grid, 256, 0, g->stream>>>(g->io_out, int(ob.h), int(ob.w), int(hs), int(ws), g->rgb_h,
                                                      g->rgb_w, g->rgb_out);
    check_launch();
    MX_CUDA(cudaMemcpyAsync(out_rgb, g->rgb_out, size_t(n) * 3, cudaMemcpyDeviceToHost, g->stream));
  });
}

int mx_gpu_run_rgb8(mx_gpu* g, const uint8_t* rgb, int32_t h, int32_t w, int32_t factor, uint8_t* out_rgb) {
  int rc = mx_gpu_upload_rgb8(g, rgb, h, w, factor);
  if (rc == MX_OK) rc = mx_gpu_enqueue(g);
  if (rc == MX_OK) rc = mx_gpu_download_rgb8(g, out_rgb);
  if (rc == MX_OK) rc = mx_gpu_sync(g);
  return rc;
}

int mx_gpu_begin(mx_gpu* g, const float* input) {
  return guard([&] {
    if (!g || !input) throw Error("mx_gpu_begin: null argument");
    DevicePin pin(g->device);
    if (std::getenv("MAXIM_POISON"))
      MX_CUDA(cudaMemsetAsync(g->arena, 0xCD, size_t(g->arena_len) * 4, g->stream));
    MX_CUDA(cudaMemcpyAsync(g->io_in, input, size_t(len_of(g->bufs[size_t(g->input)]) * 4), cudaMemcpyHostToDevice,
                            g->stream));
    g->steps.front().run(g->stream);
    check_launch();
    MX_CUDA(cudaStreamSynchronize(g->stream));
    check_status(*g);
    g->holds = mx_gpu::HOLDS_WALK;
  });
}

int mx_gpu_step_op(mx_gpu* g, int32_t i) {
  return guard([&] {
    if (!g || i < 0 || size_t(i) >= g->ops.size()) throw Error("mx_gpu_step_op: op index out of range");
    if (g->holds != mx_gpu::HOLDS_WALK) throw Error("mx_gpu_step_op: begin the walk first (mx_gpu_begin)");
    DevicePin pin(g->device);
    int s = g->step_of_op[size_t(i)];
    if (s >= 0) g->steps[size_t(s)].run(g->stream);
    check_launch();
    MX_CUDA(cudaStreamSynchronize(g->stream));
    check_status(*g);
  });
}

int mx_gpu_read_buf(mx_gpu* g, int32_t id, float* out, int64_t len) {
  return guard([&] {
    if (!g || !out || id < 0 || size_t(id) >= g->offs.size()) throw Error("mx_gpu_read_buf: bad argument");
    if (len != len_of(g->bufs[size_t(id)])) throw Error("mx_gpu_read_buf: length does not match the buffer");
    DevicePin pin(g->device);
    if (g->holds == mx_gpu::HOLDS_PASS && id == g->output) {
      MX_CUDA(cudaMemcpyAsync(out, g->io_out, size_t(len) * 4, cudaMemcpyDeviceToHost, g->stream));
      MX_CUDA(cudaStreamSynchronize(g->stream));
      return;
    }
    hold_walk(*g);
    View v = view_of(*g, g->offs, id);
    float* tmp = nullptr;
    MX_CUDA(cudaMalloc(&tmp, size_t(std::max<int64_t>(len, 1)) * 4));
    nhwc_to_nchw_kernel<<<blocks_for(v.npix * v.c, TPB), TPB, 0, g->stream>>>(v.npix, int(v.c), v.ptr, v.stride, tmp);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaMemcpyAsync(out, tmp, size_t(len) * 4, cudaMemcpyDeviceToHost, g->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(g->stream);
    cudaFree(tmp);
    if (e != cudaSuccess) throw Error(std::string("read_buf: ") + cudaGetErrorString(e), MX_E_CUDA);
  });
}

int mx_gpu_read_into(mx_gpu* g, int64_t off, float* out, int64_t len) {
  return guard([&] {
    if (!g || (!out && len > 0)) throw Error("mx_gpu_read_into: null argument");
    DevicePin pin(g->device);
    read_plan_layout(*g, off, len, out);
  });
}

int mx_gpu_read_arena(mx_gpu* g, float* out, int64_t len) {
  return guard([&] {
    if (!g || !out || len != g->arena_len) throw Error("mx_gpu_read_arena: bad argument");
    DevicePin pin(g->device);
    read_plan_layout(*g, 0, len, out);
  });
}

int mx_gpu_set_timeline(mx_gpu* g, int on) {
  return guard([&] {
    if (!g) throw Error("mx_gpu_set_timeline: null handle");
    g->timeline_on = on != 0;
  });
}

int mx_gpu_timeline(mx_gpu* g, float* per_op_ms, int32_t n_ops, float* total_ms) {
  return guard([&] {
    if (!g) throw Error("mx_gpu_timeline: null handle");
    if (g->timeline_ms.empty()) throw Error("no timeline recorded: turn it on and run a pass first");
    if (per_op_ms) {
      if (size_t(n_ops) != g->ops.size()) throw Error("mx_gpu_timeline: n_ops does not match the plan");
      memcpy(per_op_ms, g->timeline_ms.data(), g->ops.size() * 4);
    }
    if (total_ms) *total_ms = g->timeline_total;
  });
}

int mx_gpu_timeline_kernels(mx_gpu* g, int32_t* kernels_per_op, int32_t n_ops) {
  return guard([&] {
    if (!g || !kernels_per_op) throw Error("mx_gpu_timeline_kernels: null argument");
    if (g->timeline_kernels.empty()) throw Error("no timeline recorded: turn it on and run a pass first");
    if (size_t(n_ops) != g->ops.size()) throw Error("mx_gpu_timeline_kernels: n_ops does not match the plan");
    memcpy(kernels_per_op, g->timeline_kernels.data(), g->ops.size() * sizeof(int32_t));
  });
}

int mx_gpu_get_stats(mx_gpu* g, mx_gpu_stats* s) {
  return guard([&] {
    if (!g || !s) throw Error("mx_gpu_get_stats: null argument");
    memset(s, 0, sizeof(*s));
    snprintf(s->device_name, sizeof(s->device_name), "%s", g->name.c_str());
    s->arena_bytes = g->arena_len * 4;
    s->weight_bytes = g->weight_bytes;
    s->pool_bytes = 0;
    s->ops = int64_t(g->ops.size());
    s->kernels = g->kernels;
    s->steps = int64_t(g->fsteps.size()) - 2;
    s->ops_fused = g->ops_fused;
    s->perms_dropped = g->perms_dropped;
    s->pass_arena_bytes = g->farena_len * 4;
  });
}

int mx_gpu_schedule(mx_gpu* g, int32_t* primary, int32_t* flags, int32_t n_ops) {
  return guard([&] {
    if (!g || !primary) throw Error("mx_gpu_schedule: null argument");
    if (size_t(n_ops) != g->ops.size()) throw Error("mx_gpu_schedule: n_ops does not match the plan");
    memcpy(primary, g->primary_of.data(), g->primary_of.size() * sizeof(int32_t));
    if (flags) memcpy(flags, g->sched_flags.data(), g->sched_flags.size() * sizeof(int32_t));
  });
}

int mx_plan_schedule(const mx_plan* plan, mx_gpu_stats* stats, int32_t* primary, int32_t* flags, int32_t n_ops) {
  return guard([&] {
    if (!plan || !stats) throw Error("mx_plan_schedule: null argument");
    if ((primary || flags) && n_ops != plan->n_ops) throw Error("mx_plan_schedule: n_ops does not match the plan");
    mx_gpu g;
    g.use_umma = std::getenv("MAXIM_NO_UMMA") == nullptr;
    const Schedule S = plan_schedule(g, *plan);
    memset(stats, 0, sizeof(*stats));
    stats->ops = plan->n_ops;
    stats->arena_bytes = plan->arena_len * 4;
    stats->steps = int64_t(S.steps.size());
    stats->ops_fused = S.ops_fused;
    stats->perms_dropped = S.perms_dropped;
    stats->pass_arena_bytes = S.arena_len * 4;
    if (primary) {
      for (int32_t i = 0; i < n_ops; ++i) primary[i] = -1;
      for (const SchedStep& ss : S.steps)
        for (int32_t c : ss.covers) primary[c] = ss.op;
    }
    if (flags) {
      for (int32_t i = 0; i < n_ops; ++i) flags[i] = 0;
      for (const SchedStep& ss : S.steps) {
        flags[ss.op] = (ss.stats_only ? MX_SCHED_STATS_ONLY : 0) | (ss.ln_stats >= 0 ? MX_SCHED_LN_ON_LOAD : 0);
        if (ss.ln_out_op >= 0)
          flags[ss.ln_out_op] |= MX_SCHED_LN_IN_EPILOGUE | (ss.ln_out_only ? MX_SCHED_LN_INPUT_UNSTORED : 0);
      }
    }
  });
}

}  // extern "C"
