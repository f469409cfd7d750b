/*
 * maxim_b200.h - the C ABI of the B200-native MAXIM forward pass.
 *
 * Two groups of entry points live here:
 *
 *   1. The GPU executor (mx_driver_ready, mx_gpu_*). This is the drop-in
 *      boundary: it replaces the reference's `exec_gpu::Gpu`
 *      (src/exec_gpu.rs:48-357) and the device glue under it (src/cuda.rs).
 *      A caller hands it a plan as a flat POD op table (mx_plan) plus host
 *      weight blobs in the plan's own layouts, and gets the same methods the
 *      Rust type has: new / run / begin / step_op / read_buf / read_into /
 *      read_arena / timeline / stats. Nothing here takes or returns a torch or
 *      CUDA type; device memory is owned by the handle.
 *
 *   2. The host contract (mx_weights_*, mx_plan_*, mx_image_*, mx_param_spec),
 *      a C++ restatement of the reference's Rust host: safetensors weights with
 *      the checkpoint-derived config (src/weights.rs, src/config.rs), the plan
 *      builder and live-range arena packer (src/model.rs), and the PNG / pad /
 *      crop pipeline (src/image.rs). A caller that already has a Plan (the Rust
 *      crate itself) only needs group 1.
 *
 * Conventions (src/lib.rs:29-56 is the reference's error type):
 *   - every function returns an int status: MX_OK (0) or a negative MX_E_*;
 *   - on failure the thread-local message is available from mx_last_error();
 *   - sizes are in elements of float (fp32) unless the name says bytes;
 *   - buffer ids, op indices and weight ids are the plan's own indices.
 */
#ifndef MAXIM_B200_H
#define MAXIM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------ status codes */
enum {
  MX_OK = 0,
  MX_E_INVALID = -1,    /* bad argument, bad shape, unsupported plan */
  MX_E_IO = -2,         /* file / PNG / safetensors problem */
  MX_E_NO_DEVICE = -3,  /* the CUDA driver or device is unavailable */
  MX_E_OOM = -4,        /* the pass does not fit in device memory */
  MX_E_CUDA = -5,       /* a CUDA call failed */
  MX_E_DEVICE = -6,     /* a kernel reported an error through its status word */
};

/* Copy the calling thread's last error message into buf (always NUL
 * terminated). Returns the full message length. */
size_t mx_last_error(char* buf, size_t len);

/* ----------------------------------------------------------- the plan (POD)
 * The op kinds of `model::Op` (src/model.rs:66-112), in the enum's order. */
enum {
  MX_OP_COPY = 0,
  MX_OP_ADD = 1,
  MX_OP_MUL = 2,
  MX_OP_GATE_APPLY = 3,
  MX_OP_GELU = 4,
  MX_OP_LRELU = 5,
  MX_OP_SIGMOID = 6,
  MX_OP_CHAN_LN = 7,
  MX_OP_CHAN_MEAN = 8,
  MX_OP_CHAN_SCALE = 9,
  MX_OP_CONV1X1 = 10,
  MX_OP_CONV3X3 = 11,
  MX_OP_CONV4X4S2 = 12,
  MX_OP_CONVT2X2 = 13,
  MX_OP_GATE_MM = 14,
  MX_OP_BLOCK_PERM = 15,
  MX_OP_RESIZE = 16,
  MX_OP_DOWN_S = 17,
  MX_OP_KINDS = 18
};

/* One op. Unused fields are -1 (ids) or 0 (sizes). Field meaning per kind
 * follows `model::Op` (src/model.rs:66-112):
 *   Copy/Add/Mul/GateApply/Gelu/Lrelu/Sigmoid: dst, src (a / u), src2 (b / v), n, slope
 *   ChanLn: dst, src, scale, bias, c, hw
 *   ChanMean: dst, src, c, hw          ChanScale: dst, src, src2 (= s), c, hw
 *   Conv1x1/Conv3x3: dst, src, w, wt, bias, c_in, c_out, h, wd
 *   Conv4x4s2: ... + pad_top, pad_left, oh, ow     ConvT2x2: dst, src, w, bias, c_in, c_out, h, wd
 *   GateMm: dst, src, w, bias, c, outer, inner, mode
 *   BlockPerm: dst, src, c, h, wd, gh, gw, fh, fw, swap, forward
 *   Resize: dst, src, tmp, c, hin, win, hout, wout
 *   DownS: dst, src, c, h, wd, stride, off, oh, ow                                  */
typedef struct mx_op {
  int32_t kind;
  int32_t dst, src, src2, tmp;
  int32_t w, wt, bias, scale;
  int64_t n;
  int32_t c, c_in, c_out, h, wd, oh, ow, pad_top, pad_left;
  int32_t outer, inner, mode;
  int32_t gh, gw, fh, fw, swap, forward;
  int32_t stride, off;
  int32_t hin, win, hout, wout;
  int64_t hw;
  float slope;
} mx_op;

/* A buffer's [c][h][w] shape (`model::BufShape`, src/model.rs:37-62). */
typedef struct mx_buf {
  int64_t c, h, w;
} mx_buf;

/* The plan as a read-only POD view (`model::Plan`, src/model.rs:1237-1272).
 * `offs` are element offsets into the arena, views already resolved;
 * `alias_parent[i]` is -1 for a buffer that owns its storage, else the buffer
 * it is a channel range of, at element delta `alias_delta[i]`. */
typedef struct mx_plan {
  int32_t n_bufs;
  const mx_buf* bufs;
  const int64_t* offs;
  const int32_t* alias_parent;
  const int64_t* alias_delta;
  int32_t n_ops;
  const mx_op* ops;
  int32_t n_weights;
  const float* const* weights; /* host blobs in the plan's layouts */
  const int64_t* weight_lens;
  int64_t arena_len;
  int32_t input, output;
  mx_buf shape; /* the padded input shape the plan was built for */
} mx_plan;

/* ================================================== 1. the GPU executor ==== */

typedef struct mx_gpu mx_gpu;

/* `exec_gpu::driver_ready` (src/exec_gpu.rs:81-83): bring the driver up. */
int mx_driver_ready(void);
/* Number of visible CUDA devices (0 when the driver is unavailable). */
int mx_device_count(int* count);

/* `Gpu::new` (src/exec_gpu.rs:96-157): size the pass, refuse it with the
 * numbers if arena + weights exceed free device memory, then make ONE arena
 * allocation and upload every weight in the kernels' layouts (resident, not
 * lazy). The plan is copied; the caller may free its view afterwards. */
int mx_gpu_new(int device, const mx_plan* plan, mx_gpu** out);
/* The same with a device-memory budget: the pass is refused, with the same
 * message, when it needs more than budget_bytes even if the device has more
 * free (a GPU shared with other work). 0 means the device's free memory. No
 * counterpart in the reference. */
int mx_gpu_new_budget(int device, const mx_plan* plan, int64_t budget_bytes, mx_gpu** out);
/* The same, with a converted-weights cache file (the weights loader's
 * on-disk format; the reference derives its layouts at every start,
 * src/weights.rs:57-211). Besides the plan's own layouts the executor derives
 * tensor-core ones from every weight (tap-major orders, TF32 hi/lo halves,
 * transposes); a cache file holds those derived layouts, each tagged with
 * the length and a 64-bit hash of the plan weight it was made from. At
 * construction every layout whose source weight is unchanged is read from
 * the file instead of derived, at any image size and in either walk; the
 * rest are derived, and when anything was derived the file is (re)written
 * (under a temporary name, then renamed). A missing file is an empty cache;
 * a file that is not a cache is refused (MX_E_IO); a cache of another
 * format version is ignored. Passes are bit for bit those of mx_gpu_new.
 * cache_path null is mx_gpu_new_budget. */
int mx_gpu_new_cached(int device, const mx_plan* plan, int64_t budget_bytes, const char* cache_path, mx_gpu** out);
/* Write this executor's derived layouts to a cache file now (the executor
 * must come from mx_gpu_new_cached, which records the source weights'
 * hashes). */
int mx_gpu_save_weight_cache(mx_gpu* g, const char* path);
/* How the executor was built: weight layouts `loaded` from the cache file
 * and `derived` from the plan's weights; `cache_saved` 1 when
 * mx_gpu_new_cached wrote the file, 0 when it had no reason to, -1 when
 * writing it failed; and the wall time of each phase: reading and indexing
 * the cache file, scheduling and making the steps (which derives the layouts
 * not loaded), device allocation with the weight upload and tensor maps, and
 * writing the cache. No counterpart in the reference. */
typedef struct mx_build_info {
  int64_t layouts_loaded;
  int64_t layouts_derived;
  int32_t cache_saved;
  int32_t reserved;
  double seconds_cache_read;
  double seconds_steps;
  double seconds_device;
  double seconds_cache_write;
} mx_build_info;
int mx_gpu_build_info(mx_gpu* g, mx_build_info* out);
void mx_gpu_free(mx_gpu* g);

/* `Gpu::run` (src/exec_gpu.rs:196-229): input [3][H][W] host floats in,
 * output [3][H][W] host floats out (the plan's output buffer), synchronous. */
int mx_gpu_run(mx_gpu* g, const float* input, float* output);

/* The same pass split into its parts, for callers that keep the input and
 * output on the device or overlap copies with other work: upload the input,
 * enqueue the whole op stream (one CUDA graph launch), download the output.
 * All three are asynchronous on the handle's stream; mx_gpu_sync waits. */
int mx_gpu_upload_input(mx_gpu* g, const float* input);
int mx_gpu_enqueue(mx_gpu* g);
int mx_gpu_download_output(mx_gpu* g, float* output);
int mx_gpu_sync(mx_gpu* g);
/* The status of the passes finished so far, without waiting for the stream:
 * MX_E_DEVICE when a kernel has recorded a pipeline failure (the record is
 * then cleared), else MX_OK. For callers that wait on their own events and
 * keep the next pass running meanwhile. */
int mx_gpu_poll(mx_gpu* g);
/* The same two copies from / to DEVICE memory of the handle's device (a
 * batch of images already resident in HBM): device-to-device, async. */
int mx_gpu_upload_input_device(mx_gpu* g, const float* dev_input);
int mx_gpu_download_output_device(mx_gpu* g, float* dev_output);
/* The reference CLI's whole image path (`run_gpu` between `read_png` and
 * `write_png`: src/main.rs:467-504 with src/image.rs:40-104 and 171-246) with
 * its per-pixel steps on the device. The caller passes the PNG's 8-bit
 * samples (interleaved RGB, h x w x 3 bytes, e.g. from mx_png_read_rgb8_mem)
 * and gets the restored image's 8-bit samples back (h x w x 3 bytes, the
 * original size). On the device: divide by 255, reflect to the even shape,
 * reflect-pad centred to a multiple of `factor` (the plan must be built for
 * that padded shape, mx_pad_geometry), the pass, then the centred crop,
 * clamp to 0..1 and round half up to 8 bits. Only the 8-bit images cross
 * PCIe (a quarter of the float copies each way). Results are bit for bit
 * those of mx_preprocess + mx_gpu_run + mx_crop_out + the PNG writer's
 * rounding. The first call allocates the handle's 8-bit staging (two
 * buffers of the padded size). Images the host pipeline refuses (too small
 * to reflect) are refused with the same message.
 * upload_rgb8 / download_rgb8 are the two halves (asynchronous on the
 * handle's stream, around mx_gpu_enqueue; download crops with the geometry
 * of the image last uploaded); run_rgb8 does all of it and waits. As with
 * cudaMemcpyAsync, a pinned (page-locked) host buffer given to either half
 * must stay untouched until mx_gpu_sync; a pageable one may be reused when
 * the call returns. The staging is not part of mx_gpu_new's memory budget. */
int mx_gpu_upload_rgb8(mx_gpu* g, const uint8_t* rgb, int32_t h, int32_t w, int32_t factor);
int mx_gpu_download_rgb8(mx_gpu* g, uint8_t* out_rgb);
int mx_gpu_run_rgb8(mx_gpu* g, const uint8_t* rgb, int32_t h, int32_t w, int32_t factor, uint8_t* out_rgb);
/* The handle's CUDA stream (a cudaStream_t, as an opaque pointer) so a caller
 * can order its own work or record timing events against the pass. */
int mx_gpu_stream(mx_gpu* g, void** stream);

/* `Gpu::begin` / `step_op` / `read_buf` (src/exec_gpu.rs:329-357): the
 * op-by-op walk behind `--verify-gpu`. step_op runs op `i` alone, unfused,
 * after mx_gpu_begin. read_buf returns buffer `id` in the plan's [c][h][w]
 * layout (converted from the executor's internal NHWC layout), after a walk
 * or after a pass.
 *
 * `Gpu::read_into` / `read_arena` (src/exec_gpu.rs:292-303): the arena as the
 * reference's executor leaves it - every buffer at its plan offset
 * (`mx_plan.offs`, element units) in [c][h][w] order. read_into copies `len`
 * floats starting at element `off` (run_gpu reads the output with it,
 * src/main.rs:501); read_arena copies all `arena_len` floats (`--dump`,
 * src/main.rs:494-499). Buffers still live at the end of the plan - the
 * output, and every named activation of a plan built with dumps - read
 * exactly. Reading the output after a pass is one copy; any other range after
 * a pass replays the plan op by op from the staged input first (the same
 * values), then transposes each buffer into place. Ranges no buffer wrote
 * read as zero, and the stale remains of buffers that died earlier are not
 * reproduced. */
int mx_gpu_begin(mx_gpu* g, const float* input);
int mx_gpu_step_op(mx_gpu* g, int32_t i);
int mx_gpu_read_buf(mx_gpu* g, int32_t id, float* out, int64_t len);
int mx_gpu_read_into(mx_gpu* g, int64_t off, float* out, int64_t len);
int mx_gpu_read_arena(mx_gpu* g, float* out, int64_t len);

/* `Gpu::set_timeline` / `timeline` (src/exec_gpu.rs:180-265): with the
 * timeline on, mx_gpu_run records an event around every launch group and
 * per_op_ms[i] receives op i's device time (0 for ops fused into another). */
int mx_gpu_set_timeline(mx_gpu* g, int on);
int mx_gpu_timeline(mx_gpu* g, float* per_op_ms, int32_t n_ops, float* total_ms);
/* `Timeline::kernels_per_op` (src/exec_gpu.rs:68-72): kernel launches op i
 * made in the last timed pass (a fused op's launches count to the op whose
 * step carried it out; ops fused into another read 0). */
int mx_gpu_timeline_kernels(mx_gpu* g, int32_t* kernels_per_op, int32_t n_ops);

/* `device_name` / `arena_bytes` / `weight_bytes` / `pool_bytes` /
 * `ops_launched` (src/exec_gpu.rs:160-190). `kernels` is the number of kernel
 * launches one pass enqueues. The rest describe the executor's own schedule
 * of the plan (no counterpart in the reference): `steps` scheduled steps,
 * `ops_fused` plan ops carried out inside another op's step, `perms_dropped`
 * block permutations replaced by reading the blocks in place, and
 * `pass_arena_bytes` the arena that schedule needs (the allocation holds the
 * larger of it and `arena_bytes`, the plan's own, which op-by-op stepping
 * uses). */
typedef struct mx_gpu_stats {
  char device_name[128];
  int64_t arena_bytes;
  int64_t weight_bytes;
  int64_t pool_bytes;
  int64_t ops;
  int64_t kernels;
  int64_t steps;
  int64_t ops_fused;
  int64_t perms_dropped;
  int64_t pass_arena_bytes;
} mx_gpu_stats;
int mx_gpu_get_stats(mx_gpu* g, mx_gpu_stats* s);

/* Which scheduled step carries out each plan op: primary[i] is the plan op
 * whose step runs op i (i itself when it is not fused), -1 for an op the
 * schedule removed. flags[i] (may be null): MX_SCHED_STATS_ONLY when op i, a
 * channel LayerNorm, only computes its per-pixel statistics;
 * MX_SCHED_LN_ON_LOAD when op i, a conv, normalises its input with such
 * statistics as it loads it; MX_SCHED_LN_IN_EPILOGUE when op i, a channel
 * LayerNorm, is written whole by the epilogue of the conv that produces its
 * input (primary[i]), plus MX_SCHED_LN_INPUT_UNSTORED when no other op reads
 * that input, so the epilogue stores the LayerNorm alone. n_ops must be the
 * plan's op count. No counterpart in the reference (its executor runs every
 * op as its own launch). */
enum { MX_SCHED_STATS_ONLY = 1, MX_SCHED_LN_ON_LOAD = 2, MX_SCHED_LN_IN_EPILOGUE = 4, MX_SCHED_LN_INPUT_UNSTORED = 8 };
int mx_gpu_schedule(mx_gpu* g, int32_t* primary, int32_t* flags, int32_t n_ops);

/* The same schedule worked out on the host alone, without a device: for
 * tests and tools. `stats` receives steps / ops_fused / perms_dropped /
 * pass_arena_bytes (other fields zero); `primary` and `flags` as above (may
 * be null). */
int mx_plan_schedule(const mx_plan* plan, mx_gpu_stats* stats, int32_t* primary, int32_t* flags, int32_t n_ops);

/* The per-channel mean (the CALayer squeeze) of an NHWC tensor in device
 * memory, computed without allocating anything. This entry point has no
 * counterpart in the reference.
 *
 * It is for callers that cannot call cudaMalloc: an engine that gives the GPU
 * a fixed memory budget up front, code running inside a CUDA stream capture
 * (where allocation is not allowed), or a service whose allocator forbids
 * stray allocations. The caller passes the input x (npix pixels, c channels
 * contiguous, pixel_stride floats between pixels, 16-byte aligned) and the
 * output out (c floats), both in device memory; the partial sums live in one
 * fixed 1 MiB device array inside the library (held on every GPU that loads
 * it, until the process exits) instead of in allocated scratch. The result is
 * bit for bit the executor's own channel mean of the same tensor (the same
 * partition of pixels into blocks, the same two kernels).
 * Limits: c a multiple of 4 and at most 256; npix and npix * pixel_stride
 * below 2^31. Larger sizes are rejected with MX_E_INVALID.
 * The first call on each device looks up that device's address of the array
 * (with the device current) and caches it; make that first call before any
 * stream capture. All calls share the array, so calls that overlap on the
 * GPU (unordered streams) race on it; each call overwrites every partial it
 * reads, so nothing needs clearing between calls. `stream` is a cudaStream_t
 * (null for the legacy default stream); the call is asynchronous on it. */
int mx_channel_mean_noalloc(const float* x, int64_t npix, int32_t c, int64_t pixel_stride, float* out,
                            void* stream);

/* ------------------------------------------------------ the batch runner
 * Independent images sharded round-robin over GPUs: one worker thread and
 * one executor handle (arena, weights, stream, graph) per device, and no
 * collective between them. The reference restores one image per process
 * (src/main.rs:173-458); this is the multi-GPU batch mode built on group 1,
 * with host-side failure handling:
 *   - each worker has a status (mx_batch_workers);
 *   - a device whose executor cannot be built (the pass does not fit its
 *     memory, or its budget) is left out and the batch runs on the others;
 *     mx_batch_new fails only when no device can take it;
 *   - a worker that fails on an image is retired, and the images it had not
 *     finished, the failing one included, go round-robin to the workers
 *     still standing. An image no worker could restore keeps the status of
 *     its last attempt in image_status, and mx_batch_run returns that error
 *     (with a message naming the image and the device) - it does not hang:
 *     the executors' device-side waits are bounded in time.
 * The executor is pluggable: null means this library's GPU executor (the
 * plan in `cfg`, copied per device; the caller may free it after
 * mx_batch_new). A caller-supplied executor must return from every call;
 * `open`, `run` and `close` run on the worker threads (one thread per
 * handle at a time). */
typedef struct mx_batch mx_batch;
enum { MX_WORKER_READY = 0, MX_WORKER_FAILED = 1 };
typedef struct mx_batch_worker {
  int32_t device;      /* the device the worker drives */
  int32_t state;       /* MX_WORKER_READY or MX_WORKER_FAILED */
  int32_t error_code;  /* MX_OK, or the status that retired it */
  int32_t images_done; /* images it restored in the last mx_batch_run */
  double seconds;      /* its wall time in the last mx_batch_run */
  char error[256];     /* the message behind error_code */
} mx_batch_worker;
typedef struct mx_batch_config {
  const mx_plan* plan;       /* the plan every image runs (the GPU executor's) */
  int64_t device_mem_budget; /* bytes a device's pass may use; 0: its free memory */
} mx_batch_config;
typedef struct mx_batch_executor {
  void* ctx;
  int (*open)(void* ctx, int32_t device, void** handle);
  int (*run)(void* ctx, void* handle, const float* input, float* output);
  void (*close)(void* ctx, void* handle);
} mx_batch_executor;
int mx_batch_new(const mx_batch_config* cfg, const int32_t* devices, int32_t n_devices,
                 const mx_batch_executor* executor, mx_batch** out);
/* Restore n_images: inputs[i] ([3][H][W] host floats, the plan's input) to
 * outputs[i] (the plan's output shape); image i goes to the (i mod R)-th of
 * the R ready workers. image_status (may be null) receives each image's
 * MX_OK / MX_E_*. Synchronous. */
int mx_batch_run(mx_batch* b, int32_t n_images, const float* const* inputs, float* const* outputs,
                 int32_t* image_status);
/* PNG files in, PNG files out, over the device-side image path
 * (mx_gpu_run_rgb8): in_paths[i] is read, decoded, padded on the GPU,
 * restored, cropped and rounded on the GPU, and written to out_paths[i] as
 * an RGB PNG. Every image must pad (by `factor`) to the plan's input shape.
 * Each worker reads and decodes its next image while the GPU runs the
 * current one (two in flight), and encoder threads of its own (the host
 * threads left over, shared out: one to four a worker) compress and write
 * the finished ones at zlib level 1, so the PNG work overlaps the passes. An
 * image that cannot be read, decoded, padded to the plan's shape or written
 * fails alone (its image_status); a device failure retires the worker and
 * its unfinished images go to the others, as in mx_batch_run. Needs the
 * built-in GPU executor. Synchronous. */
int mx_batch_run_png(mx_batch* b, int32_t n_images, const char* const* in_paths, const char* const* out_paths,
                     int32_t factor, int32_t* image_status);
int32_t mx_batch_worker_count(const mx_batch* b);
int mx_batch_workers(const mx_batch* b, mx_batch_worker* out, int32_t n);
void mx_batch_free(mx_batch* b);

/* ================================================= 2. the host contract ==== */

typedef struct mx_weights mx_weights;
typedef struct mx_plan_handle mx_plan_handle;

/* `Weights::open` + `Config::of_checkpoint` (src/weights.rs:37-41,
 * src/config.rs:71-100): the variant is derived from the file. */
int mx_weights_open(const char* path, mx_weights** out);
void mx_weights_free(mx_weights* w);
/* The variant name ("S-3", ...) the checkpoint was derived as. */
int mx_weights_variant(const mx_weights* w, char* buf, size_t len);

/* The parameter inventory a checkpoint of `variant` must hold, in the
 * builder's request order: one "name\tshape\n" line per tensor, shape as
 * comma-separated dims. `*needed` receives the full byte length.
 * Variants: "S-1".."S-3", "M-1".."M-3" (src/config.rs:34-62), and
 * "gMLP-<c>": one residual split-head multi-axis gMLP layer over a c-channel
 * input with 16x16 blocks and a 16x16 grid, the builder's own
 * `split_head_gmlp` (src/model.rs:576-603) as a plan of its own (input and
 * output [c][H][W]). A checkpoint holding that layer's tensors opens as it. */
int mx_param_spec(const char* variant, char* buf, size_t len, size_t* needed);

/* `Builder::new(..)[.without_dumps()].build(h, w)` (src/model.rs:743-891):
 * h and w are the PADDED dimensions. With dumps != 0 the named activations
 * (`Plan::dumps`) are kept live to the end of the run, as `--dump` needs. */
int mx_plan_build(const mx_weights* w, int32_t h, int32_t wd, int dumps, mx_plan_handle** out);
/* The same plan for a named variant with no checkpoint: every weight blob is
 * empty. For shape, op-count and arena queries (the reference's arena and
 * packing tests need a checkpoint only for its shapes). */
int mx_plan_build_variant(const char* variant, int32_t h, int32_t wd, int dumps, mx_plan_handle** out);
void mx_plan_free(mx_plan_handle* p);
const mx_plan* mx_plan_view(const mx_plan_handle* p);
/* Named activations: count, and the i-th name / buffer id. */
int32_t mx_plan_dump_count(const mx_plan_handle* p);
int mx_plan_dump(const mx_plan_handle* p, int32_t i, char* name, size_t len, int32_t* id);
/* A buffer's human-readable label (`Plan::labels`). */
int mx_plan_label(const mx_plan_handle* p, int32_t id, char* buf, size_t len);

/* An image, [c][h][w] floats in 0..1 (`image::Image`, src/image.rs:9-30).
 * Memory is owned by the library; free with mx_image_free. */
typedef struct mx_image {
  int32_t c, h, w;
  float* data;
} mx_image;
void mx_image_free(mx_image* img);
/* `image::read_png` / `write_png` (src/image.rs:33-104): 8-bit PNG, gray /
 * gray+alpha / RGB / RGBA read as RGB; written RGB with round-half-up. */
int mx_png_read(const char* path, mx_image* out);
int mx_png_read_mem(const uint8_t* bytes, size_t n, mx_image* out);
int mx_png_write(const char* path, const mx_image* img);
/* `image::preprocess(img, factor)` (src/image.rs:171-207): even reflect, then
 * centred reflect to a multiple of `factor`; returns the even shape too.
 * Refuses an image too small to reflect, with the reference's reasoning. */
int mx_preprocess(const mx_image* img, int32_t factor, mx_image* padded, int32_t* even_h, int32_t* even_w);
/* `image::crop_out` (src/image.rs:233-246). */
int mx_crop_out(const mx_image* pred, int32_t orig_h, int32_t orig_w, int32_t even_h, int32_t even_w,
                mx_image* out);

/* The shapes `image::preprocess` (src/image.rs:171-207) gives an h x w image,
 * without its pixels: the padded shape (what to build the plan for) and the
 * even shape (what to crop with). Refuses exactly the images preprocess
 * refuses, with the same message. */
int mx_pad_geometry(int32_t h, int32_t w, int32_t factor, int32_t* padded_h, int32_t* padded_w, int32_t* even_h,
                    int32_t* even_w);

/* The 8-bit side of `read_png_stream` / `write_png_stream`
 * (src/image.rs:40-104): the PNG's samples as decoded, interleaved RGB
 * (c = 3, h x w x 3 bytes; gray and gray+alpha expanded, alpha dropped), as
 * the device-side pipeline (mx_gpu_run_rgb8) takes them. Memory is owned by
 * the library; free with mx_image8_free. mx_png_size_mem reads the width and
 * height from the IHDR chunk alone, so a caller can size and build its plan
 * while the pixels are still being decoded. */
typedef struct mx_image8 {
  int32_t c, h, w;
  uint8_t* data;
} mx_image8;
void mx_image8_free(mx_image8* img);
int mx_png_size_mem(const uint8_t* bytes, size_t n, int32_t* h, int32_t* w);
int mx_png_read_rgb8_mem(const uint8_t* bytes, size_t n, mx_image8* out);
int mx_png_write_rgb8(const char* path, const mx_image8* img);

#ifdef __cplusplus
}
#endif
#endif /* MAXIM_B200_H */
