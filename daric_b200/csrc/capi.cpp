// Host side of the C ABI declared in include/daric_b200.h.
//
// Responsibilities: argument validation with the reference's rules
// (csrc/cache_ops/helpers.cu:94-174, copier.cpp:32-39, kernels.cu:151-161),
// building the per-call device descriptors (layers, jobs, chunks) and
// uploading them through a pinned ring, and launching the kernels on the
// caller's stream. Nothing here blocks the host except a ring slot whose
// previous use (16 calls earlier on the same device) is still running.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <sstream>
#include <string>
#include <unordered_map>
#include <vector>

#include "internal.h"

using namespace daric;

namespace {

thread_local std::string g_last_error;

template <class F>
int guarded(F&& f) {
  try {
    f();
    g_last_error.clear();
    return DARIC_OK;
  } catch (const Error& e) {
    g_last_error = e.what();
    return e.code;
  } catch (const std::exception& e) {
    g_last_error = e.what();
    return DARIC_ERR_STATE;
  }
}

std::string fmt_vec(const std::vector<int64_t>& v) {
  std::ostringstream ss;
  ss << "[";
  for (size_t i = 0; i < v.size(); ++i) ss << (i ? ", " : "") << v[i];
  ss << "]";
  return ss.str();
}

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    DARIC_CUDA(cudaGetDevice(&prev));
    if (prev != dev) DARIC_CUDA(cudaSetDevice(dev));
  }
  ~DeviceGuard() {
    int cur = -1;
    if (cudaGetDevice(&cur) == cudaSuccess && cur != prev && prev >= 0) cudaSetDevice(prev);
  }
};

// ------------------------------------------------------ per-device state --
constexpr int kRingSlots = 16;

constexpr size_t kSlotBytes = 1024 * 1024;  // pre-allocated descriptor bytes per ring slot

struct RingSlot {
  std::mutex mu;
  uint8_t* host = nullptr;
  uint8_t* dev = nullptr;
  size_t cap = 0;
  cudaEvent_t done = nullptr;  // the call that used the slot last has finished with it
  cudaEvent_t sent = nullptr;  // the slot's upload has landed
  bool pending = false;
};

// Device scratch of the rotating calls (rotary factors), one per device.
// A call waits on the GPU for the previous user (event) before writing it,
// so calls on different streams stay ordered without blocking the host.
struct Scratch {
  std::mutex mu;
  uint8_t* ptr = nullptr;
  size_t cap = 0;
  cudaEvent_t last = nullptr;
  bool used = false;
};

struct DeviceCtx {
  int device = -1;
  int sm_count = 0;
  int smem_optin = 0;  // per block
  int smem_sm = 0;     // per SM
  int* err_word = nullptr;
  cudaStream_t up_stream = nullptr;  // descriptor uploads (non-blocking stream)
  std::mutex mu;
  unsigned next = 0;
  RingSlot slots[kRingSlots];
  // rotary-factor scratch, double-buffered so that one call's factor
  // pre-pass (on fac_stream) can run beside the previous call's kernels
  Scratch scratch[2];
  unsigned scratch_next = 0;
  cudaStream_t fac_stream = nullptr;
  cudaEvent_t fac_done[2] = {nullptr, nullptr};
  cudaEvent_t caller_mark = nullptr;
  uint64_t table_gen_seen = 0;  // rotary-table generation the factor stream has waited for
};

// Bumped by every register_rotary: the next factor pre-pass on a device
// first waits for all earlier work on its caller's stream (a table may
// have just been written there).
std::atomic<uint64_t> g_table_gen{1};

std::mutex g_ctx_mu;
std::map<int, std::unique_ptr<DeviceCtx>> g_ctx;

DeviceCtx& device_ctx(int device) {
  std::lock_guard<std::mutex> g(g_ctx_mu);
  auto it = g_ctx.find(device);
  if (it != g_ctx.end()) return *it->second;
  auto c = std::make_unique<DeviceCtx>();
  c->device = device;
  DARIC_CUDA(cudaDeviceGetAttribute(&c->sm_count, cudaDevAttrMultiProcessorCount, device));
  DARIC_CUDA(cudaDeviceGetAttribute(&c->smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device));
  DARIC_CUDA(cudaDeviceGetAttribute(&c->smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, device));
  DeviceGuard dg(device);
  DARIC_CUDA(cudaMalloc(&c->err_word, sizeof(int)));
  DARIC_CUDA(cudaMemset(c->err_word, 0, sizeof(int)));
  for (auto& s : c->slots) {
    // all slots up front, so the first calls after start-up allocate nothing
    DARIC_CUDA(cudaEventCreateWithFlags(&s.done, cudaEventDisableTiming));
    DARIC_CUDA(cudaEventCreateWithFlags(&s.sent, cudaEventDisableTiming));
    DARIC_CUDA(cudaHostAlloc((void**)&s.host, kSlotBytes, cudaHostAllocDefault));
    DARIC_CUDA(cudaMalloc((void**)&s.dev, kSlotBytes));
    s.cap = kSlotBytes;
  }
  for (int i = 0; i < 2; ++i) {
    DARIC_CUDA(cudaEventCreateWithFlags(&c->scratch[i].last, cudaEventDisableTiming));
    DARIC_CUDA(cudaEventCreateWithFlags(&c->fac_done[i], cudaEventDisableTiming));
  }
  DARIC_CUDA(cudaEventCreateWithFlags(&c->caller_mark, cudaEventDisableTiming));
  DARIC_CUDA(cudaStreamCreateWithFlags(&c->up_stream, cudaStreamNonBlocking));
  DARIC_CUDA(cudaStreamCreateWithFlags(&c->fac_stream, cudaStreamNonBlocking));
  auto& ref = *c;
  g_ctx[device] = std::move(c);
  return ref;
}

// One descriptor upload: a ring slot held for the duration of the call.
// The host waits until the slot's previous call has finished with it, so the
// copy can go out on the device's upload stream right away and overlap the
// kernels still running on the caller's stream; the caller's stream waits
// for it with an event. Under stream capture the copy is captured on the
// caller's stream instead.
class Upload {
 public:
  Upload(DeviceCtx& c, size_t bytes) : up_stream_(c.up_stream) {
    {
      std::lock_guard<std::mutex> g(c.mu);
      slot_ = &c.slots[c.next++ % kRingSlots];
    }
    lock_ = std::unique_lock<std::mutex>(slot_->mu);
    if (slot_->pending) {
      DARIC_CUDA(cudaEventSynchronize(slot_->done));
      slot_->pending = false;
    }
    if (slot_->cap < bytes) {
      size_t cap = std::max<size_t>(bytes, 64 * 1024);
      cap = std::max(cap, slot_->cap * 2);
      if (slot_->host) DARIC_CUDA(cudaFreeHost(slot_->host));
      if (slot_->dev) DARIC_CUDA(cudaFree(slot_->dev));
      slot_->host = nullptr;
      slot_->dev = nullptr;
      slot_->cap = 0;
      DARIC_CUDA(cudaHostAlloc((void**)&slot_->host, cap, cudaHostAllocDefault));
      DARIC_CUDA(cudaMalloc((void**)&slot_->dev, cap));
      slot_->cap = cap;
    }
  }
  uint8_t* host() { return slot_->host; }
  uint8_t* dev() { return slot_->dev; }
  void send(size_t bytes, cudaStream_t s) {
    if (!bytes) return;
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    DARIC_CUDA(cudaStreamIsCapturing(s, &cap));
    if (cap != cudaStreamCaptureStatusNone) {
      DARIC_CUDA(cudaMemcpyAsync(slot_->dev, slot_->host, bytes, cudaMemcpyHostToDevice, s));
      return;
    }
    DARIC_CUDA(cudaMemcpyAsync(slot_->dev, slot_->host, bytes, cudaMemcpyHostToDevice, up_stream_));
    DARIC_CUDA(cudaEventRecord(slot_->sent, up_stream_));
    side_sent_ = true;
    DARIC_CUDA(cudaStreamWaitEvent(s, slot_->sent, 0));
  }
  // Another stream that reads the uploaded descriptors waits for them too.
  void also_wait(cudaStream_t other) {
    if (side_sent_) DARIC_CUDA(cudaStreamWaitEvent(other, slot_->sent, 0));
  }
  void finish(cudaStream_t s) {
    DARIC_CUDA(cudaEventRecord(slot_->done, s));
    slot_->pending = true;
    finished_ = true;
  }
  // A call that failed after its upload went out: the slot's next user
  // waits for that copy before it rewrites the pinned buffer.
  ~Upload() {
    if (side_sent_ && !finished_ && cudaEventRecord(slot_->done, up_stream_) == cudaSuccess) slot_->pending = true;
  }

 private:
  cudaStream_t up_stream_;
  bool side_sent_ = false, finished_ = false;
  RingSlot* slot_ = nullptr;
  std::unique_lock<std::mutex> lock_;
};

// Holds the device scratch for one call: the stream first waits (on the GPU)
// for the scratch's previous user; release() marks this call as the user.
// Growth (rare: a larger call than any before) waits on the host and
// reallocates.
class ScratchLease {
 public:
  ScratchLease(DeviceCtx& c, size_t bytes, cudaStream_t s) : sc_(c.scratch[0]), lock_(c.scratch[0].mu), s_(s) {
    if (sc_.cap < bytes) {
      if (sc_.used) DARIC_CUDA(cudaEventSynchronize(sc_.last));
      if (sc_.ptr) DARIC_CUDA(cudaFree(sc_.ptr));
      sc_.ptr = nullptr;
      const size_t cap = std::max(bytes, sc_.cap * 2);
      sc_.cap = 0;
      DARIC_CUDA(cudaMalloc((void**)&sc_.ptr, cap));
      sc_.cap = cap;
    } else if (sc_.used) {
      DARIC_CUDA(cudaStreamWaitEvent(s, sc_.last, 0));
    }
  }
  uint8_t* ptr() const { return sc_.ptr; }
  void release() {
    DARIC_CUDA(cudaEventRecord(sc_.last, s_));
    sc_.used = true;
  }

 private:
  Scratch& sc_;
  std::lock_guard<std::mutex> lock_;
  cudaStream_t s_;
};

// The rotary-factor pre-pass of one call. Outside stream capture it runs on
// the device's factor stream, so it overlaps the kernels still running on
// the caller's stream (the previous call's load): it takes the scratch
// buffer the call before the previous one used, the factor stream waits
// (on the GPU) for that buffer's last reader and for the descriptor upload,
// and the caller's stream waits for the factors before the page kernel.
// The first pre-pass after a rotary table was (re)registered also waits
// for all earlier work on the caller's stream. Under capture everything
// stays on the caller's stream.
class FactorPass {
 public:
  FactorPass(DeviceCtx& c, size_t bytes, cudaStream_t s) : c_(c), s_(s) {
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    DARIC_CUDA(cudaStreamIsCapturing(s, &cap));
    side_ = cap == cudaStreamCaptureStatusNone;
    fs_ = side_ ? c.fac_stream : s;
    {
      std::lock_guard<std::mutex> g(c.mu);
      idx_ = (int)(c.scratch_next++ % 2);
      const uint64_t gen = g_table_gen.load();
      if (side_ && c.table_gen_seen != gen) {
        DARIC_CUDA(cudaEventRecord(c.caller_mark, s));
        DARIC_CUDA(cudaStreamWaitEvent(fs_, c.caller_mark, 0));
        c.table_gen_seen = gen;
      }
    }
    sc_ = &c.scratch[idx_];
    lock_ = std::unique_lock<std::mutex>(sc_->mu);
    if (sc_->cap < bytes) {
      if (sc_->used) DARIC_CUDA(cudaEventSynchronize(sc_->last));
      if (sc_->ptr) DARIC_CUDA(cudaFree(sc_->ptr));
      sc_->ptr = nullptr;
      const size_t cap2 = std::max(bytes, sc_->cap * 2);
      sc_->cap = 0;
      DARIC_CUDA(cudaMalloc((void**)&sc_->ptr, cap2));
      sc_->cap = cap2;
    } else if (sc_->used) {
      DARIC_CUDA(cudaStreamWaitEvent(fs_, sc_->last, 0));
    }
  }
  uint8_t* ptr() const { return sc_->ptr; }
  cudaStream_t stream() const { return fs_; }
  // after the factor kernel: the caller's stream waits for it
  void launched() {
    if (!side_) return;
    DARIC_CUDA(cudaEventRecord(c_.fac_done[idx_], fs_));
    DARIC_CUDA(cudaStreamWaitEvent(s_, c_.fac_done[idx_], 0));
  }
  // after the page kernel: the buffer's last reader
  void release() {
    DARIC_CUDA(cudaEventRecord(sc_->last, s_));
    sc_->used = true;
  }

 private:
  DeviceCtx& c_;
  cudaStream_t s_;
  cudaStream_t fs_ = nullptr;
  bool side_ = false;
  int idx_ = 0;
  Scratch* sc_ = nullptr;
  std::unique_lock<std::mutex> lock_;
};

// Lays out [section 0 | section 1 | ...] with 16-byte aligned sections.
struct Blob {
  size_t size = 0;
  size_t add(size_t bytes) {
    size_t off = (size + 15) & ~size_t(15);
    size = off + bytes;
    return off;
  }
};

// Work counter of a bulk-pipeline launch, written into its uploaded
// descriptors: the units past every CTA's first batch. Returns the first
// batch (0 when the launch does not run the bulk pipeline).
int64_t put_work_counter(uint8_t* dst, int64_t units, const BulkGeom& bg, int sm_count) {
  unsigned long long start = 0;
  int64_t first = 0;
  if (bg.nstage >= 3 && units > 0) {
    const int grid = bulk_grid(units, sm_count, bg.ctas_per_sm);
    first = bulk_first_batch(units, grid);
    start = (unsigned long long)std::min<int64_t>(units, first * grid);
  }
  std::memcpy(dst, &start, sizeof(start));
  return first;
}

// ----------------------------------------------------------- layers -----
struct LayerHost {
  std::string name;
  uint8_t* data = nullptr;
  int device = 0;
  std::vector<int64_t> sizes, strides;
  int64_t es = 1;
  bool page_first = false;
  int num_pages = 0, prefix_size = 0;
  int64_t page_stride = 0, suffix = 0, prefix_stride = 0;
  // rotation
  bool has_rot = false;
  int kv_dtype = -1, tab_dtype = -1, neox = 1;
  LayerDev dev{};  // rotation part filled by register_rotary
};

int64_t checked_mul(int64_t a, int64_t b, const char* what) {
  DARIC_CHECK(a >= 0 && b >= 0, std::string(what) + " must be non-negative");
  DARIC_CHECK(a == 0 || b <= INT64_MAX / a, std::string(what) + " exceeds int64 range");
  return a * b;
}

// Element span of dims [first, ndim) that must be dense in memory
// (helpers.cu:22-64): non-singleton dims sorted by stride must have strides
// 1, s0, s0*s1, ... .
int64_t dense_span(const LayerHost& t, int first) {
  struct D { int dim; int64_t size, stride; };
  std::vector<D> dims;
  for (int d = first; d < (int)t.sizes.size(); ++d) {
    DARIC_CHECK(t.sizes[d] > 0, "KV cache copy dimensions must be non-empty | shape=" +
                                    fmt_vec(t.sizes) + " | stride=" + fmt_vec(t.strides) +
                                    " | failed_dim=" + std::to_string(d));
    if (t.sizes[d] == 1) continue;
    DARIC_CHECK(t.strides[d] > 0,
                "KV cache non-singleton dimensions must have positive strides | shape=" +
                    fmt_vec(t.sizes) + " | stride=" + fmt_vec(t.strides) +
                    " | failed_dim=" + std::to_string(d));
    dims.push_back({d, t.sizes[d], t.strides[d]});
  }
  std::stable_sort(dims.begin(), dims.end(), [](const D& a, const D& b) { return a.stride < b.stride; });
  int64_t expect = 1;
  for (const auto& d : dims) {
    DARIC_CHECK(d.stride == expect,
                "KV cache copy dimensions must form a dense physical span | shape=" +
                    fmt_vec(t.sizes) + " | stride=" + fmt_vec(t.strides) +
                    " | failed_dim=" + std::to_string(d.dim) + " | expected_stride=" +
                    std::to_string(expect) + " | actual_stride=" + std::to_string(d.stride) +
                    " | relation=" + (d.stride > expect ? "hole" : "overlap"));
    expect = checked_mul(expect, d.size, "KV cache dense span");
  }
  return expect;
}

// Page-copy shape of a layer (helpers.cu:94-148).
void page_copy_shape(LayerHost& t) {
  const int nd = (int)t.sizes.size();
  DARIC_CHECK(nd >= 1, "KV cache tensor must have at least one dimension");
  if (t.page_first) {
    DARIC_CHECK(t.sizes[0] > 0, "page dimension must be non-zero");
    DARIC_CHECK(t.sizes[0] <= INT32_MAX, "number of pages exceeds int range: " + std::to_string(t.sizes[0]));
    t.num_pages = (int)t.sizes[0];
    t.prefix_size = 1;
    t.prefix_stride = 0;
    t.page_stride = checked_mul(t.strides[0], t.es, "KV cache page stride");
    t.suffix = checked_mul(dense_span(t, 1), t.es, "KV cache page span");
    if (t.num_pages > 1)
      DARIC_CHECK(t.page_stride >= t.suffix,
                  "KV cache pages overlap | shape=" + fmt_vec(t.sizes) + " | stride=" +
                      fmt_vec(t.strides) + " | page_stride=" + std::to_string(t.page_stride) +
                      " | page_span=" + std::to_string(t.suffix));
  } else {
    DARIC_CHECK(nd >= 2, "non-page-first KV cache tensor must have at least two dimensions");
    DARIC_CHECK(t.sizes[0] > 0, "prefix dimension must be non-zero");
    DARIC_CHECK(t.sizes[1] > 0, "page dimension must be non-zero");
    DARIC_CHECK(t.sizes[0] <= INT32_MAX, "prefix size exceeds int range: " + std::to_string(t.sizes[0]));
    DARIC_CHECK(t.sizes[1] <= INT32_MAX, "number of pages exceeds int range: " + std::to_string(t.sizes[1]));
    t.prefix_size = (int)t.sizes[0];
    t.num_pages = (int)t.sizes[1];
    t.prefix_stride = checked_mul(t.strides[0], t.es, "KV cache prefix stride");
    t.page_stride = checked_mul(t.strides[1], t.es, "KV cache page stride");
    t.suffix = checked_mul(dense_span(t, 2), t.es, "KV cache suffix span");
    // prefix/page regions must not overlap (helpers.cu:66-90)
    std::vector<std::pair<int64_t, int64_t>> axes;
    if (t.prefix_size > 1) axes.emplace_back(t.prefix_stride, t.prefix_size);
    if (t.num_pages > 1) axes.emplace_back(t.page_stride, t.num_pages);
    std::sort(axes.begin(), axes.end());
    int64_t span = t.suffix;
    for (auto& [stride, size] : axes) {
      DARIC_CHECK(stride >= span, "KV cache prefix/page regions overlap | shape=" + fmt_vec(t.sizes) +
                                      " | stride=" + fmt_vec(t.strides) + " | region_size=" +
                                      std::to_string(t.suffix) + " | required_stride=" +
                                      std::to_string(span) + " | actual_stride=" + std::to_string(stride));
      const int64_t ext = checked_mul(size - 1, stride, "KV cache outer span");
      DARIC_CHECK(ext <= INT64_MAX - span, "KV cache outer span exceeds int64 range");
      span += ext;
    }
  }
  DARIC_CHECK(t.page_stride > 0, "page_stride must be positive");
}

int dtype_size(int dt) {
  switch (dt) {
    case DARIC_DTYPE_F32: return 4;
    case DARIC_DTYPE_F16:
    case DARIC_DTYPE_BF16: return 2;
    case DARIC_DTYPE_FP8_E4M3: return 1;
  }
  throw Error(DARIC_ERR_INVALID, "unknown dtype code " + std::to_string(dt));
}

}  // namespace

struct daric_copier {
  std::unordered_map<std::string, LayerHost> layers;
  bool has_store = false;
  uint8_t* store = nullptr;
  int64_t store_bytes = 0;
  int store_device = -1;
};

namespace {

LayerHost& find_layer(daric_copier* c, const char* name) {
  DARIC_CHECK(name != nullptr, "layer name is NULL");
  auto it = c->layers.find(name);
  DARIC_CHECK(it != c->layers.end(), std::string("layer not registered: ") + name);
  return it->second;
}

LayerDev base_layer_dev(const LayerHost& L) {
  LayerDev d = L.dev;
  d.base = L.data;
  d.page_stride = L.page_stride;
  d.prefix_stride = L.prefix_stride;
  d.suffix = L.suffix;
  d.prefix_size = L.prefix_size;
  d.num_pages = L.num_pages;
  d.has_rot = L.has_rot ? 1 : 0;
  return d;
}

// Job validation common to gather/scatter (helpers.cu:150-174,
// copier.cpp:32-39) and the byte-size check (kernels.cu:151-161).
struct JobPlan {
  std::vector<LayerHost*> layers;  // per job
  std::vector<int> layer_slot;     // per job, index into uniq
  std::vector<LayerHost*> uniq;
  std::vector<int64_t> n_sel;
  int64_t total_units = 0;
  int device = -1;
  bool vec16 = true;
};

JobPlan plan_jobs(daric_copier* c, int64_t num_jobs, const char* const* names, const int64_t* offsets,
                  const int64_t* byte_sizes, const int32_t* indices_flat, int64_t indices_numel,
                  int indices_device, const int64_t* indices_offsets) {
  DARIC_CHECK(c != nullptr, "copier is NULL");
  DARIC_CHECK(c->has_store, "store buffer not registered; call register_store() first");
  JobPlan jp;
  DARIC_CHECK(num_jobs >= 0, "num_jobs must be non-negative");
  if (num_jobs == 0) return jp;
  DARIC_CHECK(names && offsets && byte_sizes && indices_offsets, "job arrays must not be NULL");
  DARIC_CHECK(indices_flat != nullptr || indices_numel == 0, "indices_flat is NULL");
  DARIC_CHECK(indices_offsets[0] >= 0, "indices_offsets[0] must be non-negative");
  DARIC_CHECK(indices_offsets[num_jobs] <= indices_numel,
              "indices_offsets.back() exceeds indices_flat.numel()");
  for (int64_t i = 0; i < num_jobs; ++i) {
    DARIC_CHECK(offsets[i] >= 0, "negative store offset at job " + std::to_string(i));
    DARIC_CHECK(byte_sizes[i] >= 0, "negative byte size at job " + std::to_string(i));
    DARIC_CHECK(indices_offsets[i] >= 0, "negative indices offset at job " + std::to_string(i));
    DARIC_CHECK(indices_offsets[i] <= indices_offsets[i + 1],
                "indices_offsets must be non-decreasing at job " + std::to_string(i));
    DARIC_CHECK(offsets[i] <= c->store_bytes, "store offset out of range at job " + std::to_string(i));
    DARIC_CHECK(byte_sizes[i] <= c->store_bytes - offsets[i],
                "store range out of bounds at job " + std::to_string(i));
  }
  std::unordered_map<LayerHost*, int> slot_of;
  std::unordered_map<const char*, LayerHost*> by_ptr;  // callers repeat name buffers
  jp.layers.resize(num_jobs);
  jp.layer_slot.resize(num_jobs);
  jp.n_sel.resize(num_jobs);
  for (int64_t i = 0; i < num_jobs; ++i) {
    auto hit = by_ptr.find(names[i]);
    if (hit == by_ptr.end()) hit = by_ptr.emplace(names[i], &find_layer(c, names[i])).first;
    LayerHost& L = *hit->second;
    if (i == 0) jp.device = L.device;
    DARIC_CHECK(L.device == jp.device,
                "all layers must be on the same device; job " + std::to_string(i));
    jp.layers[i] = &L;
    auto it = slot_of.find(&L);
    if (it == slot_of.end()) {
      it = slot_of.emplace(&L, (int)jp.uniq.size()).first;
      jp.uniq.push_back(&L);
    }
    jp.layer_slot[i] = it->second;
    const int64_t ns = indices_offsets[i + 1] - indices_offsets[i];
    DARIC_CHECK(ns <= INT32_MAX, "too many pages in job " + std::to_string(i));
    jp.n_sel[i] = ns;
    const int64_t expect = (int64_t)L.prefix_size * ns * L.suffix;
    if (byte_sizes[i] != expect) {
      std::ostringstream ss;
      ss << "byte_size mismatch at job " << i << " | C++ expected bytes: " << expect
         << " | Python passed bytes: " << byte_sizes[i] << " | Tensor shape: " << fmt_vec(L.sizes)
         << " | Tensor strides: " << fmt_vec(L.strides);
      throw Error(DARIC_ERR_INVALID, ss.str());
    }
    if (L.suffix % 16 || L.page_stride % 16 || L.prefix_stride % 16 || expect % 16 || offsets[i] % 16 ||
        ((uintptr_t)L.data % 16))
      jp.vec16 = false;
    jp.total_units += ns;
  }
  if ((uintptr_t)c->store % 16) jp.vec16 = false;
  DARIC_CHECK(indices_device == jp.device, "indices_flat must be on the same device as kvcache");
  DARIC_CHECK(c->store_device == jp.device, "store buffer must be on the same device as kvcache");
  return jp;
}

// Limit of the pipelines' waits: DARIC_WAIT_NS (1 ns .. 200 ms) when set,
// else 200 ms. Tests make a wait run out with a short limit together with
// DARIC_TEST_UNARMED=1, which leaves each CTA's first unit unarmed (a
// barrier nothing completes): the call returns and reports the time-out.
int32_t pipeline_wait_ns() {
  const char* v = std::getenv("DARIC_WAIT_NS");
  if (!v) return kDefaultWaitNs;
  const long x = std::strtol(v, nullptr, 10);
  return (x >= 1 && x <= kDefaultWaitNs) ? (int32_t)x : kDefaultWaitNs;
}
int32_t pipeline_unarmed() {
  const char* v = std::getenv("DARIC_TEST_UNARMED");
  return (v && std::strcmp(v, "1") == 0) ? 1 : 0;
}

// Page-kernel choice: the bulk-copy pipeline unless DARIC_PAGE_KERNEL=simt
// (diagnostic switch for A/B measurements of the two implementations).
bool bulk_pipeline_enabled() {
  const char* v = std::getenv("DARIC_PAGE_KERNEL");
  return !(v && std::strcmp(v, "simt") == 0);
}

size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Bulk pipeline geometry for a launch, or nstage = 0 when the pipeline
// cannot hold three stages (load, rotate and store in flight together).
// A unit's producer work is about constant, so units carry up to about
// 64 KiB: up to 8 consecutive pages of a job (the largest that fits three
// stages). Units run page range by page range across the layers of a chunk,
// so one factor block serves many consecutive units: it sits in one of two
// shared-memory factor buffers when they fit too (else in one, loaded once
// the units reading the previous block are done), else the consumer warps
// read it from L2.
// Small pages run 2 or 4 CTAs per SM (more with deviation scores), others
// one (DARIC_BULK_CTAS pins 1 to 4; each CTA has its own producer warp and
// a share of the consumer warps and shared memory);
// DARIC_BULK_CGROUPS splits the consumer warps into 2 or 4 groups.
// DARIC_BULK_CTAS, DARIC_BULK_CGROUPS, DARIC_BULK_CWARPS,
// DARIC_BULK_UNIT_PAGES, DARIC_BULK_FACTORS=l2, DARIC_BULK_FACTOR_BUFFERS and
// DARIC_BULK_FACTOR_FORMAT=f32 pin choices for A/B measurements.
BulkGeom plan_bulk(const DeviceCtx& dc, const std::vector<LayerDev>& layers, bool rotate, bool scores,
                   int tab_dtype) {
  const char* fmt = std::getenv("DARIC_BULK_FACTOR_FORMAT");
  const bool compact = rotate && tab_dtype == DARIC_DTYPE_BF16 && !(fmt && std::strcmp(fmt, "f32") == 0);
  size_t page = 0, slots = 0, fac = 0;
  bool stageable = true;  // factor blocks are whole 16-byte words (bulk copy rule)
  for (const auto& l : layers) {
    page = std::max(page, (size_t)l.prefix_size * (size_t)l.suffix);
    slots = std::max(slots, (size_t)std::max(l.page_size, 1));
    if (rotate && l.has_rot) {
      fac = std::max(fac, page_factor_bytes(l.page_size, l.half_rot, compact));
      stageable = stageable && token_factor_bytes(l.half_rot, compact) % 16 == 0;
    }
  }
  if (page == 0 || page >= (1u << 20)) return BulkGeom{};
  auto env_int = [](const char* name, long lo, long hi) -> long {
    const char* v = std::getenv(name);
    if (!v) return 0;
    const long x = std::strtol(v, nullptr, 10);
    return x >= lo && x <= hi ? x : 0;
  };
  const size_t pin_unit = (size_t)env_int("DARIC_BULK_UNIT_PAGES", 1, 8);
  // Consumer stores (the consumer warps write the paged cache with 16-byte
  // stores instead of the producer's bulk stores) only when
  // DARIC_BULK_CSTORE=1: measured slower on the one- and two-head shards.
  const char* cv = std::getenv("DARIC_BULK_CSTORE");
  const bool cstore = cv && std::strcmp(cv, "1") == 0;
  const long pin_ctas = env_int("DARIC_BULK_CTAS", 1, 4);
  const long pin_groups = env_int("DARIC_BULK_CGROUPS", 1, 4);
  const long pin_cwarps = env_int("DARIC_BULK_CWARPS", 1, 16);
  const char* fv = std::getenv("DARIC_BULK_FACTORS");
  const bool allow_staged = fac > 0 && stageable && !(fv && std::strcmp(fv, "l2") == 0);
  // CTAs per SM: small pages run several CTAs per SM, so several producers
  // feed the SM's copy engine and more units are rotated at once: pages of
  // 8 KiB or less (one KV head of 128 at block 16) two, or four when the
  // launch writes deviation scores (consumer-bound); pages of 16 KiB or less
  // with scores two (measured on the TP4/TP8 head shards of the 70B shape)
  int ctas = 1;
  if (page <= 8 * 1024) ctas = scores ? 4 : 2;
  else if (page <= 16 * 1024 && scores) ctas = 2;
  if (pin_ctas >= 1 && pin_ctas <= 4) ctas = (int)pin_ctas;
  for (; ctas >= 1; ctas /= 2) {
    const size_t budget =
        std::min<size_t>((size_t)dc.smem_optin, (size_t)dc.smem_sm / (size_t)ctas - 1024);  // 1 KiB reserved per CTA
    const size_t groups = (pin_groups == 2 || pin_groups == 4) ? (size_t)pin_groups : 1;
    // stage count: at least 3, a multiple of the consumer groups
    auto stages_for = [&](size_t stage, size_t dev, size_t fixed) -> size_t {
      for (size_t k = 8; k >= 3; --k)
        if (k % groups == 0 && kBulkHeader + round_up(k * dev, 128) + fixed + k * stage <= budget) return k;
      return 0;
    };
    BulkGeom g{};
    auto fill = [&](size_t per_unit, int nbuf) -> bool {  // nbuf factor buffers (0: L2)
      const size_t dev = scores ? round_up(per_unit * slots * 4, 16) : 0;
      const size_t stage = round_up(per_unit * page, 128);
      const size_t fbuf = nbuf ? round_up(per_unit * fac, 128) : 0;
      const size_t ns = stages_for(stage, dev, (size_t)nbuf * fbuf);
      if (ns < 3) return false;
      g.nstage = (int32_t)ns;
      g.stage_bytes = (int32_t)stage;
      g.pages_per_unit = (int32_t)per_unit;
      g.page_data = (int32_t)page;
      g.dev_bytes = (int32_t)round_up(ns * dev, 128);
      g.fac_off = nbuf ? (int32_t)(kBulkHeader + g.dev_bytes) : 0;
      g.fac_buf = (int32_t)fbuf;
      g.fac_nbuf = nbuf;
      g.fac_compact = compact ? 1 : 0;
      g.ctas_per_sm = ctas;
      g.cgroups = (int32_t)groups;
      // consumer warps: the SM's 16 shared by its CTAs; 14 for a single CTA
      // without deviation scores, whose consumers idle part of the time and
      // only add issue contention (measured: 2% faster; with scores the
      // consumers are the bound and keep all 16). DARIC_BULK_CWARPS pins a
      // count, rounded down to a multiple of the groups.
      int cw = (ctas == 1 && !scores) ? 14 : 16 / ctas;
      if (pin_cwarps > 0 && pin_cwarps <= 16 / ctas) cw = (int)pin_cwarps;
      cw -= cw % (int)groups;
      g.cwarps = cw > 0 ? cw : (int)groups;
      g.cstore = cstore ? 1 : 0;
      g.wait_ns = pipeline_wait_ns();
      g.unarmed = pipeline_unarmed();
      return true;
    };
    // The largest unit (up to the per-CTA target) that fits three stages,
    // with its factors in two shared-memory factor buffers when those fit
    // too, else in one, else read from L2.
    const size_t max_unit = std::min<size_t>(8, std::max<size_t>(1, (64 * 1024) / ((size_t)ctas * page)));
    const size_t hi = pin_unit ? pin_unit : max_unit, lo = pin_unit ? pin_unit : 1;
    const long pin_nbuf = env_int("DARIC_BULK_FACTOR_BUFFERS", 1, 2);
    for (size_t u = hi; u >= lo; --u) {
      if (allow_staged && pin_nbuf != 1 && fill(u, 2)) return g;
      if (allow_staged && pin_nbuf != 2 && fill(u, 1)) return g;
      if (fill(u, 0)) return g;
    }
  }
  return BulkGeom{};
}

// Copy-engine geometry of an in-place rotation launch, or nstage = 0 when
// the SIMT kernel runs it (DARIC_PAGE_KERNEL=simt, or a K region too large
// for three stages). Units of up to 8 pages carry about 64 KiB of K rows;
// K regions of 8 KiB or less run two CTAs per SM. DARIC_INPLACE_CTAS,
// DARIC_INPLACE_CWARPS and DARIC_INPLACE_UNIT_PAGES pin the choices for A/B
// measurements.
InplaceGeom plan_inplace(const DeviceCtx& dc, const std::vector<LayerDev>& layers, int tab_dtype) {
  InplaceGeom g{};
  if (!bulk_pipeline_enabled()) return g;
  size_t kbytes = 0;
  for (const auto& l : layers) {
    kbytes = std::max(kbytes, (size_t)l.nrows * (size_t)l.row_bytes);
    // token runs must tile the K region (token-major rows, or head-major
    // rows with whole page-size runs)
    if (l.page_size > 65535 || l.nrows % ((int)l.tok_div.d * l.page_size) != 0) return g;
  }
  if (kbytes == 0 || kbytes % 16 || kbytes >= (1u << 20)) return g;
  auto env_int = [](const char* name, long lo, long hi) -> long {
    const char* v = std::getenv(name);
    if (!v) return 0;
    const long x = std::strtol(v, nullptr, 10);
    return x >= lo && x <= hi ? x : 0;
  };
  int ctas = kbytes <= 8 * 1024 ? 2 : 1;
  if (const long c = env_int("DARIC_INPLACE_CTAS", 1, 2)) ctas = (int)c;
  int cwarps = ctas == 1 ? 16 : 8;
  if (const long w = env_int("DARIC_INPLACE_CWARPS", 1, 16 / ctas)) cwarps = (int)w;
  const size_t budget = std::min<size_t>((size_t)dc.smem_optin, (size_t)dc.smem_sm / (size_t)ctas - 1024);
  const size_t pin = (size_t)env_int("DARIC_INPLACE_UNIT_PAGES", 1, 8);
  size_t pu = pin ? pin : std::min<size_t>(8, std::max<size_t>(1, (64 * 1024) / ((size_t)ctas * kbytes)));
  for (; pu >= 1; --pu) {
    const size_t stage = round_up(pu * kbytes, 128);
    const size_t ns = std::min<size_t>(8, (budget - kBulkHeader) / stage);
    if (ns >= 3) {
      g.nstage = (int32_t)ns;
      g.stage_bytes = (int32_t)stage;
      g.pages_per_unit = (int32_t)pu;
      g.kbytes = (int32_t)kbytes;
      g.ctas_per_sm = ctas;
      g.cwarps = cwarps;
      g.tab_dtype = tab_dtype;
      g.wait_ns = pipeline_wait_ns();
      g.unarmed = pipeline_unarmed();
      return g;
    }
    if (pin) break;
  }
  return InplaceGeom{};
}

// Elements of a 16-byte vector / factors per rotation task of a layer.
int factors_per_task(int kv_dtype, bool neox) {
  const int epv = 16 / dtype_size(kv_dtype);
  return neox ? epv : epv / 2;
}

// Builds and launches page jobs. mode/metas only for the rotating scatter.
void run_page_jobs(daric_copier* c, const JobPlan& jp, const std::vector<int64_t>& job_index,
                   const int64_t* offsets, const int32_t* indices_flat, int64_t indices_numel,
                   const int64_t* indices_offsets, bool gather, bool rotate, int mode,
                   const int64_t* job_meta, const std::vector<MetaDev>& metas, float* scores,
                   int64_t score_ld, const int64_t* job_score_row, RotKey key, cudaStream_t stream) {
  DeviceCtx& dc = device_ctx(jp.device);
  // Layer table restricted to this launch's layers.
  std::vector<int> slot_map(jp.uniq.size(), -1);
  std::vector<LayerDev> layers;
  for (int64_t i : job_index) {
    const int us = jp.layer_slot[i];
    if (slot_map[us] < 0) {
      slot_map[us] = (int)layers.size();
      layers.push_back(base_layer_dev(*jp.uniq[us]));
    }
  }
  // Kernel choice: the bulk pipeline (units of pages_per_unit pages) when
  // jobs are 16-byte aligned and a unit fits three stages, else SIMT (units
  // of one page).
  const BulkGeom bg =
      (jp.vec16 && bulk_pipeline_enabled()) ? plan_bulk(dc, layers, rotate, rotate && scores, key.tab_dtype)
                                            : BulkGeom{};
  const int64_t upp = bg.nstage >= 3 ? bg.pages_per_unit : 1;
  const bool compact = bg.nstage >= 3 && bg.fac_compact;
  std::vector<JobDev> jobs;
  jobs.reserve(job_index.size());
  // Factor runs: one per (rotating chunk, rotary table), padded to whole pages.
  std::map<std::pair<int64_t, const void*>, size_t> run_of;
  std::vector<FacJobDev> runs;
  std::vector<int64_t> run_tokens;  // padded token count of each run
  int64_t units = 0;
  for (int64_t i : job_index) {
    const int us = jp.layer_slot[i];
    if (jp.n_sel[i] == 0) continue;
    JobDev j{};
    j.stg_off = offsets[i];
    j.idx_off = indices_offsets[i];
    j.unit_begin = units;
    j.n_sel = (int32_t)jp.n_sel[i];
    j.layer = slot_map[us];
    j.meta = rotate ? (int32_t)job_meta[i] : -1;
    j.score_row = (rotate && scores) ? (int32_t)job_score_row[i] : -1;
    if (rotate && metas[j.meta].rotate) {
      const LayerDev& L = layers[j.layer];
      const MetaDev& m = metas[j.meta];
      const int64_t ntok = (int64_t)j.n_sel * L.page_size;
      const int64_t len = std::min(m.len, ntok);
      // positions must lie inside the table (index_select would raise)
      const bool ok = mode == DARIC_ROPE_FLEXIBLE
                          ? (m.pos_a >= 0 && m.pos_b >= 0 && m.pos_a + len <= L.max_pos && m.pos_b + len <= L.max_pos)
                          : (m.pos_a >= 0 && m.pos_a < L.max_pos);
      DARIC_CHECK(len <= 0 || ok, "rotary position out of range of cos_sin_cache (max_position=" +
                                      std::to_string(L.max_pos) + ") at chunk " + std::to_string(j.meta));
      auto key2 = std::make_pair((int64_t)j.meta, (const void*)L.table);
      auto it = run_of.find(key2);
      if (it == run_of.end()) {
        FacJobDev f{};
        f.table = L.table;
        f.table_row = L.table_row;
        f.pos_a = m.pos_a;
        f.pos_b = m.pos_b;
        f.len = len;
        f.half_rot = L.half_rot;
        f.P = L.pair_vecs;
        it = run_of.emplace(key2, runs.size()).first;
        runs.push_back(f);
        run_tokens.push_back(ntok);
      } else {
        DARIC_CHECK(runs[it->second].half_rot == L.half_rot && runs[it->second].P == L.pair_vecs,
                    "layers sharing a rotary table must share its rotary_dim");
        runs[it->second].len = std::max(runs[it->second].len, len);
        run_tokens[it->second] = std::max(run_tokens[it->second], ntok);
      }
    }
    jobs.push_back(j);
    units += (jp.n_sel[i] + upp - 1) / upp;
  }
  if (units == 0) return;
  // token offsets and entry offsets of the runs
  // runs of different rotary_dim use different token strides: each run
  // starts at the first token of its own stride past the previous run
  int64_t items = 0, fac_bytes = 0;
  for (size_t r = 0; r < runs.size(); ++r) {
    const int64_t tok_bytes = (int64_t)token_factor_bytes(runs[r].half_rot, compact);
    runs[r].out_tok = (fac_bytes + tok_bytes - 1) / tok_bytes;
    runs[r].item_begin = items;
    items += runs[r].len * (runs[r].half_rot / 2);
    fac_bytes = (runs[r].out_tok + run_tokens[r]) * tok_bytes;
  }
  for (auto& j : jobs)
    if (j.meta >= 0 && metas[j.meta].rotate)
      j.fac_tok = runs[run_of[std::make_pair((int64_t)j.meta, (const void*)layers[j.layer].table)]].out_tok;
  runs.erase(std::remove_if(runs.begin(), runs.end(), [](const FacJobDev& f) { return f.len <= 0; }), runs.end());
  // Bulk pipeline unit order: groups of consecutive jobs of one chunk with
  // the same page count and factor run (same tokens, same factors).
  std::vector<GroupDev> groups;
  if (bg.nstage >= 3) {
    int64_t u = 0;
    for (size_t a = 0; a < jobs.size();) {
      const JobDev& A = jobs[a];
      const LayerDev& LA = layers[A.layer];
      size_t e = a + 1;
      for (; e < jobs.size(); ++e) {
        const JobDev& B = jobs[e];
        const LayerDev& LB = layers[B.layer];
        if (B.meta != A.meta || B.n_sel != A.n_sel || B.fac_tok != A.fac_tok || LB.page_size != LA.page_size ||
            LB.half_rot != LA.half_rot || LB.has_rot != LA.has_rot)
          break;
      }
      GroupDev gd{};
      gd.unit_begin = u;
      gd.j0 = (int32_t)a;
      gd.cnt = (int32_t)(e - a);
      gd.n_sel = A.n_sel;
      gd.nranges = (int32_t)((A.n_sel + upp - 1) / upp);
      u += (int64_t)gd.nranges * gd.cnt;
      groups.push_back(gd);
      a = e;
    }
    DARIC_CHECK(u == units, "internal: bulk unit count mismatch");
  }
  DeviceGuard dg(jp.device);
  Blob b;
  const size_t o_layers = b.add(layers.size() * sizeof(LayerDev));
  const size_t o_jobs = b.add(jobs.size() * sizeof(JobDev));
  const size_t o_metas = b.add(metas.size() * sizeof(MetaDev));
  const size_t o_runs = b.add(runs.size() * sizeof(FacJobDev));
  const size_t o_groups = b.add(groups.size() * sizeof(GroupDev));
  const size_t o_work = b.add(sizeof(unsigned long long));
  Upload up(dc, b.size);
  std::memcpy(up.host() + o_layers, layers.data(), layers.size() * sizeof(LayerDev));
  std::memcpy(up.host() + o_jobs, jobs.data(), jobs.size() * sizeof(JobDev));
  if (!metas.empty()) std::memcpy(up.host() + o_metas, metas.data(), metas.size() * sizeof(MetaDev));
  if (!runs.empty()) std::memcpy(up.host() + o_runs, runs.data(), runs.size() * sizeof(FacJobDev));
  if (!groups.empty()) std::memcpy(up.host() + o_groups, groups.data(), groups.size() * sizeof(GroupDev));
  const int64_t first_batch = put_work_counter(up.host() + o_work, units, bg, dc.sm_count);
  std::unique_ptr<FactorPass> lease;
  if (fac_bytes > 0) lease = std::make_unique<FactorPass>(dc, (size_t)fac_bytes, stream);
  float4* fac = lease ? reinterpret_cast<float4*>(lease->ptr()) : nullptr;
  up.send(b.size, stream);
  if (lease) up.also_wait(lease->stream());
  if (!runs.empty()) {
    FactorLaunch fl{};
    fl.jobs = reinterpret_cast<const FacJobDev*>(up.dev() + o_runs);
    fl.num_jobs = (int64_t)runs.size();
    fl.total_items = items;
    fl.out = fac;
    fl.mode = mode;
    fl.fpv = factors_per_task(key.kv_dtype, key.neox != 0);
    fl.compact = compact ? 1 : 0;
    fl.contig = (bg.nstage >= 3 && !bg.fac_off) ? 1 : 0;  // the bulk kernel reads factors from L2
    launch_factors(fl, key.tab_dtype, dc.sm_count, lease->stream());
  }
  if (lease) lease->launched();
  PageLaunch p{};
  p.layers = reinterpret_cast<const LayerDev*>(up.dev() + o_layers);
  p.jobs = reinterpret_cast<const JobDev*>(up.dev() + o_jobs);
  p.metas = reinterpret_cast<const MetaDev*>(up.dev() + o_metas);
  p.store = c->store;
  p.store_mut = c->store;
  p.indices = indices_flat;
  p.indices_numel = indices_numel;
  p.num_jobs = (int64_t)jobs.size();
  p.total_units = units;
  p.mode = mode;
  p.scores = scores;
  p.score_ld = score_ld;
  p.err = dc.err_word;
  p.fac = fac;
  p.groups = reinterpret_cast<const GroupDev*>(up.dev() + o_groups);
  p.num_groups = (int64_t)groups.size();
  p.work = reinterpret_cast<unsigned long long*>(up.dev() + o_work);
  p.first_batch = first_batch;
  if (bg.nstage >= 3) {
    if (rotate) launch_bulk_rotate(p, bg, key, dc.sm_count, stream);
    else launch_bulk_plain(p, bg, gather, dc.sm_count, stream);
  } else if (rotate) {
    launch_rotate_scatter(p, key, dc.sm_count, stream);
  } else {
    launch_plain_pages(p, gather, jp.vec16, dc.sm_count, stream);
  }
  if (lease) lease->release();
  up.finish(stream);
}

void do_copy(daric_copier* c, bool gather, int64_t num_jobs, const char* const* names,
             const int64_t* offsets, const int64_t* byte_sizes, const int32_t* indices_flat,
             int64_t indices_numel, int indices_device, const int64_t* indices_offsets, void* stream) {
  JobPlan jp = plan_jobs(c, num_jobs, names, offsets, byte_sizes, indices_flat, indices_numel,
                         indices_device, indices_offsets);
  if (num_jobs == 0 || jp.total_units == 0) return;
  std::vector<int64_t> all(num_jobs);
  for (int64_t i = 0; i < num_jobs; ++i) all[i] = i;
  run_page_jobs(c, jp, all, offsets, indices_flat, indices_numel, indices_offsets, gather, false,
                DARIC_ROPE_NONE, nullptr, {}, nullptr, 0, nullptr, RotKey{}, (cudaStream_t)stream);
}

// Chunk-level load (daric_copier_load_chunks): chunk m holds, for every
// layer of `names` in order, [prefix][n_sel pages][page bytes] at
// chunk_stg_off[m] + n_sel * (bytes per page of the layers before it); the
// call loads layers [l0, l1). All layers of a chunk use the chunk's one
// block-id list. The bulk pipeline derives each (chunk, layer) job on the
// device from one descriptor per chunk; the SIMT kernels get a job table
// built here (its entries share the chunk's block-id range).
void run_chunk_load(daric_copier* c, int64_t num_layers, const char* const* names, int64_t l0, int64_t l1,
                    int64_t M, const int64_t* chunk_stg_off, const int64_t* chunk_blk_off,
                    const int64_t* chunk_pages, const int32_t* block_ids, int64_t block_ids_numel,
                    int block_ids_device, int mode, const int64_t* pos_a, const int64_t* pos_b,
                    const int64_t* len, float* scores, int64_t score_ld, const int64_t* score_col,
                    cudaStream_t stream) {
  DARIC_CHECK(c != nullptr, "copier is NULL");
  DARIC_CHECK(c->has_store, "store buffer not registered; call register_store() first");
  DARIC_CHECK(mode == DARIC_ROPE_FLEXIBLE || mode == DARIC_ROPE_DELTA || mode == DARIC_ROPE_NONE,
              "unknown rotation mode " + std::to_string(mode));
  DARIC_CHECK(num_layers >= 0 && M >= 0, "negative layer or chunk count");
  DARIC_CHECK(0 <= l0 && l0 <= l1 && l1 <= num_layers, "layer range outside the layer list");
  if (M == 0 || l0 == l1) return;
  DARIC_CHECK(names && chunk_stg_off && chunk_blk_off && chunk_pages, "chunk arrays must not be NULL");
  DARIC_CHECK(block_ids != nullptr || block_ids_numel == 0, "block_ids is NULL");
  const bool rotate = mode != DARIC_ROPE_NONE;
  if (rotate) DARIC_CHECK(pos_a && len && (mode != DARIC_ROPE_FLEXIBLE || pos_b), "chunk position arrays are NULL");
  if (scores) DARIC_CHECK(score_col && score_ld >= 0, "scores need score_col and a non-negative score_ld");
  // layers: all of them fix the store layout; [l0, l1) are loaded
  std::vector<LayerHost*> all(num_layers);
  std::vector<int64_t> page_off(num_layers + 1, 0);
  for (int64_t j = 0; j < num_layers; ++j) {
    all[j] = &find_layer(c, names[j]);
    const int64_t per_page = checked_mul(all[j]->prefix_size, all[j]->suffix, "bytes per page");
    page_off[j + 1] = page_off[j] + per_page;
  }
  const int device = all[l0]->device;
  DARIC_CHECK(block_ids_device == device, "block_ids must be on the same device as kvcache");
  DARIC_CHECK(c->store_device == device, "store buffer must be on the same device as kvcache");
  std::vector<LayerDev> layers;
  bool vec16 = ((uintptr_t)c->store % 16) == 0;
  for (int64_t j = l0; j < l1; ++j) {
    LayerHost& L = *all[j];
    DARIC_CHECK(L.device == device, "all layers must be on the same device; layer " + L.name);
    DARIC_CHECK(!rotate || L.has_rot, "layer has no rotary table (register_rotary): " + L.name);
    DARIC_CHECK(!rotate || (L.kv_dtype == all[l0]->kv_dtype && L.tab_dtype == all[l0]->tab_dtype &&
                            L.neox == all[l0]->neox),
                "load_chunks: the layers of one call must share KV dtype, table dtype and rotary style");
    LayerDev d = base_layer_dev(L);
    d.store_page_off = page_off[j];
    d.score_row = scores ? (int32_t)j : -1;
    if (L.suffix % 16 || L.page_stride % 16 || L.prefix_stride % 16 || ((uintptr_t)L.data % 16)) vec16 = false;
    layers.push_back(d);
  }
  // chunks
  std::vector<MetaDev> metas(M);
  for (int64_t m = 0; m < M; ++m) {
    const int64_t ns = chunk_pages[m];
    DARIC_CHECK(ns >= 0 && ns <= INT32_MAX, "bad page count at chunk " + std::to_string(m));
    DARIC_CHECK(chunk_stg_off[m] >= 0 && chunk_blk_off[m] >= 0, "negative chunk offset at chunk " + std::to_string(m));
    DARIC_CHECK(chunk_blk_off[m] + ns <= block_ids_numel, "chunk " + std::to_string(m) + " reaches past block_ids");
    const int64_t bytes = checked_mul(ns, page_off[num_layers], "chunk bytes");
    DARIC_CHECK(chunk_stg_off[m] <= c->store_bytes && bytes <= c->store_bytes - chunk_stg_off[m],
                "store range out of bounds at chunk " + std::to_string(m));
    if (chunk_stg_off[m] % 16) vec16 = false;
    MetaDev& d = metas[m];
    d.pos_a = rotate ? pos_a[m] : 0;
    d.pos_b = mode == DARIC_ROPE_FLEXIBLE ? pos_b[m] : 0;
    d.len = rotate ? len[m] : 0;
    DARIC_CHECK(d.len >= 0, "negative chunk length at chunk " + std::to_string(m));
    d.score_col = scores ? score_col[m] : 0;
    if (scores) DARIC_CHECK(d.score_col >= 0, "negative score column at chunk " + std::to_string(m));
    d.rotate = (!rotate || d.len == 0 || (mode == DARIC_ROPE_FLEXIBLE && d.pos_a == d.pos_b)) ? 0 : 1;
  }
  if (vec16) {
    for (int64_t j = 0; j < num_layers; ++j)
      if ((all[j]->prefix_size * all[j]->suffix) % 16) vec16 = false;
  }
  DARIC_CHECK(vec16 || !rotate, "load_chunks needs 16-byte aligned layers, chunk offsets and pages");
  DeviceCtx& dc = device_ctx(device);
  const RotKey key = rotate ? RotKey{all[l0]->kv_dtype, all[l0]->tab_dtype, all[l0]->neox} : RotKey{};
  bool uniform = true;  // one group per chunk needs one page size / rotary geometry
  for (const auto& d : layers)
    uniform = uniform && d.page_size == layers[0].page_size && d.half_rot == layers[0].half_rot &&
              d.has_rot == layers[0].has_rot && d.table == layers[0].table;
  const BulkGeom bg = (vec16 && uniform && bulk_pipeline_enabled())
                          ? plan_bulk(dc, layers, rotate, rotate && scores, key.tab_dtype)
                          : BulkGeom{};
  const bool bulk = bg.nstage >= 3;
  const int64_t upp = bulk ? bg.pages_per_unit : 1;
  const bool compact = bulk && bg.fac_compact;
  const int64_t Lc = l1 - l0;
  // factor runs: one per rotating chunk and table, padded to whole pages
  std::vector<FacJobDev> runs;
  std::vector<int64_t> fac_tok(M, 0);
  int64_t items = 0, fac_bytes = 0;
  std::vector<std::pair<const void*, int64_t>> tables;  // (table, first run) per distinct table
  for (size_t li = 0; li < layers.size() && rotate; ++li) {
    const LayerDev& L = layers[li];
    bool seen = false;
    for (auto& t : tables) seen = seen || t.first == (const void*)L.table;
    if (seen) continue;
    DARIC_CHECK(tables.empty(), "load_chunks: the layers of one call must share one rotary table");
    tables.emplace_back((const void*)L.table, 0);
    const int64_t tok_bytes = (int64_t)token_factor_bytes(L.half_rot, compact);
    for (int64_t m = 0; m < M; ++m) {
      if (!metas[m].rotate) continue;
      const int64_t ntok = chunk_pages[m] * L.page_size;
      const int64_t ln = std::min(metas[m].len, ntok);
      const MetaDev& md = metas[m];
      const bool ok = mode == DARIC_ROPE_FLEXIBLE
                          ? (md.pos_a >= 0 && md.pos_b >= 0 && md.pos_a + ln <= L.max_pos && md.pos_b + ln <= L.max_pos)
                          : (md.pos_a >= 0 && md.pos_a < L.max_pos);
      DARIC_CHECK(ln <= 0 || ok, "rotary position out of range of cos_sin_cache (max_position=" +
                                     std::to_string(L.max_pos) + ") at chunk " + std::to_string(m));
      FacJobDev f{};
      f.table = L.table;
      f.table_row = L.table_row;
      f.pos_a = md.pos_a;
      f.pos_b = md.pos_b;
      f.len = ln;
      f.half_rot = L.half_rot;
      f.P = L.pair_vecs;
      f.out_tok = (fac_bytes + tok_bytes - 1) / tok_bytes;
      f.item_begin = items;
      items += ln * (L.half_rot / 2);
      fac_bytes = (f.out_tok + ntok) * tok_bytes;
      fac_tok[m] = f.out_tok;
      if (ln > 0) runs.push_back(f);
    }
  }
  // groups (bulk: one per chunk, jobs derived on the device) or a job table
  std::vector<GroupDev> groups;
  std::vector<JobDev> jobs;
  int64_t units = 0;
  for (int64_t m = 0; m < M; ++m) {
    const int64_t ns = chunk_pages[m];
    if (ns == 0) continue;
    if (bulk) {
      GroupDev gd{};
      gd.unit_begin = units;
      gd.j0 = 0;
      gd.cnt = (int32_t)Lc;
      gd.n_sel = (int32_t)ns;
      gd.nranges = (int32_t)((ns + upp - 1) / upp);
      gd.stg_off = chunk_stg_off[m];
      gd.idx_off = chunk_blk_off[m];
      gd.fac_tok = fac_tok[m];
      gd.meta = (int32_t)m;
      units += (int64_t)gd.nranges * Lc;
      groups.push_back(gd);
    } else {
      for (int64_t li = 0; li < Lc; ++li) {
        JobDev j{};
        j.stg_off = chunk_stg_off[m] + ns * layers[li].store_page_off;
        j.idx_off = chunk_blk_off[m];
        j.unit_begin = units;
        j.fac_tok = fac_tok[m];
        j.n_sel = (int32_t)ns;
        j.layer = (int32_t)li;
        j.meta = rotate ? (int32_t)m : -1;
        j.score_row = (rotate && scores) ? layers[li].score_row : -1;
        jobs.push_back(j);
        units += ns;
      }
    }
  }
  if (units == 0) return;
  DeviceGuard dg(device);
  Blob b;
  const size_t o_layers = b.add(layers.size() * sizeof(LayerDev));
  const size_t o_jobs = b.add(jobs.size() * sizeof(JobDev));
  const size_t o_metas = b.add(metas.size() * sizeof(MetaDev));
  const size_t o_runs = b.add(runs.size() * sizeof(FacJobDev));
  const size_t o_groups = b.add(groups.size() * sizeof(GroupDev));
  const size_t o_work = b.add(sizeof(unsigned long long));
  Upload up(dc, b.size);
  std::memcpy(up.host() + o_layers, layers.data(), layers.size() * sizeof(LayerDev));
  if (!jobs.empty()) std::memcpy(up.host() + o_jobs, jobs.data(), jobs.size() * sizeof(JobDev));
  std::memcpy(up.host() + o_metas, metas.data(), metas.size() * sizeof(MetaDev));
  if (!runs.empty()) std::memcpy(up.host() + o_runs, runs.data(), runs.size() * sizeof(FacJobDev));
  if (!groups.empty()) std::memcpy(up.host() + o_groups, groups.data(), groups.size() * sizeof(GroupDev));
  const int64_t first_batch = put_work_counter(up.host() + o_work, units, bg, dc.sm_count);
  std::unique_ptr<FactorPass> lease;
  if (fac_bytes > 0) lease = std::make_unique<FactorPass>(dc, (size_t)fac_bytes, stream);
  float4* fac = lease ? reinterpret_cast<float4*>(lease->ptr()) : nullptr;
  up.send(b.size, stream);
  if (lease) up.also_wait(lease->stream());
  if (!runs.empty()) {
    FactorLaunch fl{};
    fl.jobs = reinterpret_cast<const FacJobDev*>(up.dev() + o_runs);
    fl.num_jobs = (int64_t)runs.size();
    fl.total_items = items;
    fl.out = fac;
    fl.mode = mode;
    fl.fpv = factors_per_task(key.kv_dtype, key.neox != 0);
    fl.compact = compact ? 1 : 0;
    fl.contig = (bg.nstage >= 3 && !bg.fac_off) ? 1 : 0;  // the bulk kernel reads factors from L2
    launch_factors(fl, key.tab_dtype, dc.sm_count, lease->stream());
  }
  if (lease) lease->launched();
  PageLaunch p{};
  p.layers = reinterpret_cast<const LayerDev*>(up.dev() + o_layers);
  p.jobs = bulk ? nullptr : reinterpret_cast<const JobDev*>(up.dev() + o_jobs);
  p.metas = reinterpret_cast<const MetaDev*>(up.dev() + o_metas);
  p.store = c->store;
  p.store_mut = c->store;
  p.indices = block_ids;
  p.indices_numel = block_ids_numel;
  p.num_jobs = (int64_t)jobs.size();
  p.total_units = units;
  p.mode = mode;
  p.scores = rotate ? scores : nullptr;
  p.score_ld = score_ld;
  p.err = dc.err_word;
  p.fac = fac;
  p.groups = reinterpret_cast<const GroupDev*>(up.dev() + o_groups);
  p.num_groups = (int64_t)groups.size();
  p.work = reinterpret_cast<unsigned long long*>(up.dev() + o_work);
  p.first_batch = first_batch;
  if (bulk) {
    if (rotate) launch_bulk_rotate(p, bg, key, dc.sm_count, stream);
    else launch_bulk_plain(p, bg, false, dc.sm_count, stream);
  } else if (rotate) {
    launch_rotate_scatter(p, key, dc.sm_count, stream);
  } else {
    launch_plain_pages(p, false, vec16, dc.sm_count, stream);
  }
  if (lease) lease->release();
  up.finish(stream);
}

// Rotation geometry of a registered layer (adapter.py:311-368 stride rules).
void resolve_rotary(LayerHost& L, int kv_dtype, const void* table, int tab_dtype, int64_t max_pos,
                    int64_t rot_dim, int neox) {
  const int kv_es = dtype_size(kv_dtype);
  DARIC_CHECK(kv_es == L.es, "kv_dtype size does not match the registered element size");
  const int tab_es = dtype_size(tab_dtype);
  DARIC_CHECK(tab_dtype != DARIC_DTYPE_FP8_E4M3, "fp8 rotary tables are not supported");
  DARIC_CHECK(table != nullptr, "cos_sin_cache is NULL");
  DARIC_CHECK(max_pos > 0, "cos_sin_cache must have at least one row");
  const auto& s = L.sizes;
  const auto& st = L.strides;
  const int nd = (int)s.size();
  int64_t nrows = 0, row_elems = 0, head_dim = 0, tok_div = 1, page_size = 0;
  int k_prefix = 0;
  if (nd == 5) {
    // page-first (nb, 2, bs, H, D) or (2, nb, bs, H, D): K rows (bs, H) dense.
    page_size = s[2];
    const int64_t H = s[3], D = s[4];
    DARIC_CHECK(st[4] == 1 && (H == 1 || st[3] == D) && (page_size == 1 || st[2] == H * D),
                "rerotate: 5-D KV cache needs dense (block_size, heads, head_dim) K rows");
    nrows = page_size * H;
    row_elems = D;
    head_dim = D;
    tok_div = H;
    k_prefix = 0;
  } else if (nd == 4) {
    DARIC_CHECK(L.page_first, "Invalid 4D KV cache for rerotate: page_first must be true");
    const int64_t H = s[1], packed = s[3];
    page_size = s[2];
    DARIC_CHECK(packed > 0 && packed % 2 == 0,
                "Invalid 4D KV cache for rerotate: packed content dimension must be positive and even");
    DARIC_CHECK(st[3] == 1, "Invalid 4D KV cache for rerotate: packed content feature stride must equal 1");
    DARIC_CHECK((page_size == 1 || st[2] == packed) && (H == 1 || st[1] == page_size * packed),
                "rerotate: 4-D KV cache needs dense (heads, block_size, packed) rows");
    head_dim = packed / 2;
    nrows = H * page_size;
    row_elems = packed;
    tok_div = 1;
  } else if (nd == 3) {
    DARIC_CHECK(L.page_first, "rerotate: 3-D KV cache must be registered page_first");
    page_size = s[1];
    DARIC_CHECK(st[2] == 1 && (page_size == 1 || st[1] == s[2]), "rerotate: 3-D KV cache rows must be dense");
    nrows = page_size;
    row_elems = s[2];
    head_dim = s[2];
    tok_div = 1;
  } else {
    throw Error(DARIC_ERR_INVALID, "Unsupported KV cache rank for rerotate: " + std::to_string(nd));
  }
  DARIC_CHECK(rot_dim > 0 && rot_dim % 2 == 0 && rot_dim <= head_dim,
              "rotary_dim must be positive, even, and no greater than the K head dimension");
  DARIC_CHECK(page_size >= 1 && page_size <= 1024, "rerotate: block size must be in [1, 1024]");

  const int64_t half = rot_dim / 2;
  const int64_t row_bytes = row_elems * kv_es;
  DARIC_CHECK(row_bytes % 16 == 0, "rerotate: K row bytes must be a multiple of 16");
  if (neox) DARIC_CHECK((half * kv_es) % 16 == 0, "rerotate: rotary_dim/2 * element size must be a multiple of 16");
  else DARIC_CHECK((rot_dim * kv_es) % 16 == 0, "rerotate: rotary_dim * element size must be a multiple of 16");
  DARIC_CHECK((half * tab_es) % 16 == 0 && ((uintptr_t)table % 16) == 0,
              "rerotate: cos_sin_cache must be 16-byte aligned with 16-byte aligned halves");
  DARIC_CHECK(nrows * row_bytes <= L.suffix, "rerotate: K rows exceed the page region");
  DARIC_CHECK(((uintptr_t)L.data % 16) == 0 && L.page_stride % 16 == 0 && L.prefix_stride % 16 == 0 &&
                  L.suffix % 16 == 0,
              "rerotate: KV layer must be 16-byte aligned");
  DARIC_CHECK(nrows * (row_bytes / 16) < INT32_MAX, "rerotate: page too large");
  LayerDev& d = L.dev;
  d.k_prefix = k_prefix;
  d.nrows = (int32_t)nrows;
  d.row_bytes = (int32_t)row_bytes;
  d.row_vecs = (int32_t)(row_bytes / 16);
  d.rot_vecs = (int32_t)(rot_dim * kv_es / 16);
  d.pair_vecs = neox ? d.rot_vecs / 2 : d.rot_vecs;
  d.page_size = (int32_t)page_size;
  d.pair_div = make_fastdiv((uint32_t)d.pair_vecs);
  d.tok_div = make_fastdiv((uint32_t)tok_div);
  d.tok_mod = make_fastdiv((uint32_t)page_size);
  d.tail_vecs = d.row_vecs - d.rot_vecs;
  d.tail_div = make_fastdiv((uint32_t)(d.tail_vecs > 0 ? d.tail_vecs : 1));
  d.page_div = make_fastdiv((uint32_t)(d.nrows * d.pair_vecs));
  d.half_rot = (int32_t)half;
  d.table = (const uint8_t*)table;
  d.table_row = rot_dim * tab_es;
  d.max_pos = max_pos;
  L.has_rot = true;
  L.kv_dtype = kv_dtype;
  L.tab_dtype = tab_dtype;
  L.neox = neox ? 1 : 0;
}

}  // namespace

// Error reporting for entry points implemented in other translation units.
namespace daric {
void record_error(int code, const char* msg) {
  (void)code;
  g_last_error = msg;
}
void clear_error() { g_last_error.clear(); }
}  // namespace daric

// ===================================================================== C ==
extern "C" {

const char* daric_last_error(void) { return g_last_error.c_str(); }

int daric_version(void) { return 100; }

int daric_device_sm_count(int device, int* out) {
  return guarded([&] {
    DARIC_CHECK(out, "out is NULL");
    *out = device_ctx(device).sm_count;
  });
}

int daric_device_errors(int device, int* out_bits) {
  return guarded([&] {
    DARIC_CHECK(out_bits, "out_bits is NULL");
    DeviceCtx& dc = device_ctx(device);
    DeviceGuard dg(device);
    int v = 0;
    DARIC_CUDA(cudaDeviceSynchronize());
    DARIC_CUDA(cudaMemcpy(&v, dc.err_word, sizeof(int), cudaMemcpyDeviceToHost));
    DARIC_CUDA(cudaMemset(dc.err_word, 0, sizeof(int)));
    *out_bits = v;
  });
}

int daric_copier_create(daric_copier** out) {
  return guarded([&] {
    DARIC_CHECK(out, "out is NULL");
    *out = new daric_copier();
  });
}

void daric_copier_destroy(daric_copier* c) { delete c; }

int daric_copier_register_layer(daric_copier* c, const char* name, void* data, int device, int ndim,
                                const int64_t* sizes, const int64_t* strides, int64_t element_size,
                                int is_page_first) {
  return guarded([&] {
    DARIC_CHECK(c && name, "copier/name is NULL");
    DARIC_CHECK(device >= 0, std::string("kvcache tensor must be on GPU: ") + name);
    DARIC_CHECK(ndim >= 1 && sizes && strides, "KV cache tensor must have at least one dimension");
    DARIC_CHECK(element_size > 0, "element_size must be positive");
    LayerHost L;
    L.name = name;
    L.data = (uint8_t*)data;
    L.device = device;
    L.sizes.assign(sizes, sizes + ndim);
    L.strides.assign(strides, strides + ndim);
    L.es = element_size;
    L.page_first = is_page_first != 0;
    page_copy_shape(L);
    c->layers.insert_or_assign(std::string(name), std::move(L));
  });
}

int daric_copier_register_store(daric_copier* c, void* data, int64_t nbytes, int device) {
  return guarded([&] {
    DARIC_CHECK(c, "copier is NULL");
    DARIC_CHECK(device >= 0, "staging buffer must be on CUDA");
    DARIC_CHECK(nbytes >= 0 && (data || nbytes == 0), "store buffer must be a valid device range");
    c->store = (uint8_t*)data;
    c->store_bytes = nbytes;
    c->store_device = device;
    c->has_store = true;
  });
}

int daric_copier_register_rotary(daric_copier* c, const char* layer_name, int kv_dtype,
                                 const void* table, int tab_dtype, int64_t max_pos, int64_t rot_dim,
                                 int is_neox) {
  return guarded([&] {
    DARIC_CHECK(c, "copier is NULL");
    LayerHost& L = find_layer(c, layer_name);
    resolve_rotary(L, kv_dtype, table, tab_dtype, max_pos, rot_dim, is_neox);
    g_table_gen.fetch_add(1);
  });
}

int daric_copier_gather_pages(daric_copier* c, int64_t num_jobs, const char* const* names,
                              const int64_t* offsets, const int64_t* byte_sizes,
                              const int32_t* indices_flat, int64_t indices_numel, int indices_device,
                              const int64_t* indices_offsets, void* stream) {
  return guarded([&] {
    do_copy(c, true, num_jobs, names, offsets, byte_sizes, indices_flat, indices_numel, indices_device,
            indices_offsets, stream);
  });
}

int daric_copier_scatter_pages(daric_copier* c, int64_t num_jobs, const char* const* names,
                               const int64_t* offsets, const int64_t* byte_sizes,
                               const int32_t* indices_flat, int64_t indices_numel, int indices_device,
                               const int64_t* indices_offsets, void* stream) {
  return guarded([&] {
    do_copy(c, false, num_jobs, names, offsets, byte_sizes, indices_flat, indices_numel, indices_device,
            indices_offsets, stream);
  });
}

int daric_copier_rerotate_scatter_pages(
    daric_copier* c, int64_t num_jobs, const char* const* names, const int64_t* offsets,
    const int64_t* byte_sizes, const int32_t* indices_flat, int64_t indices_numel, int indices_device,
    const int64_t* indices_offsets, const int64_t* job_meta, int mode, int64_t num_metas,
    const int64_t* meta_pos_a, const int64_t* meta_pos_b, const int64_t* meta_len, float* scores,
    int64_t score_ld, const int64_t* job_score_row, const int64_t* meta_score_col, void* stream) {
  return guarded([&] {
    DARIC_CHECK(mode == DARIC_ROPE_FLEXIBLE || mode == DARIC_ROPE_DELTA || mode == DARIC_ROPE_NONE,
                "unknown rotation mode " + std::to_string(mode));
    JobPlan jp = plan_jobs(c, num_jobs, names, offsets, byte_sizes, indices_flat, indices_numel,
                           indices_device, indices_offsets);
    if (num_jobs == 0 || jp.total_units == 0) return;
    DARIC_CHECK(num_metas >= 0 && (num_metas == 0 || (meta_pos_a && meta_len)), "chunk arrays are NULL");
    DARIC_CHECK(mode != DARIC_ROPE_FLEXIBLE || num_metas == 0 || meta_pos_b,
                "FLEXIBLE mode needs meta_pos_b (new positions)");
    DARIC_CHECK(job_meta != nullptr, "job_meta is NULL");
    if (scores) {
      DARIC_CHECK(job_score_row && meta_score_col, "scores need job_score_row and meta_score_col");
      DARIC_CHECK(score_ld >= 0, "score_ld must be non-negative");
    }
    std::vector<MetaDev> metas(num_metas);
    for (int64_t m = 0; m < num_metas; ++m) {
      MetaDev& d = metas[m];
      d.pos_a = meta_pos_a[m];
      d.pos_b = mode == DARIC_ROPE_FLEXIBLE ? meta_pos_b[m] : 0;
      d.len = meta_len[m];
      DARIC_CHECK(d.len >= 0, "negative chunk length at chunk " + std::to_string(m));
      d.score_col = scores ? meta_score_col[m] : 0;
      if (scores) DARIC_CHECK(d.score_col >= 0, "negative score column at chunk " + std::to_string(m));
      d.rotate = (mode == DARIC_ROPE_NONE || d.len == 0 ||
                  (mode == DARIC_ROPE_FLEXIBLE && d.pos_a == d.pos_b)) ? 0 : 1;
    }
    // Group jobs by kernel signature (dtype of KV, dtype of table, NeoX).
    std::map<std::tuple<int, int, int>, std::vector<int64_t>> groups;
    for (int64_t i = 0; i < num_jobs; ++i) {
      const LayerHost& L = *jp.layers[i];
      DARIC_CHECK(job_meta[i] >= 0 && job_meta[i] < num_metas,
                  "job_meta out of range at job " + std::to_string(i));
      DARIC_CHECK(L.has_rot || mode == DARIC_ROPE_NONE,
                  "layer has no rotary table (register_rotary): " + L.name);
      if (scores)
        DARIC_CHECK(job_score_row[i] >= 0 && job_score_row[i] <= INT32_MAX,
                    "job_score_row out of range at job " + std::to_string(i));
      groups[{L.has_rot ? L.kv_dtype : -1, L.has_rot ? L.tab_dtype : -1, L.neox}].push_back(i);
    }
    for (auto& [k, idx] : groups) {
      const bool rot = std::get<0>(k) >= 0;
      if (rot) {
        DARIC_CHECK(jp.vec16, "rerotate_scatter_pages needs 16-byte aligned jobs and store offsets");
        run_page_jobs(c, jp, idx, offsets, indices_flat, indices_numel, indices_offsets, false, true,
                      mode, job_meta, metas, scores, score_ld, job_score_row,
                      RotKey{std::get<0>(k), std::get<1>(k), std::get<2>(k)}, (cudaStream_t)stream);
      } else {
        run_page_jobs(c, jp, idx, offsets, indices_flat, indices_numel, indices_offsets, false, false,
                      DARIC_ROPE_NONE, nullptr, {}, nullptr, 0, nullptr, RotKey{}, (cudaStream_t)stream);
      }
    }
  });
}

int daric_copier_load_chunks(daric_copier* c, int64_t num_layers, const char* const* layer_names,
                             int64_t layer_begin, int64_t layer_end, int64_t num_chunks,
                             const int64_t* chunk_stg_off, const int64_t* chunk_blk_off,
                             const int64_t* chunk_pages, const int32_t* block_ids, int64_t block_ids_numel,
                             int block_ids_device, int mode, const int64_t* pos_a, const int64_t* pos_b,
                             const int64_t* len, float* scores, int64_t score_ld, const int64_t* score_col,
                             void* stream) {
  return guarded([&] {
    run_chunk_load(c, num_layers, layer_names, layer_begin, layer_end, num_chunks, chunk_stg_off, chunk_blk_off,
                   chunk_pages, block_ids, block_ids_numel, block_ids_device, mode, pos_a, pos_b, len, scores,
                   score_ld, score_col, (cudaStream_t)stream);
  });
}

int daric_copier_rerotate_inplace(daric_copier* c, int64_t num_layers, const char* const* names, int mode,
                                  int64_t num_segs, const int32_t* block_table, int64_t block_table_numel,
                                  const int64_t* seg_blk_off, const int64_t* seg_tok_start,
                                  const int64_t* seg_tok_len, const int64_t* seg_pos_a,
                                  const int64_t* seg_pos_b, void* stream) {
  return guarded([&] {
    DARIC_CHECK(c, "copier is NULL");
    DARIC_CHECK(mode == DARIC_ROPE_FLEXIBLE || mode == DARIC_ROPE_DELTA,
                "rerotate_inplace: mode must be FLEXIBLE or DELTA");
    if (num_layers <= 0 || num_segs <= 0) return;
    DARIC_CHECK(names && seg_blk_off && seg_tok_start && seg_tok_len && seg_pos_a, "segment arrays are NULL");
    DARIC_CHECK(mode != DARIC_ROPE_FLEXIBLE || seg_pos_b, "FLEXIBLE mode needs seg_pos_b");
    DARIC_CHECK(block_table != nullptr, "block_table is NULL");
    std::vector<LayerHost*> all(num_layers);
    for (int64_t l = 0; l < num_layers; ++l) {
      all[l] = &find_layer(c, names[l]);
      DARIC_CHECK(all[l]->has_rot, "layer has no rotary table (register_rotary): " + all[l]->name);
    }
    const LayerHost& L0 = *all[0];
    for (auto* L : all) {
      DARIC_CHECK(L->device == L0.device, "all layers must be on the same device");
      DARIC_CHECK(L->kv_dtype == L0.kv_dtype && L->neox == L0.neox && L->dev.page_size == L0.dev.page_size,
                  "rerotate_inplace: layers of one call must share dtype, rotary style and block size");
    }
    // one launch per rotary table (the factors of a token depend on the table)
    std::vector<std::vector<LayerHost*>> by_table;
    for (auto* L : all) {
      bool placed = false;
      for (auto& grp : by_table)
        if (grp[0]->dev.table == L->dev.table && grp[0]->dev.half_rot == L->dev.half_rot &&
            grp[0]->tab_dtype == L->tab_dtype) {
          grp.push_back(L);
          placed = true;
          break;
        }
      if (!placed) by_table.push_back({L});
    }
    const int64_t bs = L0.dev.page_size;
    DeviceCtx& dc = device_ctx(L0.device);
    DeviceGuard dg(L0.device);
    for (auto& grp : by_table) {
      const LayerDev& T0 = grp[0]->dev;
      std::vector<LayerDev> ld(grp.size());
      for (size_t l = 0; l < grp.size(); ++l) ld[l] = base_layer_dev(*grp[l]);
      // the copy-engine pipeline reads the factors from the table itself
      // (DELTA: one row per segment), or in FLEXIBLE mode from a factor
      // pre-pass on the side stream (one combination of the two rows per
      // token instead of one per rotation task; DARIC_INPLACE_FACTORS=table
      // keeps the table reads for A/B measurements)
      const InplaceGeom ig = plan_inplace(dc, ld, grp[0]->tab_dtype);
      const int64_t upp = ig.nstage >= 3 ? ig.pages_per_unit : 1;
      const char* fv = std::getenv("DARIC_INPLACE_FACTORS");
      const bool prepass =
          ig.nstage >= 3 && mode == DARIC_ROPE_FLEXIBLE && !(fv && std::strcmp(fv, "table") == 0);
      const bool compact = prepass && grp[0]->tab_dtype == DARIC_DTYPE_BF16;
      std::vector<SegDev> segs;
      std::vector<FacJobDev> runs;
      segs.reserve(num_segs);
      int64_t units = 0, tok = 0, items = 0;
      for (int64_t s = 0; s < num_segs; ++s) {
        DARIC_CHECK(seg_tok_len[s] >= 0 && seg_tok_start[s] >= 0 && seg_blk_off[s] >= 0,
                    "negative segment field at segment " + std::to_string(s));
        if (seg_tok_len[s] == 0) continue;
        SegDev d{};
        d.blk_off = seg_blk_off[s];
        d.tok_start = seg_tok_start[s];
        d.tok_len = seg_tok_len[s];
        d.pos_a = seg_pos_a[s];
        d.pos_b = mode == DARIC_ROPE_FLEXIBLE ? seg_pos_b[s] : 0;
        const bool ok = mode == DARIC_ROPE_FLEXIBLE
                            ? (d.pos_a >= 0 && d.pos_b >= 0 && d.pos_a + d.tok_len <= T0.max_pos &&
                               d.pos_b + d.tok_len <= T0.max_pos)
                            : (d.pos_a >= 0 && d.pos_a < T0.max_pos);
        DARIC_CHECK(ok, "rotary position out of range of cos_sin_cache (max_position=" +
                            std::to_string(T0.max_pos) + ") at segment " + std::to_string(s));
        const int64_t p0 = d.tok_start / bs, p1 = (d.tok_start + d.tok_len - 1) / bs;
        DARIC_CHECK(d.blk_off + p1 < block_table_numel,
                    "segment " + std::to_string(s) + " reaches past the block table");
        DARIC_CHECK(p1 < INT32_MAX, "segment " + std::to_string(s) + " reaches past int32 pages");
        d.first_page = (int32_t)p0;
        d.num_pages = (int32_t)(p1 - p0 + 1);
        d.num_units = (int32_t)((d.num_pages + upp - 1) / upp);
        d.unit_begin = units;
        d.fac_tok = tok;
        units += d.num_units;
        if (ig.nstage < 3 || prepass) {
          FacJobDev f{};
          f.table = T0.table;
          f.table_row = T0.table_row;
          f.pos_a = d.pos_a;
          f.pos_b = d.pos_b;
          f.len = d.tok_len;
          f.out_tok = tok;
          f.item_begin = items;
          f.half_rot = T0.half_rot;
          f.P = T0.pair_vecs;
          runs.push_back(f);
          items += d.tok_len * (T0.half_rot / 2);
          tok += d.tok_len;
        }
        segs.push_back(d);
      }
      if (units == 0) continue;
      Blob b;
      const size_t o_l = b.add(ld.size() * sizeof(LayerDev));
      const size_t o_s = b.add(segs.size() * sizeof(SegDev));
      const size_t o_r = b.add(runs.size() * sizeof(FacJobDev));
      Upload up(dc, b.size);
      std::memcpy(up.host() + o_l, ld.data(), ld.size() * sizeof(LayerDev));
      std::memcpy(up.host() + o_s, segs.data(), segs.size() * sizeof(SegDev));
      if (!runs.empty()) std::memcpy(up.host() + o_r, runs.data(), runs.size() * sizeof(FacJobDev));
      InplaceLaunch p{};
      p.layers = reinterpret_cast<const LayerDev*>(up.dev() + o_l);
      p.num_layers = (int64_t)grp.size();
      p.segs = reinterpret_cast<const SegDev*>(up.dev() + o_s);
      p.num_segs = (int64_t)segs.size();
      p.units_per_layer = units;
      p.block_table = block_table;
      p.block_table_numel = block_table_numel;
      p.mode = mode;
      p.err = dc.err_word;
      const RotKey key{L0.kv_dtype, grp[0]->tab_dtype, L0.neox};
      if (ig.nstage >= 3) {
        std::unique_ptr<FactorPass> lease;
        if (prepass && tok > 0)
          lease = std::make_unique<FactorPass>(dc, (size_t)tok * token_factor_bytes(T0.half_rot, compact),
                                               (cudaStream_t)stream);
        up.send(b.size, (cudaStream_t)stream);
        if (lease) {
          up.also_wait(lease->stream());
          FactorLaunch fl{};
          fl.jobs = reinterpret_cast<const FacJobDev*>(up.dev() + o_r);
          fl.num_jobs = (int64_t)runs.size();
          fl.total_items = items;
          fl.out = reinterpret_cast<float4*>(lease->ptr());
          fl.mode = mode;
          fl.fpv = factors_per_task(L0.kv_dtype, L0.neox != 0);
          fl.compact = compact ? 1 : 0;
          launch_factors(fl, grp[0]->tab_dtype, dc.sm_count, lease->stream());
          lease->launched();
          p.fac = reinterpret_cast<const float4*>(lease->ptr());
        }
        launch_bulk_inplace(p, ig, key, dc.sm_count, (cudaStream_t)stream);
        if (lease) lease->release();
        up.finish((cudaStream_t)stream);
        continue;
      }
      ScratchLease lease(dc, (size_t)tok * T0.half_rot * 8, (cudaStream_t)stream);
      float4* fac = reinterpret_cast<float4*>(lease.ptr());
      up.send(b.size, (cudaStream_t)stream);
      FactorLaunch fl{};
      fl.jobs = reinterpret_cast<const FacJobDev*>(up.dev() + o_r);
      fl.num_jobs = (int64_t)runs.size();
      fl.total_items = items;
      fl.out = fac;
      fl.mode = mode;
      fl.fpv = factors_per_task(L0.kv_dtype, L0.neox != 0);
      launch_factors(fl, grp[0]->tab_dtype, dc.sm_count, (cudaStream_t)stream);
      p.fac = fac;
      launch_rotate_inplace(p, key, dc.sm_count, (cudaStream_t)stream);
      lease.release();
      up.finish((cudaStream_t)stream);
    }
  });
}

int daric_batched_memcpy_d2h(const void* staging, void* host, int64_t n, const int64_t* stg_offsets,
                             const int64_t* host_offsets, const int64_t* sizes, int device, void* stream) {
  return guarded([&] {
    if (n <= 0) return;
    DARIC_CHECK(staging && host && stg_offsets && host_offsets && sizes, "NULL argument");
    DeviceGuard dg(device);
    for (int64_t i = 0; i < n; ++i) {
      DARIC_CHECK(sizes[i] >= 0 && stg_offsets[i] >= 0 && host_offsets[i] >= 0,
                  "negative copy region at " + std::to_string(i));
      if (sizes[i] == 0) continue;
      DARIC_CUDA(cudaMemcpyAsync((uint8_t*)host + host_offsets[i], (const uint8_t*)staging + stg_offsets[i],
                                 (size_t)sizes[i], cudaMemcpyDeviceToHost, (cudaStream_t)stream));
    }
  });
}

int daric_batched_memcpy_h2d(const void* host, void* staging, int64_t n, const int64_t* host_offsets,
                             const int64_t* stg_offsets, const int64_t* sizes, int device, void* stream) {
  return guarded([&] {
    if (n <= 0) return;
    DARIC_CHECK(staging && host && stg_offsets && host_offsets && sizes, "NULL argument");
    DeviceGuard dg(device);
    for (int64_t i = 0; i < n; ++i) {
      DARIC_CHECK(sizes[i] >= 0 && stg_offsets[i] >= 0 && host_offsets[i] >= 0,
                  "negative copy region at " + std::to_string(i));
      if (sizes[i] == 0) continue;
      DARIC_CUDA(cudaMemcpyAsync((uint8_t*)staging + stg_offsets[i], (const uint8_t*)host + host_offsets[i],
                                 (size_t)sizes[i], cudaMemcpyHostToDevice, (cudaStream_t)stream));
    }
  });
}

int daric_score_select(const float* scores, int64_t num_layers, int64_t score_ld, int64_t num_segs,
                       const int64_t* seg_col_off, const int64_t* seg_len, const int64_t* seg_pos0,
                       const int64_t* seg_k, int mode, float threshold, const int32_t* block_table,
                       int64_t block_table_numel, const int64_t* seg_blk_off, int64_t block_size,
                       int32_t* out_idx, int64_t* out_slot, int32_t* out_count, int64_t out_ld,
                       const int64_t* out_off, int device, void* stream) {
  return guarded([&] {
    DARIC_CHECK(mode == DARIC_SELECT_TOPK || mode == DARIC_SELECT_THRESHOLD,
                "unknown selection mode " + std::to_string(mode));
    if (num_layers <= 0 || num_segs <= 0) return;
    DARIC_CHECK(scores && out_idx && out_slot && out_count, "NULL device pointer");
    DARIC_CHECK(seg_col_off && seg_len && seg_pos0 && seg_blk_off && out_off, "NULL segment array");
    DARIC_CHECK(mode != DARIC_SELECT_TOPK || seg_k, "TOPK needs seg_k");
    DARIC_CHECK(block_size > 0, "block_size must be positive");
    DARIC_CHECK(block_table != nullptr || block_table_numel == 0, "block_table is NULL");
    std::vector<SelSegDev> segs(num_segs);
    int64_t max_len = 0;
    for (int64_t s = 0; s < num_segs; ++s) {
      SelSegDev& d = segs[s];
      d.col_off = seg_col_off[s];
      d.len = seg_len[s];
      d.pos0 = seg_pos0[s];
      d.k = mode == DARIC_SELECT_TOPK ? seg_k[s] : 0;
      d.blk_off = seg_blk_off[s];
      d.out_off = out_off[s];
      DARIC_CHECK(d.col_off >= 0 && d.len >= 0 && d.pos0 >= 0 && d.k >= 0 && d.blk_off >= 0 && d.out_off >= 0,
                  "negative segment field at segment " + std::to_string(s));
      DARIC_CHECK(d.col_off + d.len <= score_ld,
                  "segment " + std::to_string(s) + " exceeds the score row (score_ld)");
      DARIC_CHECK(d.pos0 + d.len <= INT32_MAX, "positions exceed int32");
      const int64_t cap = mode == DARIC_SELECT_TOPK ? std::min(d.k, d.len) : d.len;
      DARIC_CHECK(d.out_off + cap <= out_ld, "segment " + std::to_string(s) + " output exceeds out_ld");
      max_len = std::max(max_len, d.len);
    }
    DeviceCtx& dc = device_ctx(device);
    DeviceGuard dg(device);
    Upload up(dc, segs.size() * sizeof(SelSegDev));
    std::memcpy(up.host(), segs.data(), segs.size() * sizeof(SelSegDev));
    up.send(segs.size() * sizeof(SelSegDev), (cudaStream_t)stream);
    SelectLaunch p{};
    p.scores = scores;
    p.num_layers = num_layers;
    p.score_ld = score_ld;
    p.num_segs = num_segs;
    p.segs = reinterpret_cast<const SelSegDev*>(up.dev());
    p.mode = mode;
    p.threshold = threshold;
    p.block_table = block_table;
    p.block_table_numel = block_table_numel;
    p.block_size = block_size;
    p.out_idx = out_idx;
    p.out_slot = out_slot;
    p.out_count = out_count;
    p.out_ld = out_ld;
    p.err = dc.err_word;
    launch_score_select(p, max_len, dc.sm_count, (cudaStream_t)stream);
    up.finish((cudaStream_t)stream);
  });
}

int daric_ptrs_to_slots(int64_t num_ranges, const int64_t* range_start, const int64_t* range_end,
                        const int64_t* range_blk_off, const int32_t* block_table, int64_t block_table_numel,
                        int64_t block_size, int32_t* out_idx, int64_t* out_slot, int device, void* stream) {
  return guarded([&] {
    if (num_ranges <= 0) return;
    DARIC_CHECK(range_start && range_end && range_blk_off, "NULL range array");
    DARIC_CHECK(block_size > 0, "block_size must be positive");
    std::vector<RangeDev> rs;
    rs.reserve(num_ranges);
    int64_t total = 0;
    for (int64_t r = 0; r < num_ranges; ++r) {
      DARIC_CHECK(range_start[r] >= 0 && range_blk_off[r] >= 0, "negative range field at " + std::to_string(r));
      DARIC_CHECK(range_end[r] <= INT32_MAX, "positions exceed int32");
      if (range_end[r] <= range_start[r]) continue;
      rs.push_back(RangeDev{range_start[r], range_end[r], range_blk_off[r], total});
      total += range_end[r] - range_start[r];
    }
    if (total == 0) return;
    DARIC_CHECK(out_idx && out_slot && block_table, "NULL device pointer");
    DeviceCtx& dc = device_ctx(device);
    DeviceGuard dg(device);
    Upload up(dc, rs.size() * sizeof(RangeDev));
    std::memcpy(up.host(), rs.data(), rs.size() * sizeof(RangeDev));
    up.send(rs.size() * sizeof(RangeDev), (cudaStream_t)stream);
    RangeLaunch p{};
    p.ranges = reinterpret_cast<const RangeDev*>(up.dev());
    p.num_ranges = (int64_t)rs.size();
    p.total = total;
    p.block_table = block_table;
    p.block_table_numel = block_table_numel;
    p.block_size = block_size;
    p.out_idx = out_idx;
    p.out_slot = out_slot;
    p.err = dc.err_word;
    launch_ranges_to_slots(p, (cudaStream_t)stream);
    up.finish((cudaStream_t)stream);
  });
}

}  // extern "C"
