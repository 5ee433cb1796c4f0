// Recompute-selection kernels.
//
//  * select_kernel : per (segment, layer) CTA, radix select of the k highest
//    fp32 scores (8-bit digits, four histogram passes over an order-preserving
//    32-bit key held in shared memory; per-warp histograms merged per pass),
//    then a stable compaction in token order (warp ballots + one block scan)
//    that emits the recompute positions and their paged-KV slots. Threshold
//    mode skips the radix passes. Ties at the k-th score go to the lower
//    token index.
//  * ranges_kernel : expands [start, end) ranges of the DARIC policy
//    (daric/adaption/policy.py:45-103) into positions and slots, the slot
//    formula of the recompute sub-requests (integration/vllm/worker.py:310-346):
//    slot = block_ids[p // bs] * bs + p % bs.
#include <mutex>
#include <set>

#include "internal.h"

namespace daric {
namespace {

constexpr int kSelThreads = 512;
constexpr int kSelWarps = kSelThreads / 32;

// Order-preserving key: larger float -> larger key. Every NaN maps to the
// largest key (NaN ranks above +inf, as torch.topk orders it).
__device__ __forceinline__ uint32_t score_key(float f) {
  if (f != f) return 0xFFFFFFFFu;
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Exclusive block-wide prefix sum of v; *total receives the block sum.
__device__ __forceinline__ int block_scan(int v, int* total, int* sm) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  __syncthreads();  // protect sm from a previous call
  if (lane == 31) sm[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = lane < kSelWarps ? sm[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < kSelWarps) sm[lane] = w;  // inclusive warp totals
  }
  __syncthreads();
  *total = sm[kSelWarps - 1];
  return x - v + (warp > 0 ? sm[warp - 1] : 0);
}

// Rows of up to kSmemKeys keys are staged in shared memory (one read of the
// scores); longer rows are re-read from global memory (L2) on every pass.
constexpr int kSmemKeys = 12288;

__device__ __forceinline__ uint32_t key_at(const float* row, const uint32_t* skeys, bool staged, int64_t i) {
  return staged ? skeys[i] : score_key(row[i]);
}

__global__ void __launch_bounds__(kSelThreads) select_kernel(SelectLaunch p) {
  __shared__ uint32_t whist[kSelWarps][256];  // per-warp digit histograms
  __shared__ uint32_t hist[256];
  __shared__ int scan_sm[32];
  __shared__ uint32_t s_digit, s_above;
  extern __shared__ uint32_t skeys[];

  const int64_t si = blockIdx.x, l = blockIdx.y;
  const SelSegDev sg = p.segs[si];
  const float* row = p.scores + l * p.score_ld + sg.col_off;
  const int64_t n = sg.len;
  int32_t* oidx = p.out_idx + l * p.out_ld + sg.out_off;
  int64_t* oslot = p.out_slot + l * p.out_ld + sg.out_off;
  const bool topk = p.mode == DARIC_SELECT_TOPK;
  const bool staged = n <= kSmemKeys;
  const int warp_id = threadIdx.x >> 5;

  uint32_t thr = 0;     // k-th largest key (top-k)
  int64_t take_eq = 0;  // keys equal to thr that are taken, lowest index first
  bool take_all = false;
  if (topk) {
    const int64_t k = sg.k < n ? sg.k : n;
    if (k <= 0) {
      if (threadIdx.x == 0) p.out_count[l * p.num_segs + si] = 0;
      return;
    }
    take_all = (k == n);
    if (!take_all) {
      if (staged) {  // all loads of a batch in flight before any key is stored
        constexpr int kBatch = 8;
        for (int64_t b0 = threadIdx.x; b0 < n; b0 += (int64_t)kBatch * blockDim.x) {
          float v[kBatch];
#pragma unroll
          for (int u = 0; u < kBatch; ++u) {
            const int64_t i = b0 + (int64_t)u * blockDim.x;
            v[u] = i < n ? __ldg(&row[i]) : 0.f;
          }
#pragma unroll
          for (int u = 0; u < kBatch; ++u) {
            const int64_t i = b0 + (int64_t)u * blockDim.x;
            if (i < n) skeys[i] = score_key(v[u]);
          }
        }
      }
      uint32_t prefix = 0, mask = 0;
      int64_t rem = k;
      const int lane = threadIdx.x & 31;
      for (int shift = 24; shift >= 0; shift -= 8) {
        for (int b = threadIdx.x; b < kSelWarps * 256; b += blockDim.x) (&whist[0][0])[b] = 0;
        __syncthreads();
        uint32_t* wh = whist[warp_id];
        for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
          const uint32_t key = key_at(row, skeys, staged, i);
          if ((key & mask) == prefix) atomicAdd(&wh[(key >> shift) & 255u], 1u);
        }
        __syncthreads();
        for (int b = threadIdx.x; b < 256; b += blockDim.x) {
          uint32_t t = 0;
#pragma unroll
          for (int w = 0; w < kSelWarps; ++w) t += whist[w][b];
          hist[b] = t;
        }
        __syncthreads();
        if (threadIdx.x < 32) {
          // lane L owns digits [248-8L, 255-8L], scanned from the top.
          uint32_t cnt[8], sum = 0;
#pragma unroll
          for (int q = 0; q < 8; ++q) { cnt[q] = hist[255 - 8 * lane - q]; sum += cnt[q]; }
          uint32_t incl = sum;
#pragma unroll
          for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += y;
          }
          const uint32_t excl = incl - sum;
          if (excl < (uint64_t)rem && (uint64_t)rem <= incl) {
            uint32_t acc = excl;
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              if (acc < (uint64_t)rem && (uint64_t)rem <= (uint64_t)acc + cnt[q]) {
                s_digit = 255 - 8 * lane - q;
                s_above = acc;
              }
              acc += cnt[q];
            }
          }
        }
        __syncthreads();
        prefix |= s_digit << shift;
        mask |= 255u << shift;
        rem -= s_above;
        __syncthreads();
      }
      thr = prefix;
      take_eq = rem;
    }
  }

  // Compaction in token order: warp w owns the 512 consecutive keys
  // [c0 + 512w, c0 + 512(w+1)) of each pass, as 16 rounds of 32 (lane = key),
  // so ballots give in-warp ranks and one block scan orders the warps.
  const bool use_keys = topk && !take_all;
  const int lane = threadIdx.x & 31, warp = warp_id;
  const uint32_t lt_mask = (1u << lane) - 1u;
  constexpr int R = 16;
  const int64_t span = (int64_t)kSelWarps * 32 * R;
  int64_t running = 0, eq_seen = 0;
  for (int64_t c0 = 0; c0 < n; c0 += span) {
    const int64_t wb = c0 + (int64_t)warp * 32 * R;
    uint32_t selm[R], eqm[R];
    int sel_cnt = 0, eq_cnt = 0;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int64_t i = wb + r * 32 + lane;
      bool sel = false, eq = false;
      if (i < n) {
        if (!topk) {
          sel = row[i] >= p.threshold;
        } else if (take_all) {
          sel = true;
        } else {
          const uint32_t key = key_at(row, skeys, staged, i);
          sel = key > thr;
          eq = key == thr;
        }
      }
      selm[r] = __ballot_sync(0xffffffffu, sel);
      eqm[r] = __ballot_sync(0xffffffffu, eq);
      sel_cnt += __popc(selm[r]);
      eq_cnt += __popc(eqm[r]);
    }
    if (use_keys) {
      int eq_tot;
      const int eq_off = __shfl_sync(0xffffffffu, block_scan(lane == 0 ? eq_cnt : 0, &eq_tot, scan_sm), 0);
      // the lowest-index keys equal to thr are taken
      int64_t rank = eq_seen + eq_off;
      sel_cnt = 0;
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const bool mine = (eqm[r] >> lane) & 1u;
        const bool take = mine && rank + __popc(eqm[r] & lt_mask) < take_eq;
        selm[r] |= __ballot_sync(0xffffffffu, take);
        rank += __popc(eqm[r]);
        sel_cnt += __popc(selm[r]);
      }
      eq_seen += eq_tot;
    }
    int sel_tot;
    int64_t o = running + __shfl_sync(0xffffffffu, block_scan(lane == 0 ? sel_cnt : 0, &sel_tot, scan_sm), 0);
#pragma unroll
    for (int r = 0; r < R; ++r) {
      if ((selm[r] >> lane) & 1u) {
        const int64_t i = wb + r * 32 + lane;
        const int64_t at = o + __popc(selm[r] & lt_mask);
        const int64_t pos = sg.pos0 + i;
        const int64_t bt = sg.blk_off + pos / p.block_size;
        int64_t slot = -1;
        if (bt >= 0 && bt < p.block_table_numel) {
          slot = (int64_t)__ldg(&p.block_table[bt]) * p.block_size + pos % p.block_size;
        } else {
          atomicOr(p.err, DEV_ERR_INDEX_RANGE);
        }
        oidx[at] = (int32_t)pos;
        oslot[at] = slot;
      }
      o += __popc(selm[r]);
    }
    running += sel_tot;
  }
  if (threadIdx.x == 0) p.out_count[l * p.num_segs + si] = (int32_t)running;
}

__global__ void ranges_kernel(RangeLaunch p) {
  for (int64_t o = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; o < p.total;
       o += (int64_t)gridDim.x * blockDim.x) {
    int64_t lo = 0, hi = p.num_ranges - 1;
    while (lo < hi) {
      const int64_t mid = (lo + hi + 1) >> 1;
      if (__ldg(&p.ranges[mid].out_begin) <= o) lo = mid; else hi = mid - 1;
    }
    const RangeDev r = p.ranges[lo];
    const int64_t pos = r.start + (o - r.out_begin);
    const int64_t bt = r.blk_off + pos / p.block_size;
    int64_t slot = -1;
    if (bt >= 0 && bt < p.block_table_numel) {
      slot = (int64_t)__ldg(&p.block_table[bt]) * p.block_size + pos % p.block_size;
    } else {
      atomicOr(p.err, DEV_ERR_INDEX_RANGE);
    }
    p.out_idx[o] = (int32_t)pos;
    p.out_slot[o] = slot;
  }
}

}  // namespace

void launch_score_select(const SelectLaunch& p, cudaStream_t s) {
  if (p.num_segs <= 0 || p.num_layers <= 0) return;
  DARIC_CHECK(p.num_layers <= 65535, "score_select: at most 65535 layers per call");
  const dim3 grid((unsigned)p.num_segs, (unsigned)p.num_layers, 1);
  {
    static std::mutex mu;
    static std::set<int> done;  // devices whose function attribute is set
    int dev = 0;
    DARIC_CUDA(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> g(mu);
    if (!done.count(dev)) {
      DARIC_CUDA(cudaFuncSetAttribute(select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      kSmemKeys * (int)sizeof(uint32_t)));
      done.insert(dev);
    }
  }
  select_kernel<<<grid, kSelThreads, kSmemKeys * sizeof(uint32_t), s>>>(p);
  DARIC_CUDA(cudaGetLastError());
}

void launch_ranges_to_slots(const RangeLaunch& p, cudaStream_t s) {
  if (p.total <= 0) return;
  const int threads = 256;
  int64_t blocks = (p.total + threads - 1) / threads;
  if (blocks > 65535) blocks = 65535;
  ranges_kernel<<<(unsigned)blocks, threads, 0, s>>>(p);
  DARIC_CUDA(cudaGetLastError());
}

}  // namespace daric

// ---------------------------------------------------------------------------
// daric_score_select_noalloc: the selection above for callers that must not
// allocate device memory once running (a serving process whose free device
// memory all went to its KV cache at start-up, or a host whose memory pool
// owns every device allocation). The per-request descriptors, which
// daric_score_select keeps in library-allocated scratch, live in the fixed
// file-scope array below; the call allocates nothing (no cudaMalloc /
// cudaFree, no host containers on the success path).
// ---------------------------------------------------------------------------
namespace {
constexpr int kNoallocMaxSegs = DARIC_NOALLOC_MAX_SEGMENTS;
constexpr size_t kNoallocSegBytes = (size_t)kNoallocMaxSegs * sizeof(daric::SelSegDev);  // 48 KiB
constexpr int kNoallocMaxDevices = 64;
}  // namespace

// [kNoallocMaxSegs descriptors][256 bytes: device error word]. In host code
// this name only stands in for the array; its device address comes from
// cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_select_scratch[kNoallocSegBytes + 256];

namespace {

std::mutex g_noalloc_mu;                              // guards the host staging and set-up
daric::SelSegDev g_noalloc_host[kNoallocMaxSegs];     // host staging of one call's descriptors
unsigned char* g_noalloc_dev[kNoallocMaxDevices];     // device address of the array, per device

// Set-up, once per device, with that device current: the array's device
// address and the kernel's dynamic shared-memory limit.
unsigned char* noalloc_scratch(int device) {
  if (g_noalloc_dev[device]) return g_noalloc_dev[device];
  void* ptr = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&ptr, g_select_scratch);
  if (e != cudaSuccess || ptr == nullptr)
    throw daric::Error(DARIC_ERR_CUDA, std::string("cudaGetSymbolAddress failed: ") + cudaGetErrorString(e));
  e = cudaFuncSetAttribute(daric::select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           daric::kSmemKeys * (int)sizeof(uint32_t));
  if (e != cudaSuccess)
    throw daric::Error(DARIC_ERR_CUDA, std::string("cudaFuncSetAttribute failed: ") + cudaGetErrorString(e));
  g_noalloc_dev[device] = static_cast<unsigned char*>(ptr);
  return g_noalloc_dev[device];
}

void select_noalloc(const float* scores, int64_t num_layers, int64_t score_ld, int64_t num_segs,
                    const int64_t* seg_col_off, const int64_t* seg_len, const int64_t* seg_pos0,
                    const int64_t* seg_k, int mode, float threshold, const int32_t* block_table,
                    int64_t block_table_numel, const int64_t* seg_blk_off, int64_t block_size, int32_t* out_idx,
                    int64_t* out_slot, int32_t* out_count, int64_t out_ld, const int64_t* out_off, int device,
                    cudaStream_t stream) {
  using daric::Error;
  DARIC_CHECK(mode == DARIC_SELECT_TOPK || mode == DARIC_SELECT_THRESHOLD, "unknown selection mode");
  if (num_layers <= 0 || num_segs <= 0) return;
  DARIC_CHECK(num_segs <= kNoallocMaxSegs,
              "daric_score_select_noalloc: " + std::to_string(num_segs) +
                  " segments exceed its fixed scratch of DARIC_NOALLOC_MAX_SEGMENTS = " +
                  std::to_string(kNoallocMaxSegs));
  DARIC_CHECK(num_layers <= 65535, "score_select: at most 65535 layers per call");
  DARIC_CHECK(device >= 0 && device < kNoallocMaxDevices, "device index out of range");
  DARIC_CHECK(scores && out_idx && out_slot && out_count, "NULL device pointer");
  DARIC_CHECK(seg_col_off && seg_len && seg_pos0 && seg_blk_off && out_off, "NULL segment array");
  DARIC_CHECK(mode != DARIC_SELECT_TOPK || seg_k, "TOPK needs seg_k");
  DARIC_CHECK(block_size > 0, "block_size must be positive");
  DARIC_CHECK(block_table != nullptr || block_table_numel == 0, "block_table is NULL");
  int prev = -1;
  if (cudaGetDevice(&prev) != cudaSuccess) throw Error(DARIC_ERR_CUDA, "cudaGetDevice failed");
  if (prev != device && cudaSetDevice(device) != cudaSuccess) throw Error(DARIC_ERR_CUDA, "cudaSetDevice failed");
  struct Restore {
    int d, p;
    ~Restore() { if (d != p && p >= 0) cudaSetDevice(p); }
  } restore{device, prev};
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  unsigned char* scratch = noalloc_scratch(device);
  for (int64_t s = 0; s < num_segs; ++s) {
    daric::SelSegDev& d = g_noalloc_host[s];
    d.col_off = seg_col_off[s];
    d.len = seg_len[s];
    d.pos0 = seg_pos0[s];
    d.k = mode == DARIC_SELECT_TOPK ? seg_k[s] : 0;
    d.blk_off = seg_blk_off[s];
    d.out_off = out_off[s];
    DARIC_CHECK(d.col_off >= 0 && d.len >= 0 && d.pos0 >= 0 && d.k >= 0 && d.blk_off >= 0 && d.out_off >= 0,
                "negative segment field at segment " + std::to_string(s));
    DARIC_CHECK(d.col_off + d.len <= score_ld, "segment " + std::to_string(s) + " exceeds the score row (score_ld)");
    DARIC_CHECK(d.pos0 + d.len <= INT32_MAX, "positions exceed int32");
    const int64_t cap = mode == DARIC_SELECT_TOPK ? (d.k < d.len ? d.k : d.len) : d.len;
    DARIC_CHECK(d.out_off + cap <= out_ld, "segment " + std::to_string(s) + " output exceeds out_ld");
  }
  // Pageable source: the copy is staged by the driver before it returns, so
  // the host staging can be reused by the next call right away. The error
  // word starts at zero on every call.
  cudaError_t e = cudaMemcpyAsync(scratch, g_noalloc_host, (size_t)num_segs * sizeof(daric::SelSegDev),
                                  cudaMemcpyHostToDevice, stream);
  if (e == cudaSuccess) e = cudaMemsetAsync(scratch + kNoallocSegBytes, 0, sizeof(int), stream);
  if (e != cudaSuccess) throw Error(DARIC_ERR_CUDA, std::string("noalloc select copy: ") + cudaGetErrorString(e));
  daric::SelectLaunch p{};
  p.scores = scores;
  p.num_layers = num_layers;
  p.score_ld = score_ld;
  p.num_segs = num_segs;
  p.segs = reinterpret_cast<const daric::SelSegDev*>(scratch);
  p.mode = mode;
  p.threshold = threshold;
  p.block_table = block_table;
  p.block_table_numel = block_table_numel;
  p.block_size = block_size;
  p.out_idx = out_idx;
  p.out_slot = out_slot;
  p.out_count = out_count;
  p.out_ld = out_ld;
  p.err = reinterpret_cast<int*>(scratch + kNoallocSegBytes);
  const dim3 grid((unsigned)num_segs, (unsigned)num_layers, 1);
  daric::select_kernel<<<grid, daric::kSelThreads, daric::kSmemKeys * sizeof(uint32_t), stream>>>(p);
  e = cudaGetLastError();
  if (e != cudaSuccess) throw Error(DARIC_ERR_CUDA, std::string("noalloc select launch: ") + cudaGetErrorString(e));
}

}  // namespace

extern "C" int daric_score_select_noalloc(const float* scores, int64_t num_layers, int64_t score_ld,
                                          int64_t num_segs, const int64_t* seg_col_off, const int64_t* seg_len,
                                          const int64_t* seg_pos0, const int64_t* seg_k, int mode, float threshold,
                                          const int32_t* block_table, int64_t block_table_numel,
                                          const int64_t* seg_blk_off, int64_t block_size, int32_t* out_idx,
                                          int64_t* out_slot, int32_t* out_count, int64_t out_ld,
                                          const int64_t* out_off, int device, void* stream) {
  try {
    select_noalloc(scores, num_layers, score_ld, num_segs, seg_col_off, seg_len, seg_pos0, seg_k, mode, threshold,
                   block_table, block_table_numel, seg_blk_off, block_size, out_idx, out_slot, out_count, out_ld,
                   out_off, device, (cudaStream_t)stream);
    daric::clear_error();
    return DARIC_OK;
  } catch (const daric::Error& err) {
    daric::record_error(err.code, err.what());
    return err.code;
  } catch (const std::exception& err) {
    daric::record_error(DARIC_ERR_STATE, err.what());
    return DARIC_ERR_STATE;
  }
}
