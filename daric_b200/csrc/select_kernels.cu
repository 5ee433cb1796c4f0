// Recompute-selection kernels.
//
//  * select_kernel : per (segment, layer) a thread-block cluster of C CTAs
//    (C = 1..8, picked by the host so that short calls still fill the SMs);
//    CTA r of the cluster owns the r-th contiguous slice of the segment's
//    columns and stages its order-preserving 32-bit keys in shared memory.
//    Radix select of the k highest fp32 scores: four 8-bit digit passes, each
//    a per-warp histogram of the slice merged per CTA, then over the cluster
//    through distributed shared memory; every CTA derives the same digit.
//    One exchange of per-CTA counts (keys above the k-th key, keys equal to
//    it) then orders a stable compaction in token order (warp ballots + block
//    scans) that emits the recompute positions and their paged-KV slots.
//    Threshold mode skips the radix passes. Ties at the k-th score go to the
//    lower token index.
//  * ranges_kernel : expands [start, end) ranges of the DARIC policy
//    (daric/adaption/policy.py:45-103) into positions and slots, the slot
//    formula of the recompute sub-requests (integration/vllm/worker.py:310-346):
//    slot = block_ids[p // bs] * bs + p % bs.
#include <cooperative_groups.h>

#include <cstdlib>
#include <mutex>
#include <set>

#include "internal.h"

namespace daric {
namespace {
namespace cg = cooperative_groups;

constexpr int kSelThreads = 256;  // 4 CTAs per SM (64 registers a thread)
constexpr int kSelWarps = kSelThreads / 32;
constexpr int kMaxCluster = 8;

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

// Slices of up to kSmemKeys keys are staged in shared memory (one read of
// the scores); longer slices are re-read from global memory (L2) per pass.
constexpr int kSmemKeys = 12288;

__device__ __forceinline__ uint32_t key_at(const float* row, const uint32_t* skeys, bool staged, int64_t i) {
  return staged ? skeys[i] : score_key(row[i]);
}

// Columns of a segment of n keys owned by each CTA of a cluster of C.
__host__ __device__ inline int64_t select_slice(int64_t n, int C) { return ((n + C - 1) / C + 31) & ~(int64_t)31; }

__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }

__global__ void __launch_bounds__(kSelThreads, 4) select_kernel(SelectLaunch p) {
  __shared__ uint32_t whist[kSelWarps][256];  // per-warp digit histograms
  __shared__ uint32_t lhist[2][256];          // this slice's histogram, by pass parity (read by the cluster)
  __shared__ uint32_t ghist[256];             // the segment's histogram (sum over the cluster)
  __shared__ long long s_cnt[2];              // this slice: keys above the k-th key, keys equal to it
  __shared__ int scan_sm[32];
  __shared__ uint32_t s_digit, s_above, s_lab;
  extern __shared__ uint32_t skeys[];

  cg::cluster_group cluster = cg::this_cluster();
  const int C = (int)cluster.num_blocks();
  const int me = (int)cluster.block_rank();
  const int64_t si = blockIdx.x / C, l = blockIdx.y;
  const SelSegDev sg = p.segs[si];
  const int64_t n_all = sg.len;
  const int64_t chunk = select_slice(n_all, C);
  const int64_t s0 = min(n_all, (int64_t)me * chunk);
  const int64_t n = min(n_all - s0, chunk);  // this CTA's slice [s0, s0 + n)
  const float* row = p.scores + l * p.score_ld + sg.col_off + s0;
  int32_t* oidx = p.out_idx + l * p.out_ld + sg.out_off;
  int64_t* oslot = p.out_slot + l * p.out_ld + sg.out_off;
  const bool topk = p.mode == DARIC_SELECT_TOPK;
  const bool staged = n <= p.smem_keys;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;

  // Every branch below that skips cluster barriers depends only on the
  // segment (k, n_all, mode), so the CTAs of a cluster take it together.
  uint32_t thr = 0;     // k-th largest key (top-k)
  int64_t take_eq = 0;  // keys equal to thr that are taken, lowest index first
  bool take_all = false;
  long long my_sel = 0, my_eq = 0;
  if (topk) {
    const int64_t k = sg.k < n_all ? sg.k : n_all;
    if (k <= 0) {
      if (me == 0 && threadIdx.x == 0) p.out_count[l * p.num_segs + si] = 0;
      return;
    }
    take_all = (k == n_all);
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
      uint32_t* wh = whist[warp];
      for (int pass = 0; pass < 4; ++pass) {
        const int shift = 24 - 8 * pass;
        uint32_t* lh = lhist[pass & 1];
        for (int b = threadIdx.x; b < kSelWarps * 256; b += blockDim.x) (&whist[0][0])[b] = 0;
        __syncthreads();
        for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
          const uint32_t key = key_at(row, skeys, staged, i);
          if ((key & mask) == prefix) atomicAdd(&wh[(key >> shift) & 255u], 1u);
        }
        __syncthreads();
        for (int b = threadIdx.x; b < 256; b += blockDim.x) {
          uint32_t t = 0;
#pragma unroll
          for (int w = 0; w < kSelWarps; ++w) t += whist[w][b];
          lh[b] = t;
        }
        // lhist[pass & 1] of every CTA is complete after this barrier; the
        // buffer is rewritten two passes later, after the next barrier, which
        // no CTA reaches before it finished reading this one.
        cluster.sync();
        for (int b = threadIdx.x; b < 256; b += blockDim.x) {
          uint32_t t = 0;
          for (int r = 0; r < C; ++r) t += cluster.map_shared_rank(lh, r)[b];
          ghist[b] = t;
        }
        __syncthreads();
        if (warp == 0) {
          // lane L owns digits [248-8L, 255-8L], scanned from the top.
          uint32_t cnt[8], sum = 0;
#pragma unroll
          for (int q = 0; q < 8; ++q) { cnt[q] = ghist[255 - 8 * lane - q]; sum += cnt[q]; }
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
          __syncwarp();
          // this slice's keys in the digits above the chosen one
          const uint32_t d = s_digit;
          uint32_t la = 0;
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const uint32_t dd = 255 - 8 * lane - q;
            if (dd > d) la += lh[dd];
          }
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) la += __shfl_xor_sync(0xffffffffu, la, o);
          if (lane == 0) s_lab = la;
        }
        __syncthreads();
        prefix |= s_digit << shift;
        mask |= 255u << shift;
        rem -= s_above;
        my_sel += s_lab;
        if (pass == 3) my_eq = lh[s_digit];
        __syncthreads();
      }
      thr = prefix;
      take_eq = rem;
    } else {
      my_sel = n;
    }
  } else {
    int c = 0;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) c += row[i] >= p.threshold;
    int tot;
    block_scan(c, &tot, scan_sm);
    my_sel = tot;
  }

  // Counts of the lower-ranked slices give this slice's first output and the
  // rank of its first tied key. The arrive below follows this CTA's last
  // read of a peer's shared memory; the wait at the end keeps this CTA's
  // shared memory alive until every peer has read it.
  if (threadIdx.x == 0) {
    s_cnt[0] = my_sel;
    s_cnt[1] = my_eq;
  }
  cluster.sync();
  long long sel_before = 0, eq_before = 0;
  for (int r = 0; r < me; ++r) {
    const long long* pc = cluster.map_shared_rank(s_cnt, r);
    sel_before += pc[0];
    eq_before += pc[1];
  }
  cluster_arrive();

  // Compaction in token order: warp w owns the 256 consecutive keys
  // [c0 + 256w, c0 + 256(w+1)) of each span, as 8 rounds of 32 (lane = key),
  // so ballots give in-warp ranks and one block scan orders the warps.
  const bool use_keys = topk && !take_all;
  const uint32_t lt_mask = (1u << lane) - 1u;
  constexpr int R = 8;
  const int64_t span = (int64_t)kSelWarps * 32 * R;
  int64_t running = sel_before + (use_keys ? min((int64_t)eq_before, take_eq) : 0);
  int64_t eq_seen = eq_before;
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
        const int64_t pos = sg.pos0 + s0 + i;
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
  if (me == C - 1 && threadIdx.x == 0) p.out_count[l * p.num_segs + si] = (int32_t)running;
  cluster_wait();
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

// Cluster size of a call: grow C (up to 8) while a slice does not fit the
// key stage, or while the call has fewer than two CTAs per SM and slices
// stay at 2048 keys or more. DARIC_SELECT_CLUSTER pins it for measurements.
int select_cluster(int64_t items, int64_t max_len, int sm_count) {
  if (const char* v = std::getenv("DARIC_SELECT_CLUSTER")) {  // diagnostic override (1, 2, 4, 8)
    const int want = std::atoi(v);
    if ((want == 1 || want == 2 || want == 4 || want == 8) && select_slice(max_len, want) <= kSmemKeys * 8)
      return want;
  }
  int C = 1;
  while (C < kMaxCluster) {
    const bool too_long = select_slice(max_len, C) > kSmemKeys;
    const bool few = items * C < 2 * (int64_t)sm_count && select_slice(max_len, 2 * C) >= 2048;
    if (!too_long && !few) break;
    C *= 2;
  }
  return C;
}

// Launch with the cluster size in p.cluster; dynamic shared memory holds the
// largest slice (at most kSmemKeys keys). Allocates nothing.
cudaError_t launch_select_cluster(const SelectLaunch& p, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(p.num_segs * p.cluster), (unsigned)p.num_layers, 1);
  cfg.blockDim = dim3(kSelThreads, 1, 1);
  cfg.dynamicSmemBytes = (size_t)p.smem_keys * sizeof(uint32_t);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)p.cluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, select_kernel, p);
}

}  // namespace

void launch_score_select(SelectLaunch p, int64_t max_len, int sm_count, cudaStream_t s) {
  if (p.num_segs <= 0 || p.num_layers <= 0) return;
  DARIC_CHECK(p.num_layers <= 65535, "score_select: at most 65535 layers per call");
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
  p.cluster = select_cluster(p.num_segs * p.num_layers, max_len, sm_count);
  p.smem_keys = (int32_t)std::min<int64_t>(kSmemKeys, select_slice(max_len, p.cluster));
  DARIC_CUDA(launch_select_cluster(p, s));
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
// Descriptors per writer launch: they travel as the writer kernel's
// parameters (24 KiB of the 32 KiB parameter space), so a call's
// descriptors are fixed when its launch is enqueued and no host memory is
// read later.
constexpr int kNoallocBatch = 512;
static_assert(kNoallocMaxSegs % kNoallocBatch == 0, "whole writer batches");
}  // namespace

// [kNoallocMaxSegs descriptors][256 bytes: device error word]. In host code
// this name only stands in for the array; its device address comes from
// cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_select_scratch[kNoallocSegBytes + 256];

namespace {

struct NoallocBatch {
  int32_t first;     // first descriptor of the batch
  int32_t count;     // descriptors in the batch
  int32_t clear_err; // 1: the batch also zeroes the error word
  int32_t pad;
  daric::SelSegDev seg[kNoallocBatch];
};

// Writes one batch of descriptors (the launch parameters) into the fixed
// array; the first batch of a call also zeroes the error word.
__global__ void __launch_bounds__(256) noalloc_put_descs(const __grid_constant__ NoallocBatch b) {
  daric::SelSegDev* dst = reinterpret_cast<daric::SelSegDev*>(g_select_scratch) + b.first;
  for (int i = threadIdx.x; i < b.count; i += blockDim.x) dst[i] = b.seg[i];
  if (b.clear_err && threadIdx.x == 0) *reinterpret_cast<int*>(g_select_scratch + kNoallocSegBytes) = 0;
}

std::mutex g_noalloc_mu;                                // guards the set-up and the batch buffers
NoallocBatch g_noalloc_batch[kNoallocMaxSegs / kNoallocBatch];  // host side of one call's launches
unsigned char* g_noalloc_dev[kNoallocMaxDevices];       // device address of the array, per device
int g_noalloc_sms[kNoallocMaxDevices];                  // SM count, per device

// Set-up, once per device, with that device current: the array's device
// address, the SM count and the kernel's dynamic shared-memory limit.
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
  e = cudaDeviceGetAttribute(&g_noalloc_sms[device], cudaDevAttrMultiProcessorCount, device);
  if (e != cudaSuccess)
    throw daric::Error(DARIC_ERR_CUDA, std::string("cudaDeviceGetAttribute failed: ") + cudaGetErrorString(e));
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
  int64_t max_len = 0;
  for (int64_t s = 0; s < num_segs; ++s) {
    daric::SelSegDev& d = g_noalloc_batch[s / kNoallocBatch].seg[s % kNoallocBatch];
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
    if (d.len > max_len) max_len = d.len;
  }
  // The descriptors go to the device as kernel parameters (copied when the
  // launch is enqueued), so the host buffers are free for the next call as
  // soon as this one returns. The first batch also zeroes the error word.
  for (int64_t b0 = 0; b0 < num_segs; b0 += kNoallocBatch) {
    NoallocBatch& nb = g_noalloc_batch[b0 / kNoallocBatch];
    nb.first = (int32_t)b0;
    nb.count = (int32_t)(num_segs - b0 < kNoallocBatch ? num_segs - b0 : kNoallocBatch);
    nb.clear_err = b0 == 0 ? 1 : 0;
    nb.pad = 0;
    noalloc_put_descs<<<1, 256, 0, stream>>>(nb);
    const cudaError_t le = cudaGetLastError();
    if (le != cudaSuccess)
      throw Error(DARIC_ERR_CUDA, std::string("noalloc select descriptors: ") + cudaGetErrorString(le));
  }
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
  p.cluster = daric::select_cluster(num_segs * num_layers, max_len, g_noalloc_sms[device]);
  const int64_t slice = daric::select_slice(max_len, p.cluster);
  p.smem_keys = (int32_t)(slice < daric::kSmemKeys ? slice : daric::kSmemKeys);
  const cudaError_t e = daric::launch_select_cluster(p, stream);
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
