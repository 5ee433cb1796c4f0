// Recompute-selection kernels.
//
//  * select_kernel : per (segment, layer) CTA, radix select of the k highest
//    fp32 scores (8-bit digits, four histogram passes over an order-preserving
//    32-bit key), then a stable compaction in token order that emits the
//    recompute positions and their paged-KV slots. Threshold mode skips the
//    radix passes. Ties at the k-th score go to the lower token index.
//  * ranges_kernel : expands [start, end) ranges of the DARIC policy
//    (daric/adaption/policy.py:45-103) into positions and slots, the slot
//    formula of the recompute sub-requests (integration/vllm/worker.py:310-346):
//    slot = block_ids[p // bs] * bs + p % bs.
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

__global__ void __launch_bounds__(kSelThreads) select_kernel(SelectLaunch p) {
  __shared__ uint32_t hist[256];
  __shared__ int scan_sm[32];
  __shared__ uint32_t s_digit, s_above;

  const int64_t si = blockIdx.x, l = blockIdx.y;
  const SelSegDev sg = p.segs[si];
  const float* row = p.scores + l * p.score_ld + sg.col_off;
  const int64_t n = sg.len;
  int32_t* oidx = p.out_idx + l * p.out_ld + sg.out_off;
  int64_t* oslot = p.out_slot + l * p.out_ld + sg.out_off;
  const bool topk = p.mode == DARIC_SELECT_TOPK;

  uint32_t thr = 0;     // k-th largest key (top-k)
  int64_t take_eq = 0;  // keys equal to thr that are taken, lowest index first
  bool take_all = false;
  if (topk) {
    const int64_t k = sg.k < n ? sg.k : n;
    if (k <= 0) {
      if (threadIdx.x == 0) p.out_count[l * p.num_segs + si] = 0;
      return;
    }
    if (k == n) {
      take_all = true;
    } else {
      uint32_t prefix = 0, mask = 0;
      int64_t rem = k;
      for (int shift = 24; shift >= 0; shift -= 8) {
        for (int b = threadIdx.x; b < 256; b += blockDim.x) hist[b] = 0;
        __syncthreads();
        for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
          const uint32_t key = score_key(row[i]);
          if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
        }
        __syncthreads();
        if (threadIdx.x < 32) {
          // lane L owns digits [248-8L, 255-8L], scanned from the top.
          const int lane = threadIdx.x;
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

  int64_t running = 0, eq_seen = 0;
  for (int64_t c0 = 0; c0 < n; c0 += blockDim.x) {
    const int64_t i = c0 + threadIdx.x;
    bool sel = false, eq = false;
    if (i < n) {
      const float f = row[i];
      if (!topk) {
        sel = f >= p.threshold;
      } else if (take_all) {
        sel = true;
      } else {
        const uint32_t key = score_key(f);
        sel = key > thr;
        eq = key == thr;
      }
    }
    if (topk && !take_all) {
      int eq_tot;
      const int eq_rank = block_scan(eq ? 1 : 0, &eq_tot, scan_sm);
      if (eq && eq_seen + eq_rank < take_eq) sel = true;
      eq_seen += eq_tot;
    }
    int sel_tot;
    const int rank = block_scan(sel ? 1 : 0, &sel_tot, scan_sm);
    if (sel) {
      const int64_t o = running + rank;
      const int64_t pos = sg.pos0 + i;
      const int64_t bt = sg.blk_off + pos / p.block_size;
      int64_t slot = -1;
      if (bt >= 0 && bt < p.block_table_numel) {
        slot = (int64_t)__ldg(&p.block_table[bt]) * p.block_size + pos % p.block_size;
      } else {
        atomicOr(p.err, DEV_ERR_INDEX_RANGE);
      }
      oidx[o] = (int32_t)pos;
      oslot[o] = slot;
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
  select_kernel<<<grid, kSelThreads, 0, s>>>(p);
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
