// Bulk-copy pipeline for the page copies of the reused-KV path (sm_100a).
//
// One persistent CTA per SM walks a contiguous range of units (one page of
// one job). Each unit's regions (prefix_size x suffix bytes: the K and V
// planes of a page) are moved by the copy engine with untiled
// cp.async.bulk loads into a shared-memory stage (mbarrier completion,
// NSTAGE stages in flight), the K rows are re-rotated in shared memory by
// the consumer warps, and the whole page goes back out with cp.async.bulk
// stores issued by a producer warp.
// V bytes never pass through registers. Same byte mapping, block-0 skip,
// rotation math and deviation scores as the SIMT kernels in page_kernels.cu.
//
// Every wait is bounded: an mbarrier wait that exceeds kWaitLimit rounds
// sets DEV_ERR_TIMEOUT, drains the copies this CTA has in flight (again with
// a bound) and returns.
#include <map>
#include <mutex>

#include "device_common.cuh"
#include "internal.h"

namespace daric {
namespace {
using namespace dev;

constexpr int kConsumerWarps = 16;
constexpr int kBulkThreads = kConsumerWarps * 32 + 32;  // + one producer warp
constexpr int kMaxStages = 8;
constexpr uint32_t kWaitLimit = 1u << 22;

constexpr int kMaxPagesPerUnit = 8;

struct StageMeta {  // what the producer recorded when it issued a stage's loads
  int64_t job;
  uint8_t* base;          // layer data
  int64_t stg_off;        // job's store offset
  int64_t page_stride;
  int64_t prefix_stride;
  float* sout;            // score output of the unit's first token (SCORE)
  const uint8_t* fac;     // factor block to stage with the pages (nullptr: none)
  int32_t pl0;            // first page (job-local) of the unit
  int32_t npg;            // pages in the unit
  int32_t skipmask;       // bit g: page g is not copied (block id 0 / out of range)
  int32_t nreg;           // regions (prefix entries) per page
  int32_t rbytes;         // bytes per region
  int32_t n_sel;          // pages of the job
  int32_t sn;             // tokens with a score to write
  int32_t fac_bytes;      // bytes of the staged factor block
  int32_t blk[kMaxPagesPerUnit];
};
static_assert(128 + kMaxStages * sizeof(StageMeta) <= kBulkHeader, "stage meta exceeds the header");

// ------------------------------------------------------------- PTX ------
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait for the phase with the given parity.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  for (uint32_t k = 0; k < kWaitLimit; ++k)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}
__device__ __forceinline__ void bulk_load(void* sdst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(sdst)),
      "l"(gsrc), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}
__device__ __forceinline__ void bulk_store(void* gdst, const void* ssrc, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst), "r"(smem_addr(ssrc)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t a) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
  return v;
}
__device__ __forceinline__ void sts128(uint32_t a, uint4 v) {
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(a), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

__device__ __forceinline__ void cta_range(int64_t total, int64_t& begin, int64_t& end) {
  const int64_t g = gridDim.x, b = blockIdx.x;
  const int64_t q = total / g, r = total % g;
  begin = b * q + (b < r ? b : r);
  end = begin + q + (b < r ? 1 : 0);
}

__device__ __forceinline__ int64_t find_job(const JobDev* jobs, int64_t n, int64_t unit) {
  int64_t lo = 0, hi = n - 1;
  while (lo < hi) {
    const int64_t mid = (lo + hi + 1) >> 1;
    if (__ldg(&jobs[mid].unit_begin) <= unit) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// Factor entry {C[d0], C[d0+1], S[d0], S[d0+1]} stored as 4 x bf16 (low
// half = d0): widening bf16 to fp32 is exact.
__device__ __forceinline__ float4 widen_factors(uint2 w) {
  return make_float4(__uint_as_float(w.x << 16), __uint_as_float(w.x & 0xffff0000u), __uint_as_float(w.y << 16),
                     __uint_as_float(w.y & 0xffff0000u));
}
__device__ __forceinline__ float4 as_float4(uint4 w) {
  return make_float4(__uint_as_float(w.x), __uint_as_float(w.y), __uint_as_float(w.z), __uint_as_float(w.w));
}

// Rotates the K rows of the unit's pages held in shared memory (in place).
// Task t of the unit -> page g, row, pair c; the factors come from the
// unit's factor block staged beside the pages (fac_staged) or straight from
// the factor buffer in global memory (L2 resident, shared by the heads).
// FC: factor entries are 4 x bf16 (8 bytes) instead of 4 x fp32 (16 bytes).
template <class E, bool NEOX, bool SCORE, bool FC>
__device__ __forceinline__ void rotate_unit_smem(const LayerDev& L, uint8_t* stage, int page_data,
                                                 const StageMeta& st, const uint8_t* fac_unit, bool fac_staged,
                                                 int64_t len, float* tok_dev, int tid, int nthreads) {
  constexpr int ES = FC ? 8 : 16;  // bytes per factor entry
  constexpr int U = E::kPerVec > 8 ? 1 : 2;  // fp8: 16 elements a vector, one task in flight
  const int per_page = L.nrows * L.pair_vecs;
  const int ntask = per_page * st.npg;
  const int hi_off = NEOX ? (L.rot_vecs / 2) * 16 : 0;
  const int per_tok = L.half_rot / 2;
  const int64_t tok_base = (int64_t)st.pl0 * L.page_size;
  const uint32_t base = smem_addr(stage) + (uint32_t)L.k_prefix * (uint32_t)st.rbytes;
  // warp-uniform trip count (score_add shuffles across the warp)
  for (int b0 = tid; b0 - (tid & 31) < ntask; b0 += U * nthreads) {
    uint4 lo[U], hi[U];
    float4 q[U][E::kPerVec / 2 > 4 ? 8 : 4];
    int off[U], slot[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int t = b0 + u * nthreads;
      off[u] = -1;
      slot[u] = -1;
      if (t < ntask) {
        const int g = (int)fdiv((uint32_t)t, L.page_div);
        const int r = t - g * per_page;
        const int row = (int)fdiv((uint32_t)r, L.pair_div);
        const int c = r - row * L.pair_vecs;
        const int sl = row_slot(L, row);
        const int64_t tok = (int64_t)g * L.page_size + sl;  // unit token
        if (!((st.skipmask >> g) & 1) && tok_base + tok < len) {
          off[u] = g * page_data + row * L.row_bytes + c * 16;
          slot[u] = (int)tok;
          lo[u] = lds128(base + off[u]);
          if (NEOX) hi[u] = lds128(base + off[u] + hi_off);
          const uint8_t* fq = fac_unit + ((int)tok * per_tok + c) * ES;
          constexpr int NG = NEOX ? E::kPerVec / 2 : E::kPerVec / 4;
          if (fac_staged) {
            const uint32_t fa = smem_addr(fq);
#pragma unroll
            for (int k = 0; k < NG; ++k) {
              const uint32_t a = fa + (uint32_t)(k * L.pair_vecs * ES);
              q[u][k] = FC ? widen_factors(lds64(a)) : as_float4(lds128(a));
            }
          } else {
#pragma unroll
            for (int k = 0; k < NG; ++k) {
              const uint8_t* gp = fq + k * L.pair_vecs * ES;
              q[u][k] = FC ? widen_factors(__ldg(reinterpret_cast<const uint2*>(gp)))
                           : __ldg(reinterpret_cast<const float4*>(gp));
            }
          }
        }
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      float dv = 0.f;
      if (off[u] >= 0) {
        if (NEOX) rotate_neox_q<E, SCORE>(q[u], 1, lo[u], hi[u], dv);
        else rotate_gptj_q<E, SCORE>(q[u], 1, lo[u], dv);
        sts128(base + off[u], lo[u]);
        if (NEOX) sts128(base + off[u] + hi_off, hi[u]);
      }
      if (SCORE) score_add(tok_dev, slot[u], dv);
    }
  }
}

// Warp-specialised pipeline. Warps 0..kConsumerWarps-1 rotate; the last
// warp is the producer: its 32 lanes prefetch the copy plans of 32 units at
// a time, and lane 0 issues the bulk loads of unit u into stage u % NS
// (full[s] completes when the bytes land), waits until every consumer warp
// has released the unit (empty[s]), issues the bulk stores, and reuses the
// stage of the previous unit once its stores have read it.
// Shared memory: [0,128) full/empty barriers | [128,kBulkHeader) stage meta |
// per-stage deviation slots | stages (page g of a unit at g * page_data).
template <int KVT, bool NEOX, bool ROTATE, bool GATHER, bool SCORE, bool FC>
__global__ void __launch_bounds__(kBulkThreads, 1) bulk_pages_kernel(PageLaunch p, BulkGeom g) {
  using E = Elem<KVT>;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kMaxStages;
  StageMeta* meta = reinterpret_cast<StageMeta*>(smem + 128);
  float* devs = reinterpret_cast<float*>(smem + kBulkHeader);  // NS x dev_stride floats
  uint8_t* stages = smem + kBulkHeader + g.dev_bytes;
  const int NS = g.nstage;
  const int G = g.pages_per_unit;
  const int dev_stride = g.dev_bytes / (4 * NS);
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const bool producer = warp == kConsumerWarps;
  constexpr int kConsumers = kConsumerWarps * 32;

  int64_t ubeg, uend;
  cta_range(p.total_units, ubeg, uend);
  if (ubeg >= uend) return;
  const int64_t n = uend - ubeg;

  // address of region pf of job-local page pl (block blk) on the source /
  // destination side
  auto store_region = [&](const StageMeta& st, int pl, int pf) -> uint8_t* {
    return p.store_mut + st.stg_off + ((int64_t)pf * st.n_sel + pl) * st.rbytes;
  };
  auto layer_region = [&](const StageMeta& st, int32_t blk, int pf) -> uint8_t* {
    return st.base + (int64_t)pf * st.prefix_stride + (int64_t)blk * st.page_stride;
  };

  if (tid == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    mbar_init_fence();
  }
  if (SCORE)
    for (int q = tid; q < NS * dev_stride; q += blockDim.x) devs[q] = 0.f;
  __syncthreads();

  if (producer) {
    const unsigned FULL = 0xffffffffu;
    int64_t jc = find_job(p.jobs, p.num_jobs, ubeg);
    int64_t batch = -1;
    // this lane's unit of the current batch
    StageMeta mine{};
    auto prefetch = [&](int64_t b) {  // all lanes
      const int64_t i = b * 32 + lane;
      int64_t j = jc;
      mine.npg = 0;
      mine.skipmask = 0;
      mine.sn = 0;
      mine.fac = nullptr;
      mine.fac_bytes = 0;
      if (i < n) {
        const int64_t u = ubeg + i;
        while (j + 1 < p.num_jobs && p.jobs[j + 1].unit_begin <= u) ++j;
        const JobDev jd = p.jobs[j];
        const LayerDev& L = p.layers[jd.layer];
        const int pl0 = (int)(u - jd.unit_begin) * G;
        const int npg = min(G, jd.n_sel - pl0);
        mine.job = j;
        mine.base = L.base;
        mine.stg_off = jd.stg_off;
        mine.page_stride = L.page_stride;
        mine.prefix_stride = L.prefix_stride;
        mine.pl0 = pl0;
        mine.npg = npg;
        mine.nreg = L.prefix_size;
        mine.rbytes = (int32_t)L.suffix;
        mine.n_sel = jd.n_sel;
        for (int q = 0; q < kMaxPagesPerUnit; ++q) {
          if (q >= npg) break;
          const int32_t blk = __ldg(&p.indices[jd.idx_off + pl0 + q]);
          int skip = blk == 0;
          if (!skip && (blk < 0 || blk >= L.num_pages)) {
            atomicOr(p.err, DEV_ERR_BLOCK_RANGE);
            skip = 1;
          }
          mine.blk[q] = blk;
          mine.skipmask |= skip << q;
        }
        if (ROTATE && g.fac_off > 0 && jd.meta >= 0 && L.has_rot && p.metas[jd.meta].rotate) {
          const int64_t tb = (int64_t)token_factor_bytes(L.half_rot, FC);
          mine.fac = reinterpret_cast<const uint8_t*>(p.fac) + (jd.fac_tok + (int64_t)pl0 * L.page_size) * tb;
          mine.fac_bytes = (int32_t)((size_t)npg * page_factor_bytes(L.page_size, L.half_rot, FC));
        }
        if (SCORE && jd.score_row >= 0 && jd.meta >= 0) {
          const MetaDev m = p.metas[jd.meta];
          const int64_t tok0 = (int64_t)pl0 * L.page_size;
          const int64_t left = m.len - tok0;
          const int64_t cap = (int64_t)npg * L.page_size;
          mine.sn = (int32_t)(left < 0 ? 0 : (left < cap ? left : cap));
          mine.sout = p.scores + (int64_t)jd.score_row * p.score_ld + m.score_col + tok0;
        }
      }
      jc = __shfl_sync(FULL, j, 31);
    };
    auto shfl64 = [&](auto v, int k) {
      return (decltype(v))__shfl_sync(FULL, (unsigned long long)v, k);
    };
    // loads of unit i into stage i % NS (warp-synchronous: every lane calls)
    auto issue = [&](int64_t i) {
      const int64_t b = i / 32;
      if (b != batch) {
        prefetch(b);
        batch = b;
      }
      const int k = (int)(i - b * 32);
      StageMeta st;
      st.job = __shfl_sync(FULL, mine.job, k);
      st.base = shfl64(mine.base, k);
      st.stg_off = __shfl_sync(FULL, mine.stg_off, k);
      st.page_stride = __shfl_sync(FULL, mine.page_stride, k);
      st.prefix_stride = __shfl_sync(FULL, mine.prefix_stride, k);
      st.sout = shfl64(mine.sout, k);
      st.pl0 = __shfl_sync(FULL, mine.pl0, k);
      st.npg = __shfl_sync(FULL, mine.npg, k);
      st.skipmask = __shfl_sync(FULL, mine.skipmask, k);
      st.nreg = __shfl_sync(FULL, mine.nreg, k);
      st.rbytes = __shfl_sync(FULL, mine.rbytes, k);
      st.n_sel = __shfl_sync(FULL, mine.n_sel, k);
      st.sn = __shfl_sync(FULL, mine.sn, k);
      st.fac = shfl64(mine.fac, k);
      st.fac_bytes = __shfl_sync(FULL, mine.fac_bytes, k);
#pragma unroll
      for (int q = 0; q < kMaxPagesPerUnit; ++q) st.blk[q] = __shfl_sync(FULL, mine.blk[q], k);
      if (lane != 0) return;
      const int s = (int)(i % NS);
      meta[s] = st;
      const int live = st.npg - __popc(st.skipmask);
      if (live == 0) {
        mbar_arrive(&full[s]);
        return;
      }
      uint8_t* buf = stages + (size_t)s * g.stage_bytes;
      const uint32_t fb = (uint32_t)st.fac_bytes;
      mbar_arrive_expect_tx(&full[s], (uint32_t)(live * st.nreg * st.rbytes) + fb);
      if (fb) bulk_load(buf + g.fac_off, st.fac, fb, &full[s]);
      for (int q = 0; q < st.npg; ++q) {
        if ((st.skipmask >> q) & 1) continue;
        for (int pf = 0; pf < st.nreg; ++pf) {
          const uint8_t* src = GATHER ? layer_region(st, st.blk[q], pf) : store_region(st, st.pl0 + q, pf);
          bulk_load(buf + (size_t)q * g.page_data + (size_t)pf * st.rbytes, src, (uint32_t)st.rbytes, &full[s]);
        }
      }
    };
    int64_t issued = 0;
    for (; issued < NS - 1 && issued < n; ++issued) issue(issued);
    bool prev_stored = false;  // unit i-1 has a pending store group (lane 0)
    int64_t i = 0;
    for (; i < n; ++i) {
      const int s = (int)(i % NS);
      const bool ok = mbar_wait(&empty[s], (uint32_t)((i / NS) & 1));
      if (__any_sync(FULL, !ok)) {
        if (lane == 0) atomicOr(p.err, DEV_ERR_TIMEOUT);
        break;
      }
      const StageMeta& st = meta[s];
      const bool stored = st.npg > __popc(st.skipmask);
      if (lane == 0 && stored) {
        uint8_t* buf = stages + (size_t)s * g.stage_bytes;
        for (int q = 0; q < st.npg; ++q) {
          if ((st.skipmask >> q) & 1) continue;
          for (int pf = 0; pf < st.nreg; ++pf) {
            uint8_t* dst = GATHER ? store_region(st, st.pl0 + q, pf) : layer_region(st, st.blk[q], pf);
            bulk_store(dst, buf + (size_t)q * g.page_data + (size_t)pf * st.rbytes, (uint32_t)st.rbytes);
          }
        }
        bulk_commit();
      }
      if (SCORE) {
        float* dv = devs + s * dev_stride;
        for (int q = lane; q < st.sn; q += 32) st.sout[q] = dv[q];
        __syncwarp();
        for (int q = lane; q < dev_stride; q += 32) dv[q] = 0.f;
      }
      __syncwarp();
      // the next load goes into the stage of unit i-1: its stores must have
      // read it (unit i's group, committed last, may still be pending)
      if (issued < n) {
        if (lane == 0 && prev_stored) {
          if (stored) bulk_wait_read<1>(); else bulk_wait_read<0>();
        }
        __syncwarp();
        issue(issued);
        ++issued;
      }
      prev_stored = stored;
      __syncwarp();
    }
    if (i < n && lane == 0) {
      // timed out: drain the loads still in flight into this CTA's stages
      for (int64_t k = i + 1; k < issued; ++k) mbar_wait(&full[k % NS], (uint32_t)((k / NS) & 1));
    }
    if (lane == 0) bulk_wait_all();
    return;
  }

  // consumers
  for (int64_t i = 0; i < n; ++i) {
    const int s = (int)(i % NS);
    if (!mbar_wait(&full[s], (uint32_t)((i / NS) & 1))) {
      atomicOr(p.err, DEV_ERR_TIMEOUT);
      break;
    }
    const StageMeta& st = meta[s];
    if (ROTATE && st.npg > __popc(st.skipmask)) {
      const JobDev j = p.jobs[st.job];
      const LayerDev& L = p.layers[j.layer];
      if (j.meta >= 0 && L.has_rot) {
        const MetaDev m = p.metas[j.meta];
        if (m.rotate) {
          uint8_t* stage = stages + (size_t)s * g.stage_bytes;
          const bool staged = g.fac_off > 0;
          const uint8_t* fac_unit =
              staged ? stage + g.fac_off
                     : reinterpret_cast<const uint8_t*>(p.fac) +
                           (j.fac_tok + (int64_t)st.pl0 * L.page_size) * (int64_t)token_factor_bytes(L.half_rot, FC);
          rotate_unit_smem<E, NEOX, SCORE, FC>(L, stage, g.page_data, st, fac_unit, staged, m.len,
                                               devs + s * dev_stride, tid, kConsumers);
          fence_proxy_async();
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }
}

// ------------------------------------------------------------ launch ----
template <class K>
void launch_bulk(K kernel, const PageLaunch& p, const BulkGeom& g, int sm_count, cudaStream_t s) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, size_t> attr;  // (kernel, device) -> smem set
  const size_t smem = bulk_smem_bytes(g);
  {
    int dev = 0;
    DARIC_CUDA(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lk(mu);
    size_t& cur = attr[std::make_pair((const void*)kernel, dev)];
    if (cur < smem) {
      DARIC_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      cur = smem;
    }
  }
  const int grid = (int)(p.total_units < sm_count ? p.total_units : sm_count);
  kernel<<<grid, kBulkThreads, smem, s>>>(p, g);
  DARIC_CUDA(cudaGetLastError());
}

template <int KVT, bool FC>
void bulk_rotate(const PageLaunch& p, const BulkGeom& g, bool neox, int sm, cudaStream_t s) {
  const bool sc = p.scores != nullptr;
  if (neox) {
    if (sc) launch_bulk(bulk_pages_kernel<KVT, true, true, false, true, FC>, p, g, sm, s);
    else launch_bulk(bulk_pages_kernel<KVT, true, true, false, false, FC>, p, g, sm, s);
  } else {
    if (sc) launch_bulk(bulk_pages_kernel<KVT, false, true, false, true, FC>, p, g, sm, s);
    else launch_bulk(bulk_pages_kernel<KVT, false, true, false, false, FC>, p, g, sm, s);
  }
}
template <int KVT>
void bulk_rotate(const PageLaunch& p, const BulkGeom& g, bool neox, int sm, cudaStream_t s) {
  if (g.fac_compact) bulk_rotate<KVT, true>(p, g, neox, sm, s);
  else bulk_rotate<KVT, false>(p, g, neox, sm, s);
}

}  // namespace

void launch_bulk_plain(const PageLaunch& p, const BulkGeom& g, bool gather, int sm, cudaStream_t s) {
  if (gather)
    launch_bulk(bulk_pages_kernel<DARIC_DTYPE_BF16, true, false, true, false, false>, p, g, sm, s);
  else
    launch_bulk(bulk_pages_kernel<DARIC_DTYPE_BF16, true, false, false, false, false>, p, g, sm, s);
}

void launch_bulk_rotate(const PageLaunch& p, const BulkGeom& g, RotKey k, int sm, cudaStream_t s) {
  switch (k.kv_dtype) {
    case DARIC_DTYPE_BF16: return bulk_rotate<DARIC_DTYPE_BF16>(p, g, k.neox, sm, s);
    case DARIC_DTYPE_F16: return bulk_rotate<DARIC_DTYPE_F16>(p, g, k.neox, sm, s);
    case DARIC_DTYPE_F32: return bulk_rotate<DARIC_DTYPE_F32>(p, g, k.neox, sm, s);
    case DARIC_DTYPE_FP8_E4M3: return bulk_rotate<DARIC_DTYPE_FP8_E4M3>(p, g, k.neox, sm, s);
  }
  throw Error(DARIC_ERR_INVALID, "unsupported KV dtype");
}

}  // namespace daric
