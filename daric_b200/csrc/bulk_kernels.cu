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

struct StageMeta {  // what the producer recorded when it issued a stage's loads
  int64_t job;
  int64_t page_local;
  int32_t blk;
  int32_t skip;
  uint8_t* dst[2];     // store destinations of the regions (nreg <= 2)
  float* sout;         // score output of the page's first slot (SCORE)
  int32_t sn;          // slots with a score to write
  int32_t nreg;        // regions (prefix entries) of the page
  int32_t rbytes;      // bytes per region
  int32_t pad;
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

// Rotates the K rows of one region held in shared memory (in place) with
// the page's factor block (also in shared memory).
template <class E, bool NEOX, bool SCORE>
__device__ __forceinline__ void rotate_rows_smem(const LayerDev& L, uint8_t* kreg, const float4* fac,
                                                 int64_t tok0, int64_t len, float* tok_dev, int tid,
                                                 int nthreads) {
  constexpr int U = 4;
  const int ntask = L.nrows * L.pair_vecs;
  const int hi_off = NEOX ? (L.rot_vecs / 2) * 16 : 0;
  const int per_tok = L.half_rot / 2;
  const uint32_t base = smem_addr(kreg);
  // warp-uniform trip count (score_add shuffles across the warp)
  for (int b0 = tid; b0 - (tid & 31) < ntask; b0 += U * nthreads) {
    uint4 lo[U], hi[U];
    int off[U], slot[U], c[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int t = b0 + u * nthreads;
      off[u] = -1;
      if (t < ntask) {
        const int row = (int)fdiv((uint32_t)t, L.pair_div);
        c[u] = t - row * L.pair_vecs;
        slot[u] = row_slot(L, row);
        if (tok0 + slot[u] < len) {
          off[u] = row * L.row_bytes + c[u] * 16;
          lo[u] = lds128(base + off[u]);
          if (NEOX) hi[u] = lds128(base + off[u] + hi_off);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      float dv = 0.f;
      if (off[u] >= 0) {
        const float4* q = fac + slot[u] * per_tok + c[u];
        if (NEOX) rotate_neox_q<E, SCORE>(q, L.pair_vecs, lo[u], hi[u], dv);
        else rotate_gptj_q<E, SCORE>(q, L.pair_vecs, lo[u], dv);
        sts128(base + off[u], lo[u]);
        if (NEOX) sts128(base + off[u] + hi_off, hi[u]);
      }
      if (SCORE) score_add(tok_dev, off[u] >= 0 ? slot[u] : -1, dv);
    }
  }
}

// Warp-specialised pipeline. Warps 0..kConsumerWarps-1 rotate; the last
// warp's lane 0 is the producer: it issues the bulk loads of unit u into
// stage u % NS (full[s] completes when the bytes land), waits until every
// consumer warp has released the unit (empty[s]), issues the bulk stores,
// and reuses the stage of the previous unit once its stores have read it.
// Shared memory: [0,128) full/empty barriers | [128,512) stage meta |
// per-stage deviation slots | stages (page data, then the page's factor
// block at fac_off).
template <int KVT, bool NEOX, bool ROTATE, bool GATHER, bool SCORE>
__global__ void __launch_bounds__(kBulkThreads, 1) bulk_pages_kernel(PageLaunch p, BulkGeom g) {
  using E = Elem<KVT>;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kMaxStages;
  StageMeta* meta = reinterpret_cast<StageMeta*>(smem + 128);
  float* devs = reinterpret_cast<float*>(smem + kBulkHeader);  // NS x dev_stride floats
  uint8_t* stages = smem + kBulkHeader + g.dev_bytes;
  const int NS = g.nstage;
  const int dev_stride = g.dev_bytes / (4 * NS);
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const bool producer = warp == kConsumerWarps;
  constexpr int kConsumers = kConsumerWarps * 32;

  int64_t ubeg, uend;
  cta_range(p.total_units, ubeg, uend);
  if (ubeg >= uend) return;
  const int64_t n = uend - ubeg;

  auto region_src = [&](const JobDev& j, const LayerDev& L, int64_t pl, int32_t blk, int pf) -> const uint8_t* {
    if (GATHER) return L.base + (int64_t)pf * L.prefix_stride + (int64_t)blk * L.page_stride;
    return p.store + j.stg_off + ((int64_t)pf * j.n_sel + pl) * L.suffix;
  };
  auto region_dst = [&](const JobDev& j, const LayerDev& L, int64_t pl, int32_t blk, int pf) -> uint8_t* {
    if (GATHER) return p.store_mut + j.stg_off + ((int64_t)pf * j.n_sel + pl) * L.suffix;
    return L.base + (int64_t)pf * L.prefix_stride + (int64_t)blk * L.page_stride;
  };
  auto unit_rotates = [&](const JobDev& j, const LayerDev& L) -> bool {
    return ROTATE && j.meta >= 0 && L.has_rot && p.metas[j.meta].rotate;
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
    // The producer warp prefetches the copy plan of 32 units at a time (one
    // unit per lane: job lookup, block id, addresses) so that lane 0, which
    // issues every bulk copy, never waits on a descriptor load.
    const unsigned FULL = 0xffffffffu;
    int64_t jc = find_job(p.jobs, p.num_jobs, ubeg);
    int64_t batch = -1;
    const uint8_t *my_src0 = nullptr, *my_src1 = nullptr;
    uint8_t *my_dst0 = nullptr, *my_dst1 = nullptr;
    const float4* my_fac = nullptr;
    float* my_sout = nullptr;
    int64_t my_job = 0, my_pl = 0;
    int32_t my_blk = 0, my_skip = 1, my_nreg = 0, my_rb = 0, my_fb = 0, my_sn = 0;
    auto prefetch = [&](int64_t b) {  // all lanes
      const int64_t i = b * 32 + lane;
      int64_t j = jc;
      my_skip = 1;
      my_nreg = 0;
      my_fb = 0;
      my_sn = 0;
      if (i < n) {
        const int64_t u = ubeg + i;
        while (j + 1 < p.num_jobs && p.jobs[j + 1].unit_begin <= u) ++j;
        const JobDev jd = p.jobs[j];
        const LayerDev& L = p.layers[jd.layer];
        const int64_t pl = u - jd.unit_begin;
        const int32_t blk = __ldg(&p.indices[jd.idx_off + pl]);
        int skip = blk == 0;
        if (!skip && (blk < 0 || blk >= L.num_pages)) {
          atomicOr(p.err, DEV_ERR_BLOCK_RANGE);
          skip = 1;
        }
        my_job = j;
        my_pl = pl;
        my_blk = blk;
        my_skip = skip;
        my_nreg = L.prefix_size;
        my_rb = (int32_t)L.suffix;
        if (!skip && L.prefix_size <= 2) {
          my_src0 = region_src(jd, L, pl, blk, 0);
          my_dst0 = region_dst(jd, L, pl, blk, 0);
          if (L.prefix_size == 2) {
            my_src1 = region_src(jd, L, pl, blk, 1);
            my_dst1 = region_dst(jd, L, pl, blk, 1);
          }
        }
        if (!skip && unit_rotates(jd, L)) {
          my_fb = (int32_t)page_factor_bytes(L.page_size, L.half_rot);
          my_fac = p.fac + (jd.fac_tok + pl * L.page_size) * (L.half_rot / 2);
        }
        if (SCORE && jd.score_row >= 0 && jd.meta >= 0) {
          const MetaDev m = p.metas[jd.meta];
          const int64_t tok0 = pl * L.page_size;
          const int64_t left = m.len - tok0;
          my_sn = (int32_t)(left < 0 ? 0 : (left < L.page_size ? left : L.page_size));
          my_sout = p.scores + (int64_t)jd.score_row * p.score_ld + m.score_col + tok0;
        }
      }
      jc = __shfl_sync(FULL, j, 31);
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
      st.job = __shfl_sync(FULL, my_job, k);
      st.page_local = __shfl_sync(FULL, my_pl, k);
      st.blk = __shfl_sync(FULL, my_blk, k);
      st.skip = __shfl_sync(FULL, my_skip, k);
      st.nreg = __shfl_sync(FULL, my_nreg, k);
      st.rbytes = __shfl_sync(FULL, my_rb, k);
      st.sn = __shfl_sync(FULL, my_sn, k);
      st.dst[0] = (uint8_t*)__shfl_sync(FULL, (unsigned long long)my_dst0, k);
      st.dst[1] = (uint8_t*)__shfl_sync(FULL, (unsigned long long)my_dst1, k);
      st.sout = (float*)__shfl_sync(FULL, (unsigned long long)my_sout, k);
      const uint8_t* src0 = (const uint8_t*)__shfl_sync(FULL, (unsigned long long)my_src0, k);
      const uint8_t* src1 = (const uint8_t*)__shfl_sync(FULL, (unsigned long long)my_src1, k);
      const float4* fac = (const float4*)__shfl_sync(FULL, (unsigned long long)my_fac, k);
      const uint32_t fb = (uint32_t)__shfl_sync(FULL, my_fb, k);
      if (lane != 0) return;
      const int s = (int)(i % NS);
      meta[s] = st;
      if (st.skip) {
        mbar_arrive(&full[s]);
        return;
      }
      uint8_t* buf = stages + (size_t)s * g.stage_bytes;
      mbar_arrive_expect_tx(&full[s], (uint32_t)(st.nreg * st.rbytes) + fb);
      if (st.nreg <= 2) {
        bulk_load(buf, src0, (uint32_t)st.rbytes, &full[s]);
        if (st.nreg == 2) bulk_load(buf + st.rbytes, src1, (uint32_t)st.rbytes, &full[s]);
      } else {  // more than two regions per page: addresses computed here
        const JobDev jd = p.jobs[st.job];
        const LayerDev& L = p.layers[jd.layer];
        for (int pf = 0; pf < st.nreg; ++pf)
          bulk_load(buf + (size_t)pf * st.rbytes, region_src(jd, L, st.page_local, st.blk, pf),
                    (uint32_t)st.rbytes, &full[s]);
      }
      if (fb) bulk_load(buf + g.fac_off, fac, fb, &full[s]);
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
      const StageMeta st = meta[s];
      const bool stored = !st.skip;
      if (lane == 0 && stored) {
        uint8_t* buf = stages + (size_t)s * g.stage_bytes;
        if (st.nreg <= 2) {
          bulk_store(st.dst[0], buf, (uint32_t)st.rbytes);
          if (st.nreg == 2) bulk_store(st.dst[1], buf + st.rbytes, (uint32_t)st.rbytes);
        } else {
          const JobDev jd = p.jobs[st.job];
          const LayerDev& L = p.layers[jd.layer];
          for (int pf = 0; pf < st.nreg; ++pf)
            bulk_store(region_dst(jd, L, st.page_local, st.blk, pf), buf + (size_t)pf * st.rbytes,
                       (uint32_t)st.rbytes);
        }
        bulk_commit();
      }
      if (SCORE && st.sn > 0) {
        float* dv = devs + s * dev_stride;
        for (int q = lane; q < st.sn; q += 32) st.sout[q] = dv[q];
      }
      if (SCORE)
        for (int q = lane; q < dev_stride; q += 32) devs[s * dev_stride + q] = 0.f;
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
    const StageMeta st = meta[s];
    const JobDev j = p.jobs[st.job];
    const LayerDev& L = p.layers[j.layer];
    if (!st.skip && unit_rotates(j, L)) {
      uint8_t* buf = stages + (size_t)s * g.stage_bytes;
      const int64_t len = p.metas[j.meta].len;
      const int64_t tok0 = st.page_local * L.page_size;
      rotate_rows_smem<E, NEOX, SCORE>(L, buf + (size_t)L.k_prefix * L.suffix,
                                       reinterpret_cast<const float4*>(buf + g.fac_off), tok0, len,
                                       devs + s * dev_stride, tid, kConsumers);
      fence_proxy_async();
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

template <int KVT>
void bulk_rotate(const PageLaunch& p, const BulkGeom& g, bool neox, int sm, cudaStream_t s) {
  const bool sc = p.scores != nullptr;
  if (neox) {
    if (sc) launch_bulk(bulk_pages_kernel<KVT, true, true, false, true>, p, g, sm, s);
    else launch_bulk(bulk_pages_kernel<KVT, true, true, false, false>, p, g, sm, s);
  } else {
    if (sc) launch_bulk(bulk_pages_kernel<KVT, false, true, false, true>, p, g, sm, s);
    else launch_bulk(bulk_pages_kernel<KVT, false, true, false, false>, p, g, sm, s);
  }
}

}  // namespace

void launch_bulk_plain(const PageLaunch& p, const BulkGeom& g, bool gather, int sm, cudaStream_t s) {
  if (gather)
    launch_bulk(bulk_pages_kernel<DARIC_DTYPE_BF16, true, false, true, false>, p, g, sm, s);
  else
    launch_bulk(bulk_pages_kernel<DARIC_DTYPE_BF16, true, false, false, false>, p, g, sm, s);
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
