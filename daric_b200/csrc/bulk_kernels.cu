// Bulk-copy pipeline for the page copies of the reused-KV path (sm_100a).
//
// One persistent CTA per SM walks a contiguous range of units (one page of
// one job). Each unit's regions (prefix_size x suffix bytes: the K and V
// planes of a page) are moved by the copy engine with untiled
// cp.async.bulk loads into a shared-memory stage (mbarrier completion,
// NSTAGE stages in flight), the K rows are re-rotated in shared memory by
// all threads, and the whole page goes back out with cp.async.bulk stores.
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

constexpr int kBulkThreads = 512;
constexpr uint32_t kWaitLimit = 1u << 22;

struct StageMeta {
  int64_t job;
  int64_t page_local;
  int32_t blk;
  int32_t skip;
};

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
                                                 int64_t tok0, int64_t len, float* tok_dev) {
  constexpr int U = 4;
  const int ntask = L.nrows * L.pair_vecs;
  const int hi_off = NEOX ? (L.rot_vecs / 2) * 16 : 0;
  const int per_tok = L.half_rot / 2;
  const uint32_t base = smem_addr(kreg);
  for (int b0 = threadIdx.x; b0 < ntask; b0 += U * blockDim.x) {
    uint4 lo[U], hi[U];
    int off[U], slot[U], c[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int t = b0 + u * blockDim.x;
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
      if (off[u] < 0) continue;
      const float4* q = fac + slot[u] * per_tok + c[u];
      float dv = 0.f;
      if (NEOX) rotate_neox_q<E, SCORE>(q, L.pair_vecs, lo[u], hi[u], dv);
      else rotate_gptj_q<E, SCORE>(q, L.pair_vecs, lo[u], dv);
      if (SCORE) atomicAdd(&tok_dev[slot[u]], dv);
      sts128(base + off[u], lo[u]);
      if (NEOX) sts128(base + off[u] + hi_off, hi[u]);
    }
  }
}

// Shared memory: [0,64) barriers | [64,256) stage meta | dev region |
// stages (page data, then the page's factor block at fac_off).
template <int KVT, bool NEOX, bool ROTATE, bool GATHER, bool SCORE>
__global__ void __launch_bounds__(kBulkThreads, 1) bulk_pages_kernel(PageLaunch p, BulkGeom g) {
  using E = Elem<KVT>;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
  StageMeta* meta = reinterpret_cast<StageMeta*>(smem + 64);
  float* tok_dev = reinterpret_cast<float*>(smem + 256);
  uint8_t* stages = smem + 256 + g.dev_bytes;
  const int NS = g.nstage;
  const int tid = threadIdx.x;

  int64_t ubeg, uend;
  cta_range(p.total_units, ubeg, uend);
  if (ubeg >= uend) return;
  const int64_t n = uend - ubeg;

  int64_t pj = 0;  // producer's job cursor (thread 0)
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
  auto issue = [&](int64_t u, int s) {
    while (pj + 1 < p.num_jobs && p.jobs[pj + 1].unit_begin <= u) ++pj;
    const JobDev j = p.jobs[pj];
    const LayerDev& L = p.layers[j.layer];
    const int64_t pl = u - j.unit_begin;
    const int32_t blk = __ldg(&p.indices[j.idx_off + pl]);
    int skip = blk == 0;
    if (!skip && (blk < 0 || blk >= L.num_pages)) {
      atomicOr(p.err, DEV_ERR_BLOCK_RANGE);
      skip = 1;
    }
    meta[s] = StageMeta{pj, pl, blk, skip};
    if (skip) {
      mbar_arrive(&bars[s]);
      return;
    }
    uint8_t* buf = stages + (size_t)s * g.stage_bytes;
    const bool rot = unit_rotates(j, L);
    const uint32_t fbytes = rot ? (uint32_t)page_factor_bytes(L.page_size, L.half_rot) : 0u;
    mbar_arrive_expect_tx(&bars[s], (uint32_t)(L.prefix_size * L.suffix) + fbytes);
    for (int pf = 0; pf < L.prefix_size; ++pf)
      bulk_load(buf + (size_t)pf * L.suffix, region_src(j, L, pl, blk, pf), (uint32_t)L.suffix, &bars[s]);
    if (rot)
      bulk_load(buf + g.fac_off, p.fac + (j.fac_tok + pl * L.page_size) * (L.half_rot / 2), fbytes, &bars[s]);
  };

  if (tid == 0) {
    for (int s = 0; s < NS; ++s) mbar_init(&bars[s], 1);
    mbar_init_fence();
    pj = find_job(p.jobs, p.num_jobs, ubeg);
    for (int s = 0; s < NS - 1 && s < n; ++s) issue(ubeg + s, s);
  }
  __syncthreads();

  int64_t i = 0;
  bool failed = false;
  for (; i < n; ++i) {
    const int s = (int)(i % NS);
    const StageMeta st = meta[s];
    const JobDev j = p.jobs[st.job];
    const LayerDev& L = p.layers[j.layer];
    uint8_t* buf = stages + (size_t)s * g.stage_bytes;
    const bool rotate = !st.skip && unit_rotates(j, L);
    const bool scoring = SCORE && j.score_row >= 0 && j.meta >= 0;
    const int64_t len = (ROTATE && j.meta >= 0) ? p.metas[j.meta].len : 0;
    const int64_t tok0 = st.page_local * L.page_size;
    if (scoring)
      for (int q = tid; q < L.page_size; q += blockDim.x) tok_dev[q] = 0.f;
    const bool ok = mbar_wait(&bars[s], (uint32_t)((i / NS) & 1));
    if (__syncthreads_or(!ok)) {
      failed = true;
      break;
    }
    if (rotate)
      rotate_rows_smem<E, NEOX, SCORE>(L, buf + (size_t)L.k_prefix * L.suffix,
                                       reinterpret_cast<const float4*>(buf + g.fac_off), tok0, len, tok_dev);
    fence_proxy_async();
    __syncthreads();
    if (tid == 0 && !st.skip) {
      for (int pf = 0; pf < L.prefix_size; ++pf)
        bulk_store(region_dst(j, L, st.page_local, st.blk, pf), buf + (size_t)pf * L.suffix, (uint32_t)L.suffix);
      bulk_commit();
    }
    if (scoring) {
      float* out = p.scores + (int64_t)j.score_row * p.score_ld + p.metas[j.meta].score_col + tok0;
      for (int q = tid; q < L.page_size; q += blockDim.x)
        if (tok0 + q < len) out[q] = rotate ? tok_dev[q] : 0.f;
    }
    // Unit i+NS-1 reuses the stage of unit i-1, whose stores must have
    // finished reading it (the newest bulk group, unit i's, may still run).
    const int64_t nxt = i + NS - 1;
    if (tid == 0 && nxt < n) {
      if (st.skip) bulk_wait_read<0>(); else bulk_wait_read<1>();
      issue(ubeg + nxt, (int)(nxt % NS));
    }
    __syncthreads();
  }
  if (failed && tid == 0) {
    atomicOr(p.err, DEV_ERR_TIMEOUT);
    // drain the loads still in flight into this CTA's shared memory
    const int64_t issued = (i + NS - 1 < n) ? i + NS - 1 : n;
    for (int64_t k = i; k < issued; ++k) mbar_wait(&bars[k % NS], (uint32_t)((k / NS) & 1));
  }
  if (tid == 0) bulk_wait_all();
  __syncthreads();
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
