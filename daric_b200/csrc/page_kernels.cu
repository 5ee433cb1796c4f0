// Page kernels of the reused-KV path, written for sm_100a.
//
//  * plain_pages_kernel     : store <-> paged KV byte copy. Same byte mapping as
//                             fused_{gather,scatter}_pages_kernel in the
//                             reference (csrc/cache_ops/kernels.cu:7-45, 86-123):
//                             store[(p*n_sel + i)*suffix + o] <->
//                             layer[p*prefix_stride + block[i]*page_stride + o],
//                             block id 0 skipped.
//  * rotate_scatter_kernel  : the same scatter with the K rows re-rotated on the
//                             way (RoPE by the chunk's position change), which the
//                             reference does afterwards with the Triton kernel
//                             _fused_rerotate_kernel (daric/adaption/adapter.py:30-88).
//  * rotate_inplace_kernel  : in-place re-rotation of K rows in the paged cache,
//                             all layers in one launch (adapter.py:118-295).
//
// All three are HBM-bound streams: 16-byte vector loads and stores, no shared
// memory staging of the data. Work is split into "units" (one page of one job,
// or one page of one segment of one layer); a persistent grid of
// sm_count x (resident CTAs per SM) CTAs takes contiguous unit ranges, so each
// CTA walks the store sequentially and finds its job with one binary search.
#include <mutex>
#include <unordered_map>

#include "device_common.cuh"
#include "internal.h"

namespace daric {
namespace {
using namespace dev;

constexpr int kThreads = 256;

// Rotation tasks of one page region: task t -> (row, pair) -> vectors at
// row*row_bytes + c*16 (and + rot_vecs/2*16 for the NeoX partner). Rows
// whose slot is not rotated (ok == 0) are copied unchanged; in-place
// callers skip them. U tasks in flight per thread.
template <class E, bool NEOX, bool INPLACE>
__device__ __forceinline__ void rotate_rows(const LayerDev& L, const uint8_t* src, uint8_t* dst,
                                            PageSmem sm, bool scoring) {
  constexpr int U = 4;
  constexpr int FPV = NEOX ? E::kPerVec : E::kPerVec / 2;  // factors per task
  const int ntask = L.nrows * L.pair_vecs;
  const int hi_off = NEOX ? (L.rot_vecs / 2) * 16 : 0;
  for (int base = threadIdx.x; base < ntask; base += U * blockDim.x) {
    uint4 lo[U], hi[U];
    int off[U], slot[U], c[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int t = base + u * blockDim.x;
      off[u] = -1;
      if (t < ntask) {
        const int row = (int)fdiv((uint32_t)t, L.pair_div);
        c[u] = t - row * L.pair_vecs;
        const uint32_t q = fdiv((uint32_t)row, L.tok_div);
        slot[u] = (int)(q - fdiv(q, L.tok_mod) * (uint32_t)L.page_size);
        if (!INPLACE || sm.ok[slot[u]]) {
          off[u] = row * L.row_bytes + c[u] * 16;
          if (INPLACE) {
            lo[u] = ld_vec(src + off[u]);
            if (NEOX) hi[u] = ld_vec(src + off[u] + hi_off);
          } else {
            lo[u] = ld_stream(src + off[u]);
            if (NEOX) hi[u] = ld_stream(src + off[u] + hi_off);
          }
        }
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (off[u] < 0) continue;
      if (sm.ok[slot[u]]) {
        const float2* f = sm.fac + slot[u] * L.half_rot + c[u] * FPV;
        float dev = 0.f;
        if (NEOX) rotate_neox<E>(f, lo[u], hi[u], dev);
        else rotate_gptj<E>(f, lo[u], dev);
        if (scoring) atomicAdd(&sm.dev[slot[u]], dev);
      }
      if (INPLACE) {
        st_vec(dst + off[u], lo[u]);
        if (NEOX) st_vec(dst + off[u] + hi_off, hi[u]);
      } else {
        st_stream(dst + off[u], lo[u]);
        if (NEOX) st_stream(dst + off[u] + hi_off, hi[u]);
      }
    }
  }
}

// ------------------------------------------------------ unit iteration --
// Contiguous range of units for this CTA.
__device__ __forceinline__ void cta_range(int64_t total, int64_t& begin, int64_t& end) {
  const int64_t g = gridDim.x, b = blockIdx.x;
  const int64_t q = total / g, r = total % g;
  begin = b * q + (b < r ? b : r);
  end = begin + q + (b < r ? 1 : 0);
}

// Last job whose unit_begin <= unit.
__device__ __forceinline__ int64_t find_job(const JobDev* jobs, int64_t n, int64_t unit) {
  int64_t lo = 0, hi = n - 1;
  while (lo < hi) {
    const int64_t mid = (lo + hi + 1) >> 1;
    if (__ldg(&jobs[mid].unit_begin) <= unit) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// Plain 16-byte vector copy of `nvec` vectors, U in flight per thread.
template <int U = 8>
__device__ __forceinline__ void copy_vecs(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                                          int64_t nvec) {
  for (int64_t base = threadIdx.x; base < nvec; base += (int64_t)U * blockDim.x) {
    uint4 v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t i = base + (int64_t)u * blockDim.x;
      if (i < nvec) v[u] = ld_stream(src + i * 16);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t i = base + (int64_t)u * blockDim.x;
      if (i < nvec) st_stream(dst + i * 16, v[u]);
    }
  }
}

__device__ __forceinline__ void copy_bytes(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                                           int64_t n) {
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) dst[i] = src[i];
}

// ------------------------------------------------------- plain kernel ----
template <bool GATHER, bool VEC>
__global__ void __launch_bounds__(kThreads) plain_pages_kernel(PageLaunch p) {
  int64_t ubeg, uend;
  cta_range(p.total_units, ubeg, uend);
  if (ubeg >= uend) return;
  int64_t ji = find_job(p.jobs, p.num_jobs, ubeg);
  for (int64_t unit = ubeg; unit < uend; ++unit) {
    while (ji + 1 < p.num_jobs && __ldg(&p.jobs[ji + 1].unit_begin) <= unit) ++ji;
    const JobDev j = p.jobs[ji];
    const LayerDev& L = p.layers[j.layer];
    const int64_t page_local = unit - j.unit_begin;
    const int32_t blk = __ldg(&p.indices[j.idx_off + page_local]);
    if (blk == 0) continue;
    if (blk < 0 || blk >= L.num_pages) {
      if (threadIdx.x == 0) atomicOr(p.err, DEV_ERR_BLOCK_RANGE);
      continue;
    }
    for (int pf = 0; pf < L.prefix_size; ++pf) {
      uint8_t* store = p.store_mut + j.stg_off + ((int64_t)pf * j.n_sel + page_local) * L.suffix;
      uint8_t* layer = L.base + (int64_t)pf * L.prefix_stride + (int64_t)blk * L.page_stride;
      const uint8_t* src = GATHER ? layer : store;
      uint8_t* dst = GATHER ? store : layer;
      if (VEC) copy_vecs(src, dst, L.suffix / 16);
      else copy_bytes(src, dst, L.suffix);
    }
  }
}

// ---------------------------------------------- rotate-scatter kernel ----
// Dynamic shared memory: page_size*half_rot float2 factors, then page_size
// floats of per-slot deviation.
template <int KVT, int TABT, bool NEOX>
__global__ void __launch_bounds__(kThreads, 2) rotate_scatter_kernel(PageLaunch p) {
  using E = Elem<KVT>;
  using T = Elem<TABT>;
  extern __shared__ float4 smem_raw[];

  int64_t ubeg, uend;
  cta_range(p.total_units, ubeg, uend);
  if (ubeg >= uend) return;
  const bool want_scores = p.scores != nullptr;
  int64_t ji = find_job(p.jobs, p.num_jobs, ubeg);
  for (int64_t unit = ubeg; unit < uend; ++unit) {
    while (ji + 1 < p.num_jobs && __ldg(&p.jobs[ji + 1].unit_begin) <= unit) ++ji;
    const JobDev j = p.jobs[ji];
    const LayerDev& L = p.layers[j.layer];
    const int64_t page_local = unit - j.unit_begin;
    const int32_t blk = __ldg(&p.indices[j.idx_off + page_local]);
    MetaDev m{};
    if (j.meta >= 0) m = p.metas[j.meta];
    const bool rotate = (j.meta >= 0) && m.rotate && L.has_rot;
    const bool scoring = want_scores && j.score_row >= 0 && j.meta >= 0;
    const PageSmem sm = page_smem(smem_raw, L);
    const int64_t tok0 = page_local * L.page_size;  // chunk token of slot 0
    bool skip = (blk == 0);
    if (!skip && (blk < 0 || blk >= L.num_pages)) {
      if (threadIdx.x == 0) atomicOr(p.err, DEV_ERR_BLOCK_RANGE);
      skip = true;
    }
    if (scoring)
      for (int s = threadIdx.x; s < L.page_size; s += blockDim.x) sm.dev[s] = 0.f;
    if (rotate && !skip) fill_factors<T>(L, p.mode, m.pos_a, m.pos_b, tok0, m.len, sm, p.err);
    if ((rotate && !skip) || scoring) __syncthreads();
    if (!skip) {
      for (int pf = 0; pf < L.prefix_size; ++pf) {
        const uint8_t* src = p.store + j.stg_off + ((int64_t)pf * j.n_sel + page_local) * L.suffix;
        uint8_t* dst = L.base + (int64_t)pf * L.prefix_stride + (int64_t)blk * L.page_stride;
        if (!(rotate && pf == L.k_prefix)) {
          copy_vecs<4>(src, dst, L.suffix / 16);
          continue;
        }
        // (1) rotated vectors of the K rows.
        rotate_rows<E, NEOX, false>(L, src, dst, sm, scoring);
        // (2) vectors of the K rows beyond the rotary part.
        if (L.tail_vecs > 0) {
          const int nt = L.nrows * L.tail_vecs;
          for (int t = threadIdx.x; t < nt; t += blockDim.x) {
            const int row = (int)fdiv((uint32_t)t, L.tail_div);
            const int c = L.rot_vecs + (t - row * L.tail_vecs);
            const int o = row * L.row_bytes + c * 16;
            st_stream(dst + o, ld_stream(src + o));
          }
        }
        // (3) the rest of the region after the K rows (page-first V half).
        const int64_t kbytes = (int64_t)L.nrows * L.row_bytes;
        if (kbytes < L.suffix) copy_vecs<4>(src + kbytes, dst + kbytes, (L.suffix - kbytes) / 16);
      }
    }
    if (scoring) {
      __syncthreads();
      float* out = p.scores + (int64_t)j.score_row * p.score_ld + m.score_col + tok0;
      for (int s = threadIdx.x; s < L.page_size; s += blockDim.x)
        if (tok0 + s < m.len) out[s] = skip ? 0.f : sm.dev[s];
    }
    if ((rotate && !skip) || scoring) __syncthreads();
  }
}

// ------------------------------------------------- in-place rotation ----
__device__ __forceinline__ int64_t find_seg(const SegDev* segs, int64_t n, int64_t unit) {
  int64_t lo = 0, hi = n - 1;
  while (lo < hi) {
    const int64_t mid = (lo + hi + 1) >> 1;
    if (__ldg(&segs[mid].unit_begin) <= unit) lo = mid; else hi = mid - 1;
  }
  return lo;
}

template <int KVT, int TABT, bool NEOX>
__global__ void __launch_bounds__(kThreads, 2) rotate_inplace_kernel(InplaceLaunch p) {
  using E = Elem<KVT>;
  using T = Elem<TABT>;
  extern __shared__ float4 smem_raw[];
  const int64_t total = p.num_layers * p.units_per_layer;
  int64_t ubeg, uend;
  cta_range(total, ubeg, uend);
  if (ubeg >= uend) return;
  int64_t li = ubeg / p.units_per_layer;
  int64_t si = find_seg(p.segs, p.num_segs, ubeg - li * p.units_per_layer);
  for (int64_t unit = ubeg; unit < uend; ++unit) {
    const int64_t l = unit / p.units_per_layer;
    const int64_t w = unit - l * p.units_per_layer;
    if (l != li) { li = l; si = find_seg(p.segs, p.num_segs, w); }
    while (si + 1 < p.num_segs && __ldg(&p.segs[si + 1].unit_begin) <= w) ++si;
    const SegDev sg = p.segs[si];
    const LayerDev& L = p.layers[l];
    const int64_t page = sg.first_page + (w - sg.unit_begin);
    const int64_t bt = sg.blk_off + page;
    if (bt < 0 || bt >= p.block_table_numel) {
      if (threadIdx.x == 0) atomicOr(p.err, DEV_ERR_INDEX_RANGE);
      continue;
    }
    const int32_t blk = __ldg(&p.block_table[bt]);
    if (blk < 0 || blk >= L.num_pages) {
      if (threadIdx.x == 0) atomicOr(p.err, DEV_ERR_BLOCK_RANGE);
      continue;
    }
    uint8_t* kreg = L.base + (int64_t)L.k_prefix * L.prefix_stride + (int64_t)blk * L.page_stride;
    // segment-relative token of slot 0
    const int64_t tok0 = page * L.page_size - sg.tok_start;
    const PageSmem sm = page_smem(smem_raw, L);
    fill_factors<T>(L, p.mode, sg.pos_a, sg.pos_b, tok0, sg.tok_len, sm, p.err);
    __syncthreads();
    rotate_rows<E, NEOX, true>(L, kreg, kreg, sm, false);
    __syncthreads();
  }
}

// ------------------------------------------------------- occupancy ----
template <class K>
int resident_ctas(K kernel, size_t smem) {
  static std::mutex mu;
  static std::unordered_map<const void*, int> cache;
  std::lock_guard<std::mutex> g(mu);
  static std::unordered_map<const void*, size_t> attr_set;
  const void* key = (const void*)kernel;
  if (smem > 48 * 1024 && attr_set[key] < smem) {
    DARIC_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    attr_set[key] = smem;
  }
  const uint64_t ck = ((uint64_t)(uintptr_t)key) ^ ((uint64_t)smem << 48);
  auto it = cache.find((const void*)ck);
  if (it != cache.end()) return it->second;
  int n = 0;
  DARIC_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, kThreads, smem));
  if (n < 1) n = 1;
  cache[(const void*)ck] = n;
  return n;
}

template <class K, class P>
void launch_persistent(K kernel, const P& params, int64_t units, int sm_count, cudaStream_t s,
                       size_t smem = 0) {
  if (units <= 0) return;
  const int64_t cap = (int64_t)sm_count * resident_ctas(kernel, smem);
  const int grid = (int)(units < cap ? units : cap);
  kernel<<<grid, kThreads, smem, s>>>(params);
  DARIC_CUDA(cudaGetLastError());
}

template <int KVT, int TABT>
void dispatch_rotate_scatter(const PageLaunch& p, bool neox, int sm, cudaStream_t s) {
  if (neox) launch_persistent(rotate_scatter_kernel<KVT, TABT, true>, p, p.total_units, sm, s, p.smem_bytes);
  else launch_persistent(rotate_scatter_kernel<KVT, TABT, false>, p, p.total_units, sm, s, p.smem_bytes);
}

template <int KVT>
void dispatch_rotate_scatter_tab(const PageLaunch& p, int tab, bool neox, int sm, cudaStream_t s) {
  switch (tab) {
    case DARIC_DTYPE_BF16: return dispatch_rotate_scatter<KVT, DARIC_DTYPE_BF16>(p, neox, sm, s);
    case DARIC_DTYPE_F16: return dispatch_rotate_scatter<KVT, DARIC_DTYPE_F16>(p, neox, sm, s);
    case DARIC_DTYPE_F32: return dispatch_rotate_scatter<KVT, DARIC_DTYPE_F32>(p, neox, sm, s);
  }
  throw Error(DARIC_ERR_INVALID, "unsupported rotary table dtype");
}

template <int KVT, int TABT>
void dispatch_rotate_inplace(const InplaceLaunch& p, bool neox, int sm, cudaStream_t s) {
  const int64_t units = p.num_layers * p.units_per_layer;
  if (neox) launch_persistent(rotate_inplace_kernel<KVT, TABT, true>, p, units, sm, s, p.smem_bytes);
  else launch_persistent(rotate_inplace_kernel<KVT, TABT, false>, p, units, sm, s, p.smem_bytes);
}

template <int KVT>
void dispatch_rotate_inplace_tab(const InplaceLaunch& p, int tab, bool neox, int sm, cudaStream_t s) {
  switch (tab) {
    case DARIC_DTYPE_BF16: return dispatch_rotate_inplace<KVT, DARIC_DTYPE_BF16>(p, neox, sm, s);
    case DARIC_DTYPE_F16: return dispatch_rotate_inplace<KVT, DARIC_DTYPE_F16>(p, neox, sm, s);
    case DARIC_DTYPE_F32: return dispatch_rotate_inplace<KVT, DARIC_DTYPE_F32>(p, neox, sm, s);
  }
  throw Error(DARIC_ERR_INVALID, "unsupported rotary table dtype");
}

}  // namespace

void launch_plain_pages(const PageLaunch& p, bool gather, bool vec16, int sm, cudaStream_t s) {
  if (gather) {
    if (vec16) launch_persistent(plain_pages_kernel<true, true>, p, p.total_units, sm, s);
    else launch_persistent(plain_pages_kernel<true, false>, p, p.total_units, sm, s);
  } else {
    if (vec16) launch_persistent(plain_pages_kernel<false, true>, p, p.total_units, sm, s);
    else launch_persistent(plain_pages_kernel<false, false>, p, p.total_units, sm, s);
  }
}

void launch_rotate_scatter(const PageLaunch& p, RotKey k, int sm, cudaStream_t s) {
  switch (k.kv_dtype) {
    case DARIC_DTYPE_BF16: return dispatch_rotate_scatter_tab<DARIC_DTYPE_BF16>(p, k.tab_dtype, k.neox, sm, s);
    case DARIC_DTYPE_F16: return dispatch_rotate_scatter_tab<DARIC_DTYPE_F16>(p, k.tab_dtype, k.neox, sm, s);
    case DARIC_DTYPE_F32: return dispatch_rotate_scatter_tab<DARIC_DTYPE_F32>(p, k.tab_dtype, k.neox, sm, s);
    case DARIC_DTYPE_FP8_E4M3:
      return dispatch_rotate_scatter_tab<DARIC_DTYPE_FP8_E4M3>(p, k.tab_dtype, k.neox, sm, s);
  }
  throw Error(DARIC_ERR_INVALID, "unsupported KV dtype");
}

void launch_rotate_inplace(const InplaceLaunch& p, RotKey k, int sm, cudaStream_t s) {
  switch (k.kv_dtype) {
    case DARIC_DTYPE_BF16: return dispatch_rotate_inplace_tab<DARIC_DTYPE_BF16>(p, k.tab_dtype, k.neox, sm, s);
    case DARIC_DTYPE_F16: return dispatch_rotate_inplace_tab<DARIC_DTYPE_F16>(p, k.tab_dtype, k.neox, sm, s);
    case DARIC_DTYPE_F32: return dispatch_rotate_inplace_tab<DARIC_DTYPE_F32>(p, k.tab_dtype, k.neox, sm, s);
    case DARIC_DTYPE_FP8_E4M3:
      return dispatch_rotate_inplace_tab<DARIC_DTYPE_FP8_E4M3>(p, k.tab_dtype, k.neox, sm, s);
  }
  throw Error(DARIC_ERR_INVALID, "unsupported KV dtype");
}

}  // namespace daric
