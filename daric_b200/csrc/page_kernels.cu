// SIMT page kernels of the reused-KV path, written for sm_100a.
//
//  * plain_pages_kernel    : store <-> paged KV byte copy. Same byte mapping as
//                            fused_{gather,scatter}_pages_kernel in the
//                            reference (csrc/cache_ops/kernels.cu:7-45, 86-123):
//                            store[(p*n_sel + i)*suffix + o] <->
//                            layer[p*prefix_stride + block[i]*page_stride + o],
//                            block id 0 skipped.
//  * factor_kernel         : rotary factors (cos/sin of the position change) of
//                            every chunk token, once per launch, in the layout
//                            the rotation tasks read (device_common.cuh).
//  * rotate_scatter_kernel : the scatter with the K rows re-rotated on the way,
//                            which the reference does afterwards with the
//                            Triton kernel _fused_rerotate_kernel
//                            (daric/adaption/adapter.py:30-88).
//  * rotate_inplace_kernel : in-place re-rotation of K rows in the paged cache,
//                            all layers in one launch (adapter.py:118-295).
//
// These are the SIMT forms (16-byte vector loads/stores through registers);
// bulk_kernels.cu holds the copy-engine pipeline used when a page fits the
// shared-memory stages. Work is split into "units" (one page of one job, or
// one page of one segment of one layer); a persistent grid of
// sm_count x (resident CTAs per SM) CTAs takes contiguous unit ranges.
#include <mutex>
#include <unordered_map>

#include "device_common.cuh"
#include "internal.h"

namespace daric {
namespace {
using namespace dev;

constexpr int kThreads = 256;

__device__ __forceinline__ void cta_range(int64_t total, int64_t& begin, int64_t& end) {
  const int64_t g = gridDim.x, b = blockIdx.x;
  const int64_t q = total / g, r = total % g;
  begin = b * q + (b < r ? b : r);
  end = begin + q + (b < r ? 1 : 0);
}

// Last entry whose `begin` field is <= key.
template <class D>
__device__ __forceinline__ int64_t find_entry(const D* a, int64_t n, int64_t key, int64_t D::*field) {
  int64_t lo = 0, hi = n - 1;
  while (lo < hi) {
    const int64_t mid = (lo + hi + 1) >> 1;
    if (a[mid].*field <= key) lo = mid; else hi = mid - 1;
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
  int64_t ji = find_entry(p.jobs, p.num_jobs, ubeg, &JobDev::unit_begin);
  for (int64_t unit = ubeg; unit < uend; ++unit) {
    while (ji + 1 < p.num_jobs && p.jobs[ji + 1].unit_begin <= unit) ++ji;
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

// ------------------------------------------------------ factor pre-pass --
// One thread per entry of the factor buffer (4 factors: fp32 float4, or
// bf16 x 4 packed in a uint2 when p.compact): job f covers tokens [0, len)
// of one chunk (or segment) for one rotary table.
template <int TABT>
__global__ void __launch_bounds__(256) factor_kernel(FactorLaunch p) {
  using T = Elem<TABT>;
  for (int64_t w = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; w < p.total_items;
       w += (int64_t)gridDim.x * blockDim.x) {
    const int64_t f = find_entry(p.jobs, p.num_jobs, w, &FacJobDev::item_begin);
    const FacJobDev jb = p.jobs[f];
    const int per_tok = jb.half_rot / 2;  // float4 per token
    const int64_t r = w - jb.item_begin;
    const int64_t t = r / per_tok;
    const int k = (int)(r - t * per_tok);
    const int g = k / jb.P, c = k - g * jb.P;
    const int d0 = c * p.fpv + 2 * g;
    int64_t a = jb.pos_a, b = jb.pos_b;
    if (p.mode == DARIC_ROPE_FLEXIBLE) { a += t; b += t; }
    const float2 f0 = rope_factor<T>(jb.table, jb.table_row, jb.half_rot, p.mode, a, b, d0);
    const float2 f1 = rope_factor<T>(jb.table, jb.table_row, jb.half_rot, p.mode, a, b, d0 + 1);
    // entry (g, c): strided g * P + c (consecutive lanes read consecutive
    // words), or contiguous c * NG + g (a task's NG entries in one run)
    const int64_t e = (jb.out_tok + t) * per_tok + (p.contig ? c * (per_tok / jb.P) + g : k);
    if (p.compact) {
      // bf16 table: every factor is already a bf16 value (rounded in
      // rope_factor), so its upper 16 bits are the exact bf16 encoding
      const uint32_t cw = (__float_as_uint(f0.x) >> 16) | (__float_as_uint(f1.x) & 0xffff0000u);
      const uint32_t sw = (__float_as_uint(f0.y) >> 16) | (__float_as_uint(f1.y) & 0xffff0000u);
      static_cast<uint2*>(p.out)[e] = make_uint2(cw, sw);
    } else {
      static_cast<float4*>(p.out)[e] = make_float4(f0.x, f1.x, f0.y, f1.y);
    }
  }
}

// ---------------------------------------------- rotate-scatter kernel ----
// Rotation tasks of one page region (src -> dst): task t -> (row, c) ->
// vectors at row*row_bytes + c*16 (+ rot_vecs/2*16 for the NeoX partner).
// Slots whose token is not rotated are copied unchanged.
template <class E, bool NEOX, bool SCORE>
__device__ __forceinline__ void rotate_rows_global(const LayerDev& L, const uint8_t* src, uint8_t* dst,
                                                   const float4* fac_page, int64_t tok0, int64_t len,
                                                   float* tok_dev) {
  constexpr int U = 4;
  const int ntask = L.nrows * L.pair_vecs;
  const int hi_off = NEOX ? (L.rot_vecs / 2) * 16 : 0;
  const int per_tok = L.half_rot / 2;
  // warp-uniform trip count (score_add shuffles across the warp)
  for (int base = threadIdx.x; base - (int)(threadIdx.x & 31) < ntask; base += U * blockDim.x) {
    uint4 lo[U], hi[U];
    int off[U], slot[U], c[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int t = base + u * blockDim.x;
      off[u] = -1;
      if (t < ntask) {
        const int row = (int)fdiv((uint32_t)t, L.pair_div);
        c[u] = t - row * L.pair_vecs;
        slot[u] = row_slot(L, row);
        off[u] = row * L.row_bytes + c[u] * 16;
        lo[u] = ld_stream(src + off[u]);
        if (NEOX) hi[u] = ld_stream(src + off[u] + hi_off);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      float dv = 0.f;
      const bool rot = off[u] >= 0 && tok0 + slot[u] < len;
      if (rot) {
        const float4* q = fac_page + (int64_t)slot[u] * per_tok + c[u];
        if (NEOX) rotate_neox_q<E, SCORE>(q, L.pair_vecs, lo[u], hi[u], dv);
        else rotate_gptj_q<E, SCORE>(q, L.pair_vecs, lo[u], dv);
      }
      if (off[u] >= 0) {
        st_stream(dst + off[u], lo[u]);
        if (NEOX) st_stream(dst + off[u] + hi_off, hi[u]);
      }
      if (SCORE) score_add(tok_dev, rot ? slot[u] : -1, dv);
    }
  }
}

template <int KVT, bool NEOX, bool SCORE>
__global__ void __launch_bounds__(kThreads, 2) rotate_scatter_kernel(PageLaunch p) {
  using E = Elem<KVT>;
  __shared__ float tok_dev[1024];
  int64_t ubeg, uend;
  cta_range(p.total_units, ubeg, uend);
  if (ubeg >= uend) return;
  int64_t ji = find_entry(p.jobs, p.num_jobs, ubeg, &JobDev::unit_begin);
  for (int64_t unit = ubeg; unit < uend; ++unit) {
    while (ji + 1 < p.num_jobs && p.jobs[ji + 1].unit_begin <= unit) ++ji;
    const JobDev j = p.jobs[ji];
    const LayerDev& L = p.layers[j.layer];
    const int64_t page_local = unit - j.unit_begin;
    const int32_t blk = __ldg(&p.indices[j.idx_off + page_local]);
    MetaDev m{};
    if (j.meta >= 0) m = p.metas[j.meta];
    const bool rotate = (j.meta >= 0) && m.rotate && L.has_rot;
    const bool scoring = SCORE && j.score_row >= 0 && j.meta >= 0;
    const int64_t tok0 = page_local * L.page_size;  // chunk token of slot 0
    if (scoring) {
      for (int s = threadIdx.x; s < L.page_size; s += blockDim.x) tok_dev[s] = 0.f;
      __syncthreads();
    }
    bool skip = (blk == 0);
    if (!skip && (blk < 0 || blk >= L.num_pages)) {
      if (threadIdx.x == 0) atomicOr(p.err, DEV_ERR_BLOCK_RANGE);
      skip = true;
    }
    if (!skip) {
      for (int pf = 0; pf < L.prefix_size; ++pf) {
        const uint8_t* src = p.store + j.stg_off + ((int64_t)pf * j.n_sel + page_local) * L.suffix;
        uint8_t* dst = L.base + (int64_t)pf * L.prefix_stride + (int64_t)blk * L.page_stride;
        if (!(rotate && pf == L.k_prefix)) {
          copy_vecs<4>(src, dst, L.suffix / 16);
          continue;
        }
        const float4* fac_page = p.fac + (j.fac_tok + tok0) * (L.half_rot / 2);
        rotate_rows_global<E, NEOX, SCORE>(L, src, dst, fac_page, tok0, m.len, tok_dev);
        // vectors of the K rows beyond the rotary part
        if (L.tail_vecs > 0) {
          const int nt = L.nrows * L.tail_vecs;
          for (int t = threadIdx.x; t < nt; t += blockDim.x) {
            const int row = (int)fdiv((uint32_t)t, L.tail_div);
            const int c = L.rot_vecs + (t - row * L.tail_vecs);
            const int o = row * L.row_bytes + c * 16;
            st_stream(dst + o, ld_stream(src + o));
          }
        }
        // the rest of the region after the K rows (page-first V half)
        const int64_t kbytes = (int64_t)L.nrows * L.row_bytes;
        if (kbytes < L.suffix) copy_vecs<4>(src + kbytes, dst + kbytes, (L.suffix - kbytes) / 16);
      }
    }
    if (scoring) {
      __syncthreads();
      float* out = p.scores + (int64_t)j.score_row * p.score_ld + m.score_col + tok0;
      for (int s = threadIdx.x; s < L.page_size; s += blockDim.x)
        if (tok0 + s < m.len) out[s] = skip ? 0.f : tok_dev[s];
      __syncthreads();
    }
  }
}

// ------------------------------------------------- in-place rotation ----
// All layers of one launch share one rotary table, so the factors of a
// segment token are the same for every layer.
template <int KVT, bool NEOX>
__global__ void __launch_bounds__(kThreads, 2) rotate_inplace_kernel(InplaceLaunch p) {
  using E = Elem<KVT>;
  constexpr int U = 4;
  const int64_t total = p.num_layers * p.units_per_layer;
  int64_t ubeg, uend;
  cta_range(total, ubeg, uend);
  if (ubeg >= uend) return;
  int64_t li = ubeg / p.units_per_layer;
  int64_t si = find_entry(p.segs, p.num_segs, ubeg - li * p.units_per_layer, &SegDev::unit_begin);
  for (int64_t unit = ubeg; unit < uend; ++unit) {
    const int64_t l = unit / p.units_per_layer;
    const int64_t w = unit - l * p.units_per_layer;
    if (l != li) { li = l; si = find_entry(p.segs, p.num_segs, w, &SegDev::unit_begin); }
    while (si + 1 < p.num_segs && p.segs[si + 1].unit_begin <= w) ++si;
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
    const int64_t tok0 = page * L.page_size - sg.tok_start;  // segment token of slot 0
    const int per_tok = L.half_rot / 2;
    const float4* fac = p.fac + sg.fac_tok * per_tok;
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
          slot[u] = row_slot(L, row);
          const int64_t tok = tok0 + slot[u];
          if (tok >= 0 && tok < sg.tok_len) {
            off[u] = row * L.row_bytes + c[u] * 16;
            lo[u] = ld_vec(kreg + off[u]);
            if (NEOX) hi[u] = ld_vec(kreg + off[u] + hi_off);
          }
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (off[u] < 0) continue;
        const float4* q = fac + (tok0 + slot[u]) * per_tok + c[u];
        float dv = 0.f;
        if (NEOX) rotate_neox_q<E, false>(q, L.pair_vecs, lo[u], hi[u], dv);
        else rotate_gptj_q<E, false>(q, L.pair_vecs, lo[u], dv);
        st_vec(kreg + off[u], lo[u]);
        if (NEOX) st_vec(kreg + off[u] + hi_off, hi[u]);
      }
    }
  }
}

// ------------------------------------------------------- occupancy ----
template <class K>
int resident_ctas(K kernel) {
  static std::mutex mu;
  static std::unordered_map<const void*, int> cache;
  std::lock_guard<std::mutex> g(mu);
  auto it = cache.find((const void*)kernel);
  if (it != cache.end()) return it->second;
  int n = 0;
  DARIC_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, kThreads, 0));
  if (n < 1) n = 1;
  cache[(const void*)kernel] = n;
  return n;
}

template <class K, class P>
void launch_persistent(K kernel, const P& params, int64_t units, int sm_count, cudaStream_t s) {
  if (units <= 0) return;
  const int64_t cap = (int64_t)sm_count * resident_ctas(kernel);
  const int grid = (int)(units < cap ? units : cap);
  kernel<<<grid, kThreads, 0, s>>>(params);
  DARIC_CUDA(cudaGetLastError());
}

template <int KVT>
void dispatch_rotate_scatter(const PageLaunch& p, bool neox, int sm, cudaStream_t s) {
  const bool sc = p.scores != nullptr;
  if (neox) {
    if (sc) launch_persistent(rotate_scatter_kernel<KVT, true, true>, p, p.total_units, sm, s);
    else launch_persistent(rotate_scatter_kernel<KVT, true, false>, p, p.total_units, sm, s);
  } else {
    if (sc) launch_persistent(rotate_scatter_kernel<KVT, false, true>, p, p.total_units, sm, s);
    else launch_persistent(rotate_scatter_kernel<KVT, false, false>, p, p.total_units, sm, s);
  }
}

template <int KVT>
void dispatch_rotate_inplace(const InplaceLaunch& p, bool neox, int sm, cudaStream_t s) {
  const int64_t units = p.num_layers * p.units_per_layer;
  if (neox) launch_persistent(rotate_inplace_kernel<KVT, true>, p, units, sm, s);
  else launch_persistent(rotate_inplace_kernel<KVT, false>, p, units, sm, s);
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

void launch_factors(const FactorLaunch& p, int tab_dtype, int sm, cudaStream_t s) {
  if (p.total_items <= 0) return;
  if (p.compact && tab_dtype != DARIC_DTYPE_BF16)
    throw Error(DARIC_ERR_INVALID, "bf16 factor entries need a bf16 rotary table");
  int64_t blocks = (p.total_items + 255) / 256;
  const int64_t cap = (int64_t)sm * 8;
  if (blocks > cap) blocks = cap;
  switch (tab_dtype) {
    case DARIC_DTYPE_BF16: factor_kernel<DARIC_DTYPE_BF16><<<(unsigned)blocks, 256, 0, s>>>(p); break;
    case DARIC_DTYPE_F16: factor_kernel<DARIC_DTYPE_F16><<<(unsigned)blocks, 256, 0, s>>>(p); break;
    case DARIC_DTYPE_F32: factor_kernel<DARIC_DTYPE_F32><<<(unsigned)blocks, 256, 0, s>>>(p); break;
    default: throw Error(DARIC_ERR_INVALID, "unsupported rotary table dtype");
  }
  DARIC_CUDA(cudaGetLastError());
}

void launch_rotate_scatter(const PageLaunch& p, RotKey k, int sm, cudaStream_t s) {
  switch (k.kv_dtype) {
    case DARIC_DTYPE_BF16: return dispatch_rotate_scatter<DARIC_DTYPE_BF16>(p, k.neox, sm, s);
    case DARIC_DTYPE_F16: return dispatch_rotate_scatter<DARIC_DTYPE_F16>(p, k.neox, sm, s);
    case DARIC_DTYPE_F32: return dispatch_rotate_scatter<DARIC_DTYPE_F32>(p, k.neox, sm, s);
    case DARIC_DTYPE_FP8_E4M3: return dispatch_rotate_scatter<DARIC_DTYPE_FP8_E4M3>(p, k.neox, sm, s);
  }
  throw Error(DARIC_ERR_INVALID, "unsupported KV dtype");
}

void launch_rotate_inplace(const InplaceLaunch& p, RotKey k, int sm, cudaStream_t s) {
  switch (k.kv_dtype) {
    case DARIC_DTYPE_BF16: return dispatch_rotate_inplace<DARIC_DTYPE_BF16>(p, k.neox, sm, s);
    case DARIC_DTYPE_F16: return dispatch_rotate_inplace<DARIC_DTYPE_F16>(p, k.neox, sm, s);
    case DARIC_DTYPE_F32: return dispatch_rotate_inplace<DARIC_DTYPE_F32>(p, k.neox, sm, s);
    case DARIC_DTYPE_FP8_E4M3: return dispatch_rotate_inplace<DARIC_DTYPE_FP8_E4M3>(p, k.neox, sm, s);
  }
  throw Error(DARIC_ERR_INVALID, "unsupported KV dtype");
}

}  // namespace daric
