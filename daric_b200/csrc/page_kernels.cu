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
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include <mutex>
#include <unordered_map>

#include "internal.h"

namespace daric {
namespace {

constexpr int kThreads = 256;

// ------------------------------------------------------------ vector I/O --
__device__ __forceinline__ uint4 ld_stream(const uint8_t* p) {
  return __ldcs(reinterpret_cast<const uint4*>(p));
}
__device__ __forceinline__ void st_stream(uint8_t* p, uint4 v) {
  __stcs(reinterpret_cast<uint4*>(p), v);
}
// In-place path: plain cached loads/stores (the data is read then written).
__device__ __forceinline__ uint4 ld_vec(const uint8_t* p) {
  return *reinterpret_cast<const uint4*>(p);
}
__device__ __forceinline__ void st_vec(uint8_t* p, uint4 v) { *reinterpret_cast<uint4*>(p) = v; }

// ------------------------------------------------------ element traits --
// Conversions follow the reference kernel: load -> fp32, rotate in fp32,
// store converted to the cache dtype with round-to-nearest-even (fp8 e4m3
// saturates to the largest finite value, as Triton's fp32->e4m3 cast does).
template <int DT>
struct Elem;

template <>
struct Elem<DARIC_DTYPE_BF16> {
  using raw = uint16_t;
  static constexpr int kPerVec = 8;
  __device__ __forceinline__ static float to_f(raw v) { return __uint_as_float(((uint32_t)v) << 16); }
  __device__ __forceinline__ static raw from_f(float f) {
    __nv_bfloat16 b = __float2bfloat16_rn(f);
    return *reinterpret_cast<raw*>(&b);
  }
  __device__ __forceinline__ static float round_f(float f) { return to_f(from_f(f)); }
};

template <>
struct Elem<DARIC_DTYPE_F16> {
  using raw = uint16_t;
  static constexpr int kPerVec = 8;
  __device__ __forceinline__ static float to_f(raw v) {
    __half h = *reinterpret_cast<__half*>(&v);
    return __half2float(h);
  }
  __device__ __forceinline__ static raw from_f(float f) {
    __half h = __float2half_rn(f);
    return *reinterpret_cast<raw*>(&h);
  }
  __device__ __forceinline__ static float round_f(float f) { return to_f(from_f(f)); }
};

template <>
struct Elem<DARIC_DTYPE_F32> {
  using raw = uint32_t;
  static constexpr int kPerVec = 4;
  __device__ __forceinline__ static float to_f(raw v) { return __uint_as_float(v); }
  __device__ __forceinline__ static raw from_f(float f) { return __float_as_uint(f); }
  __device__ __forceinline__ static float round_f(float f) { return f; }
};

template <>
struct Elem<DARIC_DTYPE_FP8_E4M3> {
  using raw = uint8_t;
  static constexpr int kPerVec = 16;
  __device__ __forceinline__ static float to_f(raw v) {
    __half_raw h = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)v, __NV_E4M3);
    return __half2float(__half(h));
  }
  __device__ __forceinline__ static raw from_f(float f) {
    return (raw)__nv_cvt_float_to_fp8(f, __NV_SATFINITE, __NV_E4M3);
  }
  __device__ __forceinline__ static float round_f(float f) { return to_f(from_f(f)); }
};

template <class E>
__device__ __forceinline__ void unpack(uint4 v, float (&out)[E::kPerVec]) {
  const typename E::raw* r = reinterpret_cast<const typename E::raw*>(&v);
#pragma unroll
  for (int i = 0; i < E::kPerVec; ++i) out[i] = E::to_f(r[i]);
}

template <class E>
__device__ __forceinline__ uint4 pack(const float (&in)[E::kPerVec]) {
  uint4 v;
  typename E::raw* r = reinterpret_cast<typename E::raw*>(&v);
#pragma unroll
  for (int i = 0; i < E::kPerVec; ++i) r[i] = E::from_f(in[i]);
  return v;
}

// cos/sin factor of one rotary frequency `d` (fp32 result).
//   FLEXIBLE: C = n_c*o_c + n_s*o_s, S = n_s*o_c - n_c*o_s, every product and
//             sum rounded to the table dtype (torch ops on the model-dtype
//             table, adapter.py:276-283).
//   DELTA   : C, S = table row `pa` (adapter.py:181-183).
template <class T>
__device__ __forceinline__ float2 rope_factor(const LayerDev& L, int mode, int64_t pa, int64_t pb, int d) {
  using R = typename T::raw;
  const R* orow = reinterpret_cast<const R*>(L.table + pa * L.table_row);
  if (mode == DARIC_ROPE_DELTA) return make_float2(T::to_f(orow[d]), T::to_f(orow[L.half_rot + d]));
  const R* nrow = reinterpret_cast<const R*>(L.table + pb * L.table_row);
  const float oc = T::to_f(orow[d]), os = T::to_f(orow[L.half_rot + d]);
  const float nc = T::to_f(nrow[d]), ns = T::to_f(nrow[L.half_rot + d]);
  const float a = T::round_f(__fmul_rn(nc, oc));
  const float b = T::round_f(__fmul_rn(ns, os));
  const float c = T::round_f(__fmul_rn(ns, oc));
  const float e = T::round_f(__fmul_rn(nc, os));
  return make_float2(T::round_f(__fadd_rn(a, b)), T::round_f(__fsub_rn(c, e)));
}

// Shared-memory layout of a page's rotation state:
//   fac[page_size*half_rot] float2 factors, ok[page_size] int flags,
//   dev[page_size] float deviations.
struct PageSmem {
  float2* fac;
  int* ok;
  float* dev;
};

__device__ __forceinline__ PageSmem page_smem(void* base, const LayerDev& L) {
  PageSmem s;
  s.fac = reinterpret_cast<float2*>(base);
  s.ok = reinterpret_cast<int*>(s.fac + L.page_size * L.half_rot);
  s.dev = reinterpret_cast<float*>(s.ok + L.page_size);
  return s;
}

// Fills the factors of the page slots s whose token t = tok0 + s lies in
// [0, len): positions (a + t, b + t) in FLEXIBLE mode, a in DELTA mode.
// ok[s] = 0 marks slots that are not rotated (outside the range, or a
// position outside the table, which also sets the device error bit).
template <class T>
__device__ __forceinline__ void fill_factors(const LayerDev& L, int mode, int64_t pa, int64_t pb,
                                             int64_t tok0, int64_t len, PageSmem sm, int* err) {
  for (int s = threadIdx.x; s < L.page_size; s += blockDim.x) {
    const int64_t t = tok0 + s;
    int ok = 0;
    if (t >= 0 && t < len) {
      int64_t a = pa, b = pb;
      if (mode == DARIC_ROPE_FLEXIBLE) { a += t; b += t; }
      ok = a >= 0 && a < L.max_pos && (mode != DARIC_ROPE_FLEXIBLE || (b >= 0 && b < L.max_pos));
      if (!ok) atomicOr(err, DEV_ERR_TABLE_RANGE);
    }
    sm.ok[s] = ok;
  }
  __syncthreads();
  const int n = L.page_size * L.half_rot;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int s = i / L.half_rot, d = i - s * L.half_rot;
    if (!sm.ok[s]) continue;
    const int64_t t = tok0 + s;
    int64_t a = pa, b = pb;
    if (mode == DARIC_ROPE_FLEXIBLE) { a += t; b += t; }
    sm.fac[i] = rope_factor<T>(L, mode, a, b, d);
  }
}

// Rotates one NeoX pair of vectors (x1 = elements d0.., x2 = d0+half..):
//   x1' = x1*C - x2*S ; x2' = x2*C + x1*S   (fp32, no contraction)
// and accumulates the squared change of the stored values into `dev`.
template <class E>
__device__ __forceinline__ void rotate_neox(const float2* f, uint4& lo, uint4& hi, float& dev) {
  constexpr int N = E::kPerVec;
  float k1[N], k2[N], o1[N], o2[N];
  unpack<E>(lo, k1);
  unpack<E>(hi, k2);
#pragma unroll
  for (int i = 0; i < N; ++i) {
    const float2 cs = f[i];
    o1[i] = __fsub_rn(__fmul_rn(k1[i], cs.x), __fmul_rn(k2[i], cs.y));
    o2[i] = __fadd_rn(__fmul_rn(k2[i], cs.x), __fmul_rn(k1[i], cs.y));
  }
  lo = pack<E>(o1);
  hi = pack<E>(o2);
  float r1[N], r2[N];
  unpack<E>(lo, r1);
  unpack<E>(hi, r2);
#pragma unroll
  for (int i = 0; i < N; ++i) {
    const float a = r1[i] - k1[i];
    const float b = r2[i] - k2[i];
    dev += a * a + b * b;
  }
}

// Rotates one GPT-J vector: adjacent pairs (2m, 2m+1) with factor f[m].
template <class E>
__device__ __forceinline__ void rotate_gptj(const float2* f, uint4& v, float& dev) {
  constexpr int N = E::kPerVec;
  float k[N], o[N];
  unpack<E>(v, k);
#pragma unroll
  for (int m = 0; m < N / 2; ++m) {
    const float2 cs = f[m];
    const float x1 = k[2 * m], x2 = k[2 * m + 1];
    o[2 * m] = __fsub_rn(__fmul_rn(x1, cs.x), __fmul_rn(x2, cs.y));
    o[2 * m + 1] = __fadd_rn(__fmul_rn(x2, cs.x), __fmul_rn(x1, cs.y));
  }
  v = pack<E>(o);
  float r[N];
  unpack<E>(v, r);
#pragma unroll
  for (int i = 0; i < N; ++i) {
    const float a = r[i] - k[i];
    dev += a * a;
  }
}

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
