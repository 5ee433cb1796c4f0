// Device helpers shared by the page kernels (SIMT and bulk-copy pipelines):
// element conversions, the rotary factor math and the pair rotation.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include "internal.h"

namespace daric {
namespace dev {

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

}  // namespace dev
}  // namespace daric
