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

// Packs N fp32 values into one 16-byte vector of the element type, two at a
// time with the paired round-to-nearest-even conversions (bit-identical to
// converting each value on its own).
template <class E>
__device__ __forceinline__ uint4 pack_vec(const float (&in)[E::kPerVec]);

template <>
__device__ __forceinline__ uint4 pack_vec<Elem<DARIC_DTYPE_BF16>>(const float (&in)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 h = __floats2bfloat162_rn(in[2 * i], in[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t*>(&h);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}
template <>
__device__ __forceinline__ uint4 pack_vec<Elem<DARIC_DTYPE_F16>>(const float (&in)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 h = __floats2half2_rn(in[2 * i], in[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t*>(&h);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}
template <>
__device__ __forceinline__ uint4 pack_vec<Elem<DARIC_DTYPE_F32>>(const float (&in)[4]) {
  return make_uint4(__float_as_uint(in[0]), __float_as_uint(in[1]), __float_as_uint(in[2]),
                    __float_as_uint(in[3]));
}
template <>
__device__ __forceinline__ uint4 pack_vec<Elem<DARIC_DTYPE_FP8_E4M3>>(const float (&in)[16]) {
  return pack<Elem<DARIC_DTYPE_FP8_E4M3>>(in);
}

// Flexible-mode combination of the old and new table entries of one
// frequency: C = n_c*o_c + n_s*o_s, S = n_s*o_c - n_c*o_s, every product and
// sum rounded to the table dtype (torch ops on the model-dtype table,
// adapter.py:276-283).
template <class T>
__device__ __forceinline__ float2 rope_combine(float oc, float os, float nc, float ns) {
  const float a = T::round_f(__fmul_rn(nc, oc));
  const float b = T::round_f(__fmul_rn(ns, os));
  const float c = T::round_f(__fmul_rn(ns, oc));
  const float e = T::round_f(__fmul_rn(nc, os));
  return make_float2(T::round_f(__fadd_rn(a, b)), T::round_f(__fsub_rn(c, e)));
}

// cos/sin factor of one rotary frequency `d` (fp32 result).
//   FLEXIBLE: rope_combine of table rows pa (old) and pb (new).
//   DELTA   : C, S = table row `pa` (adapter.py:181-183).
template <class T>
__device__ __forceinline__ float2 rope_factor(const uint8_t* table, int64_t table_row, int half_rot, int mode,
                                              int64_t pa, int64_t pb, int d) {
  using R = typename T::raw;
  const R* orow = reinterpret_cast<const R*>(table + pa * table_row);
  if (mode == DARIC_ROPE_DELTA) return make_float2(T::to_f(orow[d]), T::to_f(orow[half_rot + d]));
  const R* nrow = reinterpret_cast<const R*>(table + pb * table_row);
  return rope_combine<T>(T::to_f(orow[d]), T::to_f(orow[half_rot + d]), T::to_f(nrow[d]),
                         T::to_f(nrow[half_rot + d]));
}

// NF consecutive table entries starting at p (NF * sizeof(raw) bytes,
// aligned to that size up to 16 bytes), widened to fp32 with vector loads
// through the read-only cache.
template <class T, int NF>
__device__ __forceinline__ void load_entries(const uint8_t* p, float (&out)[NF]) {
  using R = typename T::raw;
  constexpr int B = NF * (int)sizeof(R);
  union {
    uint4 q[(B + 15) / 16];
    uint2 h[(B + 7) / 8];
    uint32_t w[(B + 3) / 4];
    R r[NF];
  } u;
  if constexpr (B % 16 == 0) {
#pragma unroll
    for (int k = 0; k < B / 16; ++k) u.q[k] = __ldg(reinterpret_cast<const uint4*>(p) + k);
  } else if constexpr (B == 8) {
    u.h[0] = __ldg(reinterpret_cast<const uint2*>(p));
  } else if constexpr (B == 4) {
    u.w[0] = __ldg(reinterpret_cast<const uint32_t*>(p));
  } else {
#pragma unroll
    for (int k = 0; k < NF; ++k) u.r[k] = reinterpret_cast<const R*>(p)[k];
  }
#pragma unroll
  for (int k = 0; k < NF; ++k) out[k] = T::to_f(u.r[k]);
}

// Factors of frequencies [d0, d0 + NF) of one token straight from the
// table, in the q layout of rotate_*_q with P = 1:
//   q[g] = {C[d0+2g], C[d0+2g+1], S[d0+2g], S[d0+2g+1]}.
// DELTA: row pa; FLEXIBLE: rope_combine of rows pa (old) and pb (new).
// Bit-identical to rope_factor per frequency.
template <class T, int NF>
__device__ __forceinline__ void table_factors(const uint8_t* table, int64_t table_row, int half_rot, bool delta,
                                              int64_t pa, int64_t pb, int d0, float4 (&q)[NF / 2]) {
  constexpr int ES = (int)sizeof(typename T::raw);
  const uint8_t* orow = table + pa * table_row;
  float oc[NF], os[NF];
  load_entries<T, NF>(orow + d0 * ES, oc);
  load_entries<T, NF>(orow + (half_rot + d0) * ES, os);
  if (!delta) {
    const uint8_t* nrow = table + pb * table_row;
    float nc[NF], ns[NF];
    load_entries<T, NF>(nrow + d0 * ES, nc);
    load_entries<T, NF>(nrow + (half_rot + d0) * ES, ns);
#pragma unroll
    for (int k = 0; k < NF; ++k) {
      const float2 f = rope_combine<T>(oc[k], os[k], nc[k], ns[k]);
      oc[k] = f.x;
      os[k] = f.y;
    }
  }
#pragma unroll
  for (int g = 0; g < NF / 2; ++g) q[g] = make_float4(oc[2 * g], oc[2 * g + 1], os[2 * g], os[2 * g + 1]);
}

// Compact factor entry {C[d0], C[d0+1], S[d0], S[d0+1]} stored as 4 x bf16
// (low half = d0): widening bf16 to fp32 is exact.
__device__ __forceinline__ float4 widen_factors(uint2 w) {
  return make_float4(__uint_as_float(w.x << 16), __uint_as_float(w.x & 0xffff0000u), __uint_as_float(w.y << 16),
                     __uint_as_float(w.y & 0xffff0000u));
}

// Factor layout of one token (written by the factor pre-pass): the rotation
// task c of a row (c < P = half_rot / FPV) uses FPV consecutive frequencies
// d = c*FPV + j; they are stored as FPV/2 float4 groups
//   q[g*P + c] = {C[d0], C[d0+1], S[d0], S[d0+1]},  d0 = c*FPV + 2g,
// so the 32 lanes of a warp (consecutive c) read consecutive 16-byte words.
// FPV = elements per 16-byte vector (NeoX) or half of it (GPT-J). Launches
// that read the factors from L2 instead of shared memory use the contiguous
// form q[c*NG + g] (NG = FPV/2 entries of a task in one run: one or a few
// 16-byte loads per task).

// x1' = x1*C - x2*S ; x2' = x2*C + x1*S on NeoX halves, in fp32 with every
// product and sum rounded separately (__fmul_rn / __fadd_rn / __fsub_rn are
// never fused into an FMA), rounded back to the element type. (Paired f32x2
// products measured slower here: the operand packing costs more moves than
// the pairing saves, and a paired product feeding a paired sum is contracted
// into an FMA by the code generator even with explicit .rn modifiers.)
template <class E, bool SCORE>
__device__ __forceinline__ void rotate_neox_q(const float4* q, int P, uint4& lo, uint4& hi, float& dev) {
  constexpr int N = E::kPerVec;
  float k1[N], k2[N], o1[N], o2[N];
  unpack<E>(lo, k1);
  unpack<E>(hi, k2);
#pragma unroll
  for (int g = 0; g < N / 2; ++g) {
    const float4 f = q[g * P];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const float c = e ? f.y : f.x, s = e ? f.w : f.z;
      const float x1 = k1[2 * g + e], x2 = k2[2 * g + e];
      o1[2 * g + e] = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
      o2[2 * g + e] = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
    }
  }
  lo = pack_vec<E>(o1);
  hi = pack_vec<E>(o2);
  if (SCORE) {
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
}

// GPT-J: adjacent pairs (2m, 2m+1) of one vector rotate with frequency
// c*FPV + m.
template <class E, bool SCORE>
__device__ __forceinline__ void rotate_gptj_q(const float4* q, int P, uint4& v, float& dev) {
  constexpr int N = E::kPerVec;
  float k[N], o[N];
  unpack<E>(v, k);
#pragma unroll
  for (int g = 0; g < N / 4; ++g) {
    const float4 f = q[g * P];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const float c = e ? f.y : f.x, s = e ? f.w : f.z;
      const float x1 = k[4 * g + 2 * e], x2 = k[4 * g + 2 * e + 1];  // (even, odd)
      o[4 * g + 2 * e] = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
      o[4 * g + 2 * e + 1] = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
    }
  }
  v = pack_vec<E>(o);
  if (SCORE) {
    float r[N];
    unpack<E>(v, r);
#pragma unroll
    for (int i = 0; i < N; ++i) {
      const float a = r[i] - k[i];
      dev += a * a;
    }
  }
}

// Adds a per-task deviation to its token's slot. The lanes of a warp that
// share a slot form aligned groups (a warp's tasks are consecutive: pair
// tasks of a row, then the rows (heads) of a token); the warp finds the
// largest such group size, sums within the groups by shuffles and one lane
// per group adds. Must be called by all 32 lanes of the warp.
__device__ __forceinline__ void score_add(float* dev, int slot, float v) {
  const unsigned full = 0xffffffffu;
  const int s0 = __shfl_sync(full, slot, 0);
  if (__all_sync(full, slot == s0)) {  // the whole warp on one token
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(full, v, o);
    if ((threadIdx.x & 31) == 0 && s0 >= 0) atomicAdd(&dev[s0], v);
    return;
  }
  int seg = 1;
#pragma unroll
  for (int o = 1; o < 16; o <<= 1) {
    if (!__all_sync(full, __shfl_xor_sync(full, slot, o) == slot)) break;
    v += __shfl_xor_sync(full, v, o);
    seg = o << 1;
  }
  if (((threadIdx.x & 31) & (seg - 1)) == 0 && slot >= 0) atomicAdd(&dev[slot], v);
}

// Token slot of K row `row` of a page region.
__device__ __forceinline__ int row_slot(const LayerDev& L, int row) {
  const uint32_t q = fdiv((uint32_t)row, L.tok_div);
  return (int)(q - fdiv(q, L.tok_mod) * (uint32_t)L.page_size);
}

}  // namespace dev
}  // namespace daric
