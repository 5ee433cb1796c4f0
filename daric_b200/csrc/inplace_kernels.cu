// Copy-engine pipeline of the in-place K re-rotation (sm_100a): strict PIC
// (adapter.py:118-194, rotate by a fixed delta per group) and flexible PIC
// on an already scattered cache (adapter.py:196-295), all layers of a KV
// group in one launch where the reference launches its Triton kernel
// (adapter.py:30-88) once per layer.
//
// A unit is up to pages_per_unit pages of one segment of one layer. For every
// page the producer warp moves the byte range of the segment's tokens inside
// the page's K region (one run for token-major rows, one per head for the
// head-major 4-D layout) into a shared-memory stage with cp.async.bulk
// (mbarrier completion); the consumer warps rotate those rows in shared
// memory and the producer writes exactly the same byte ranges back with
// cp.async.bulk stores. Rows of other tokens of a shared page are neither
// loaded nor stored, so segments that meet inside a page never race. V is
// never read. Each token's cos/sin come from the factor buffer of the factor
// pre-pass when the launch has one (FLEXIBLE: the pre-pass combines rows
// old + t and new + t once per token, on a side stream beside the previous
// kernel), else straight from the model's table (DELTA: row delta; FLEXIBLE
// without a buffer: the two rows combined per task with one rounding per op
// in the table dtype, as rope_factor).
//
// Every wait is bounded (kWaitNs):
// a wait that gives up sets DEV_ERR_TIMEOUT, the producer drains the loads
// still in flight into its stages and the CTA returns.
#include <map>
#include <mutex>
#include <type_traits>

#include "bulk_common.cuh"
#include "device_common.cuh"
#include "internal.h"

namespace daric {
namespace {
using namespace dev;
using namespace bulk;

constexpr int kInMaxWarps = 16;                     // consumer warps of the largest CTA
constexpr int kInThreads = kInMaxWarps * 32 + 32;   // plus the producer warp
constexpr int kInMaxPages = 8;

struct InMeta {                 // written by the producer lane that prefetched the unit
  uint8_t* kb[kInMaxPages];     // K region of each page in global memory; nullptr: not copied
  int64_t tok0;                 // segment token of page 0, slot 0 (may be negative)
  int64_t pos_a, pos_b;         // the segment's positions (DELTA: pos_a = delta)
  int64_t fac_tok;              // factor-buffer token of the segment's token 0
  int32_t layer;
  int32_t npg;                  // pages in the unit
  int32_t bytes;                // bytes loaded for the unit
  int32_t pad;
  uint32_t trange[kInMaxPages]; // token range [lo, hi) of each page: lo | hi << 16
};
static_assert(128 + kMaxStages * sizeof(InMeta) <= kBulkHeader, "stage meta exceeds the header");

__device__ __forceinline__ int64_t find_seg(const SegDev* segs, int64_t n, int64_t w) {
  int64_t lo = 0, hi = n - 1;
  while (lo < hi) {
    const int64_t mid = (lo + hi + 1) >> 1;
    if (__ldg(&segs[mid].unit_begin) <= w) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// Token-run geometry of a layer's K region: `runs` runs of page_size tokens
// (one per head for head-major rows), tok_bytes per token in a run.
struct RunGeom {
  int runs, tok_bytes, run_stride;
};
__device__ __forceinline__ RunGeom run_geom(const LayerDev& L) {
  const int per_tok = (int)L.tok_div.d;  // consecutive rows of one token
  RunGeom r;
  r.tok_bytes = per_tok * L.row_bytes;
  r.run_stride = L.page_size * r.tok_bytes;
  r.runs = L.nrows / (per_tok * L.page_size);
  return r;
}

// Rotates the unit's rows in shared memory. A task is (page g, token slot
// sl, head group hq, 16-byte column c): it fetches the token's cos/sin for
// the column once and rotates rows hq, hq + hs, ... of the token (of R rows;
// hs head groups share a token so that the tasks of a full unit cover the
// consumer threads). Consecutive lanes take consecutive columns, so a
// quarter warp reads one contiguous 128-byte row segment. Only tokens inside
// the page's range are touched.
// fac: the launch's factor buffer (compact 4 x bf16 entries for bf16
// tables, 4 x fp32 otherwise; entry c + k * P of token t at index
// t * half_rot / 2 + c + k * P), or nullptr to read the table.
template <class E, class T, bool NEOX>
__device__ __forceinline__ void rotate_unit(const LayerDev& L, uint32_t stage, int kbytes, const InMeta& st,
                                            bool delta, const uint8_t* fac, int tid, int nthreads) {
  constexpr int N = E::kPerVec;
  constexpr int NF = NEOX ? N : N / 2;  // frequencies of one column
  const int P = L.pair_vecs;
  const int bs = L.page_size;
  const int R = L.nrows / bs;           // rows of one token
  const int per_tok = (int)L.tok_div.d;
  // row of the token's k-th row: token-major (one run) sl * R + k, or
  // head-major (R runs of bs rows) k * bs + sl
  const int sl_mul = per_tok == R ? R : 1;
  const int k_mul = per_tok == R ? 1 : bs;
  const int base_tasks = st.npg * bs * P;
  int hs = 1;
  while (hs < R && R % (2 * hs) == 0 && base_tasks * hs < nthreads) hs *= 2;
  const int hshift = __ffs(hs) - 1;
  const int ntask = base_tasks << hshift;
  const int hi_off = NEOX ? (L.rot_vecs / 2) * 16 : 0;
  // the unit's layer and stage fields, read once into registers: every
  // shared-memory store below is an asm statement with a memory clobber,
  // after which a field read through L or st would be loaded again
  const FastDiv pair_div = L.pair_div, tok_mod = L.tok_mod;
  const uint8_t* const table = L.table;
  const int64_t table_row = L.table_row;
  const int half_rot = L.half_rot, row_bytes = L.row_bytes;
  const int64_t tok0 = st.tok0, pos_a = st.pos_a, pos_b = st.pos_b, fac_tok = st.fac_tok;
  constexpr bool kCompact = std::is_same<T, Elem<DARIC_DTYPE_BF16>>::value;
  constexpr int ES = kCompact ? 8 : 16;  // bytes of a factor-buffer entry
  for (int t = tid; t < ntask; t += nthreads) {
    const int tc = (int)fdiv((uint32_t)t, pair_div);  // t / P
    const int c = t - tc * P;
    const int hq = tc & (hs - 1);
    const int gs = tc >> hshift;                       // g * bs + sl
    const int g = (int)fdiv((uint32_t)gs, tok_mod);
    const int sl = gs - g * bs;
    const uint32_t tr = st.trange[g];
    if (st.kb[g] == nullptr || sl < (int)(tr & 0xffffu) || sl >= (int)(tr >> 16)) continue;
    const int64_t tok = tok0 + (int64_t)g * bs + sl;  // segment token
    float4 q[NF / 2];
    if (fac != nullptr) {
      const uint8_t* fq = fac + ((fac_tok + tok) * (half_rot / 2) + c) * ES;
#pragma unroll
      for (int k = 0; k < NF / 2; ++k) {
        const uint8_t* gp = fq + k * P * ES;
        q[k] = kCompact ? widen_factors(__ldg(reinterpret_cast<const uint2*>(gp)))
                        : __ldg(reinterpret_cast<const float4*>(gp));
      }
    } else {
      table_factors<T, NF>(table, table_row, half_rot, delta, delta ? pos_a : pos_a + tok, pos_b + tok, c * NF, q);
    }
    const uint32_t cbase = stage + (uint32_t)(g * kbytes + c * 16);
#pragma unroll 2
    for (int k = hq; k < R; k += hs) {
      const uint32_t a = cbase + (uint32_t)((sl * sl_mul + k * k_mul) * row_bytes);
      uint4 lo = lds128(a), hi;
      if (NEOX) hi = lds128(a + hi_off);
      float dv = 0.f;
      if (NEOX) rotate_neox_q<E, false>(q, 1, lo, hi, dv);
      else rotate_gptj_q<E, false>(q, 1, lo, dv);
      sts128(a, lo);
      if (NEOX) sts128(a + hi_off, hi);
    }
  }
}

// Warp-specialised pipeline: warps 0..cwarps-1 rotate, the last warp is the
// producer. Its lanes prefetch the plans of 32 units at a time; for unit i
// the lane that prefetched it writes the stage metadata and arms full[i % NS]
// with the unit's byte count, then the warp issues the loads (one run of one
// page per lane). Once every consumer warp has released the unit (empty[s])
// the warp stores the same runs back and reuses the stage of the previous
// unit when its stores have read it.
// Shared memory: [0,128) full/empty barriers | [128,kBulkHeader) stage meta |
// stages (page g of a unit at g * kbytes, rows at their natural offsets).
template <int KVT, int TABT, bool NEOX>
__global__ void __launch_bounds__(kInThreads, 1) bulk_inplace_kernel(InplaceLaunch p, InplaceGeom g) {
  using E = Elem<KVT>;
  using T = Elem<TABT>;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kMaxStages;
  InMeta* meta = reinterpret_cast<InMeta*>(smem + 128);
  uint8_t* stages = smem + kBulkHeader;
  const int NS = g.nstage;
  const int PU = g.pages_per_unit;
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int cwarps = (int)(blockDim.x >> 5) - 1;
  const bool producer = warp == cwarps;
  const bool delta = p.mode == DARIC_ROPE_DELTA;

  int64_t ubeg, uend;
  cta_range(p.num_layers * p.units_per_layer, ubeg, uend);
  if (ubeg >= uend) return;
  const int64_t n = uend - ubeg;

  if (tid == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], cwarps);
    }
    mbar_init_fence();
  }
  __syncthreads();

  if (producer) {
    const unsigned FULL = 0xffffffffu;
    int64_t batch = -1;
    InMeta mine{};
    auto prefetch = [&](int64_t b) {
      const int64_t i = b * 32 + lane;
      mine.npg = 0;
      mine.bytes = 0;
      if (i >= n) return;
      const int64_t u = ubeg + i;
      const int64_t l = u / p.units_per_layer;
      const int64_t w = u - l * p.units_per_layer;
      const SegDev sg = p.segs[find_seg(p.segs, p.num_segs, w)];
      const LayerDev& L = p.layers[l];
      const RunGeom rg = run_geom(L);
      const int r = (int)(w - sg.unit_begin);
      const int pg0 = sg.first_page + r * PU;
      const int npg = min(PU, sg.num_pages - r * PU);
      mine.layer = (int32_t)l;
      mine.npg = npg;
      mine.pos_a = sg.pos_a;
      mine.pos_b = sg.pos_b;
      mine.fac_tok = sg.fac_tok;
      mine.tok0 = (int64_t)pg0 * L.page_size - sg.tok_start;
      int bytes = 0;
      for (int q = 0; q < kInMaxPages; ++q) {
        if (q >= npg) break;
        const int64_t pg = pg0 + q;
        const int64_t p0 = pg * L.page_size;
        const int64_t lo = max(sg.tok_start - p0, (int64_t)0);
        const int64_t hi = min(sg.tok_start + sg.tok_len - p0, (int64_t)L.page_size);
        mine.trange[q] = (uint32_t)lo | ((uint32_t)hi << 16);
        mine.kb[q] = nullptr;
        const int64_t bt = sg.blk_off + pg;
        if (bt < 0 || bt >= p.block_table_numel) {
          atomicOr(p.err, DEV_ERR_INDEX_RANGE);
          continue;
        }
        const int32_t blk = __ldg(&p.block_table[bt]);
        if (blk < 0 || blk >= L.num_pages) {
          atomicOr(p.err, DEV_ERR_BLOCK_RANGE);
          continue;
        }
        if (hi <= lo) continue;
        mine.kb[q] = L.base + (int64_t)L.k_prefix * L.prefix_stride + (int64_t)blk * L.page_stride;
        bytes += rg.runs * (int)(hi - lo) * rg.tok_bytes;
      }
      mine.bytes = bytes;
    };
    // loads of unit i into stage i % NS (all lanes call)
    auto issue = [&](int64_t i) {
      if (g.unarmed && i == 0) return;  // test only: nothing arms unit 0
      const int64_t b = i / 32;
      if (b != batch) {
        prefetch(b);
        batch = b;
      }
      const int k = (int)(i - b * 32);
      const int s = (int)(i % NS);
      const int bytes = __shfl_sync(FULL, mine.bytes, k);
      if (lane == k) {
        meta[s] = mine;
        if (bytes == 0) mbar_arrive(&full[s]);
        else mbar_arrive_expect_tx(&full[s], (uint32_t)bytes);
      }
      if (bytes == 0) return;
      __syncwarp();
      const InMeta& sm = meta[s];
      const LayerDev& L = p.layers[sm.layer];
      const RunGeom rg = run_geom(L);
      uint8_t* buf = stages + (size_t)s * g.stage_bytes;
      const int nops = sm.npg * rg.runs;
      for (int o = lane; o < nops; o += 32) {
        const int q = o / rg.runs, run = o - q * rg.runs;
        uint8_t* kb = sm.kb[q];
        if (kb == nullptr) continue;
        const uint32_t tr = sm.trange[q];
        const int lo = (int)(tr & 0xffffu), hi = (int)(tr >> 16);
        const int off = run * rg.run_stride + lo * rg.tok_bytes;
        bulk_load(buf + (size_t)q * g.kbytes + off, kb + off, (uint32_t)((hi - lo) * rg.tok_bytes), &full[s]);
      }
    };
    bool ok = true;
    int64_t issued = 0;
    while (issued < NS - 1 && issued < n) issue(issued++);
    bool prev_stored = false;
    int64_t i = 0;
    for (; i < n; ++i) {
      const int s = (int)(i % NS);
      const bool got = mbar_wait(&empty[s], (uint32_t)((i / NS) & 1), (uint64_t)g.wait_ns);
      if (__any_sync(FULL, !got)) {
        ok = false;
        break;
      }
      const InMeta& sm = meta[s];
      const bool stored = sm.bytes > 0;
      if (stored) {
        const LayerDev& L = p.layers[sm.layer];
        const RunGeom rg = run_geom(L);
        const uint8_t* buf = stages + (size_t)s * g.stage_bytes;
        const int nops = sm.npg * rg.runs;
        for (int o = lane; o < nops; o += 32) {
          const int q = o / rg.runs, run = o - q * rg.runs;
          uint8_t* kb = sm.kb[q];
          if (kb == nullptr) continue;
          const uint32_t tr = sm.trange[q];
          const int lo = (int)(tr & 0xffffu), hi = (int)(tr >> 16);
          const int off = run * rg.run_stride + lo * rg.tok_bytes;
          bulk_store(kb + off, buf + (size_t)q * g.kbytes + off, (uint32_t)((hi - lo) * rg.tok_bytes));
        }
        bulk_commit();  // every lane commits (possibly empty) groups in step
      }
      __syncwarp();
      if (issued < n) {
        // the next load goes into the stage of unit i-1: its stores must
        // have read it (unit i's group, committed last, may be pending)
        if (prev_stored) {
          if (stored) bulk_wait_read<1>(); else bulk_wait_read<0>();
        }
        __syncwarp();
        issue(issued++);
      }
      prev_stored = stored;
      __syncwarp();
    }
    if (!ok && lane == 0) {
      atomicOr(p.err, DEV_ERR_TIMEOUT);
      // drain the loads that may still be in flight into this CTA's stages
      for (int64_t k = i; k < issued; ++k)
        if (!(g.unarmed && k == 0)) mbar_wait(&full[k % NS], (uint32_t)((k / NS) & 1));
    }
    bulk_wait_all();
    return;
  }

  // consumers
  const uint32_t sbase = smem_addr(stages);
  for (int64_t i = 0; i < n; ++i) {
    const int s = (int)(i % NS);
    if (!mbar_wait(&full[s], (uint32_t)((i / NS) & 1), (uint64_t)g.wait_ns)) {
      atomicOr(p.err, DEV_ERR_TIMEOUT);
      break;
    }
    const InMeta& st = meta[s];
    if (st.bytes > 0) {
      const LayerDev& L = p.layers[st.layer];
      rotate_unit<E, T, NEOX>(L, sbase + (uint32_t)(s * g.stage_bytes), g.kbytes, st, delta,
                              reinterpret_cast<const uint8_t*>(p.fac), tid, cwarps * 32);
      fence_proxy_async();
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }
}

template <class K>
void launch(K kernel, const InplaceLaunch& p, const InplaceGeom& g, int sm_count, cudaStream_t s) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, size_t> attr;  // (kernel, device) -> smem set
  const size_t smem = (size_t)kBulkHeader + (size_t)g.nstage * g.stage_bytes;
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
  const int64_t units = p.num_layers * p.units_per_layer;
  const int64_t ctas = (int64_t)sm_count * g.ctas_per_sm;
  const int grid = (int)(units < ctas ? units : ctas);
  if (grid <= 0) return;
  kernel<<<grid, (g.cwarps + 1) * 32, smem, s>>>(p, g);
  DARIC_CUDA(cudaGetLastError());
}

template <int KVT, int TABT>
void dispatch(const InplaceLaunch& p, const InplaceGeom& g, bool neox, int sm, cudaStream_t s) {
  if (neox) launch(bulk_inplace_kernel<KVT, TABT, true>, p, g, sm, s);
  else launch(bulk_inplace_kernel<KVT, TABT, false>, p, g, sm, s);
}

template <int KVT>
void dispatch_tab(const InplaceLaunch& p, const InplaceGeom& g, bool neox, int sm, cudaStream_t s) {
  switch (g.tab_dtype) {
    case DARIC_DTYPE_BF16: return dispatch<KVT, DARIC_DTYPE_BF16>(p, g, neox, sm, s);
    case DARIC_DTYPE_F16: return dispatch<KVT, DARIC_DTYPE_F16>(p, g, neox, sm, s);
    case DARIC_DTYPE_F32: return dispatch<KVT, DARIC_DTYPE_F32>(p, g, neox, sm, s);
  }
  throw Error(DARIC_ERR_INVALID, "unsupported rotary table dtype");
}

}  // namespace

void launch_bulk_inplace(const InplaceLaunch& p, const InplaceGeom& g, RotKey k, int sm, cudaStream_t s) {
  DARIC_CHECK(g.nstage >= 3 && g.nstage <= kMaxStages && g.pages_per_unit >= 1 &&
                  g.pages_per_unit <= kInMaxPages && g.cwarps >= 1 && g.cwarps <= kInMaxWarps,
              "internal: in-place pipeline geometry");
  switch (k.kv_dtype) {
    case DARIC_DTYPE_BF16: return dispatch_tab<DARIC_DTYPE_BF16>(p, g, k.neox, sm, s);
    case DARIC_DTYPE_F16: return dispatch_tab<DARIC_DTYPE_F16>(p, g, k.neox, sm, s);
    case DARIC_DTYPE_F32: return dispatch_tab<DARIC_DTYPE_F32>(p, g, k.neox, sm, s);
    case DARIC_DTYPE_FP8_E4M3: return dispatch_tab<DARIC_DTYPE_FP8_E4M3>(p, g, k.neox, sm, s);
  }
  throw Error(DARIC_ERR_INVALID, "unsupported KV dtype");
}

}  // namespace daric
