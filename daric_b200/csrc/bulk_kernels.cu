// Bulk-copy pipeline for the page copies of the reused-KV path (sm_100a).
//
// Persistent CTAs (one to four per SM) each walk batches of consecutive
// units (up to 8 consecutive pages of one job): a first batch by CTA index,
// then batches claimed from the launch's work counter, smaller towards the
// end, so CTAs that start late (an SM busy with another stream's kernel)
// take fewer units instead of finishing late. Each unit's regions
// (prefix_size x suffix bytes per page: the K and V planes) are moved by the
// SM's copy unit with untiled cp.async.bulk loads into a shared-memory stage
// (mbarrier completion, NSTAGE stages in flight), the K rows are re-rotated
// in shared memory by the consumer warps, and the unit goes back out with
// cp.async.bulk stores issued by a producer warp. V bytes never pass
// through registers. Same byte mapping, block-0 skip, rotation math and
// deviation scores as the SIMT kernels in page_kernels.cu. Jobs come from a
// job table, or (chunk-level loads) are derived from one descriptor per
// chunk.
//
// Every wait is bounded: an mbarrier wait that exceeds its limit (200 ms
// unless the launch sets a shorter one) sets DEV_ERR_TIMEOUT, the producer
// drains the copies this CTA has in flight (with the 200 ms bound) and the
// CTA returns.
#include <map>
#include <mutex>

#include "bulk_common.cuh"
#include "device_common.cuh"
#include "internal.h"

namespace daric {
namespace {
using namespace dev;
using namespace bulk;

// Consumer warps of a CTA: BulkGeom::cwarps (at most kConsumerWarps, the
// SM's warps shared by its ctas_per_sm CTAs), plus one producer warp.
constexpr int kConsumerWarps = 16;
constexpr int kBulkThreads = kConsumerWarps * 32 + 32;  // largest CTA

constexpr int kMaxPagesPerUnit = 8;

struct StageMeta {  // written by the producer lane that prefetched the unit
  uint8_t* base;          // layer data
  const uint8_t* fac;     // the unit's factor block in the factor buffer (global)
  float* sout;            // score output of the unit's first token (SCORE)
  int64_t stg_off;        // job's store offset
  int64_t page_stride;
  int64_t prefix_stride;
  int64_t len;            // tokens of the chunk to rotate (rotating units)
  int64_t fkey;           // factor block (group, page range); -1: none
  int32_t layer;          // index into the launch's layer table
  int32_t rot;            // the unit's K rows are rotated
  int32_t pl0;            // first page (job-local) of the unit
  int32_t npg;            // pages in the unit
  int32_t skipmask;       // bit g: page g is not copied (block id 0 / out of range)
  int32_t nreg;           // regions (prefix entries) per page
  int32_t rbytes;         // bytes per region
  int32_t n_sel;          // pages of the job
  int32_t sn;             // tokens with a score to write
  int32_t fac_bytes;      // bytes of the factor block
  int32_t fbuf;           // shared-memory factor buffer holding the block
  int32_t pad;
  int32_t blk[kMaxPagesPerUnit];
};
static_assert(128 + kMaxStages * sizeof(StageMeta) <= kBulkHeader, "stage meta exceeds the header");

__device__ __forceinline__ int64_t find_group(const GroupDev* groups, int64_t n, int64_t unit) {
  int64_t lo = 0, hi = n - 1;
  while (lo < hi) {
    const int64_t mid = (lo + hi + 1) >> 1;
    if (__ldg(&groups[mid].unit_begin) <= unit) lo = mid; else hi = mid - 1;
  }
  return lo;
}

__device__ __forceinline__ float4 as_float4(uint4 w) {
  return make_float4(__uint_as_float(w.x), __uint_as_float(w.y), __uint_as_float(w.z), __uint_as_float(w.w));
}

// Rotates the K rows of the unit's pages held in shared memory (in place).
// A task is (page g, token slot sl, head group hq, 16-byte column c): it
// reads the token's factors for the column once (from the unit's factor
// block staged beside the pages, or from the factor buffer in L2) and
// rotates rows hq, hq + hs, ... of the token's R rows; hs head groups share
// a token so that a full unit's tasks cover the consumer threads.
// Consecutive lanes take consecutive columns. With scores, a token's
// deviation is summed over its rows in registers and over the P * hs lanes
// of its tasks by a shuffle tree; one lane stores it (0 for a token that is
// not rotated). When those lanes do not tile a warp, the per-task sums go
// through score_add into zeroed slots instead.
// FC: factor entries are 4 x bf16 (8 bytes) instead of 4 x fp32 (16 bytes).
template <class E, bool NEOX, bool SCORE, bool FC>
__device__ __forceinline__ void rotate_unit_smem(const LayerDev& L, uint8_t* stage, int pages_per_unit,
                                                 const StageMeta& st, const uint8_t* fac_unit, bool fac_staged,
                                                 int64_t len, float* tok_dev, int tid, int nthreads, bool cst) {
  constexpr int ES = FC ? 8 : 16;  // bytes per factor entry
  constexpr int NG = NEOX ? E::kPerVec / 2 : E::kPerVec / 4;  // factor entries per task
  // the unit's layer and stage fields, read once into registers: every
  // shared-memory store below is an asm statement with a memory clobber,
  // after which a field read through L or st would be loaded again
  const int P = L.pair_vecs;
  const int bs = L.page_size;
  const int R = L.nrows / bs;  // rows of one token
  const FastDiv pair_div = L.pair_div, tok_mod = L.tok_mod;
  const int row_bytes = L.row_bytes, rbytes = st.rbytes, skipmask = st.skipmask;
  // token-major rows (one run): row = sl * R + k; head-major (4-D): k * bs + sl
  const bool tok_major = (int)L.tok_div.d == R;
  const int sl_mul = tok_major ? R : 1, k_mul = tok_major ? 1 : bs;
  const int per_tok = L.half_rot / 2;  // factor entries of one token
  const int hi_off = NEOX ? (L.rot_vecs / 2) * 16 : 0;
  const int64_t tok_base = (int64_t)st.pl0 * bs;
  // plane-major stage: region pf of page g at (pf * pages_per_unit + g) * rbytes
  const uint32_t base = smem_addr(stage) + (uint32_t)(L.k_prefix * pages_per_unit) * (uint32_t)rbytes;
  const int base_tasks = st.npg * bs * P;
  int hs = 1;
  while (hs < R && R % (2 * hs) == 0 && base_tasks * hs < nthreads && (!SCORE || P * hs * 2 <= 32)) hs *= 2;
  const int hshift = __ffs(hs) - 1;
  const int ntask = base_tasks << hshift;
  const int G = P << hshift;                        // lanes of one token
  const bool tree = SCORE && G <= 32 && (G & (G - 1)) == 0;
  // warp-uniform trip count (the score reduction shuffles across the warp)
  for (int t = tid; t - (tid & 31) < ntask; t += nthreads) {
    float dv = 0.f;
    int slot = -1;    // unit token of this lane's task
    bool rot = false;
    if (t < ntask) {
      const int tc = (int)fdiv((uint32_t)t, pair_div);
      const int c = t - tc * P;
      const int hq = tc & (hs - 1);
      const int gs = tc >> hshift;  // unit token g * bs + sl
      const int g = (int)fdiv((uint32_t)gs, tok_mod);
      const int sl = gs - g * bs;
      slot = gs;
      rot = !((skipmask >> g) & 1) && tok_base + gs < len;
      if (rot) {
        float4 q[NG];
        const uint8_t* fq = fac_unit + (gs * per_tok + c) * ES;
        if (fac_staged) {
          const uint32_t fa = smem_addr(fq);
#pragma unroll
          for (int k = 0; k < NG; ++k) {
            const uint32_t ad = fa + (uint32_t)(k * P * ES);
            q[k] = FC ? widen_factors(lds64(ad)) : as_float4(lds128(ad));
          }
        } else {
          // factors in L2, contiguous per task: the task's NG entries start
          // at entry c * NG of the token (16-byte aligned: NG * ES is a
          // multiple of 16 for every element type)
          const uint8_t* tq = fac_unit + (gs * per_tok + c * NG) * ES;
          if constexpr (FC) {
#pragma unroll
            for (int k = 0; k < NG; k += 2) {
              const uint4 w = __ldg(reinterpret_cast<const uint4*>(tq + k * ES));
              q[k] = widen_factors(make_uint2(w.x, w.y));
              q[k + 1] = widen_factors(make_uint2(w.z, w.w));
            }
          } else {
#pragma unroll
            for (int k = 0; k < NG; ++k) q[k] = __ldg(reinterpret_cast<const float4*>(tq + k * ES));
          }
        }
        const uint32_t cb = base + (uint32_t)(g * rbytes + c * 16);
        // consumer stores: the rotated vectors go straight to the page's K
        // region in the paged cache
        uint8_t* gb = cst ? st.base + (int64_t)L.k_prefix * st.prefix_stride + (int64_t)st.blk[g] * st.page_stride +
                                c * 16
                          : nullptr;
#pragma unroll 2
        for (int k = hq; k < R; k += hs) {
          const int roff = (sl * sl_mul + k * k_mul) * row_bytes;
          const uint32_t ad = cb + (uint32_t)roff;
          uint4 lo = lds128(ad), hi;
          if (NEOX) hi = lds128(ad + hi_off);
          if (NEOX) rotate_neox_q<E, SCORE>(q, 1, lo, hi, dv);
          else rotate_gptj_q<E, SCORE>(q, 1, lo, dv);
          if (cst) {
            st_stream(gb + roff, lo);
            if (NEOX) st_stream(gb + roff + hi_off, hi);
          } else {
            sts128(ad, lo);
            if (NEOX) sts128(ad + hi_off, hi);
          }
        }
      }
    }
    if (SCORE) {
      if (tree) {
        for (int o = 1; o < G; o <<= 1) dv += __shfl_xor_sync(0xffffffffu, dv, o);
        if (slot >= 0 && ((tid & 31) & (G - 1)) == 0) tok_dev[slot] = dv;
      } else {
        score_add(tok_dev, rot ? slot : -1, dv);
      }
    }
  }
}

// Consumer-store mode: copies the unit's live regions from shared memory to
// the paged cache with 16-byte stores, except the K vectors the rotation
// stored itself (rotated columns of rows whose token is rotated). No
// consumer waits for another: what is copied here is never modified.
__device__ __forceinline__ void store_rest(const LayerDev* Lk, const StageMeta& st, const uint8_t* stage, int PU,
                                           int tid, int nthreads) {
  const int vecs = st.rbytes >> 4;
  int kpf = -1, kbytes = 0;
  bool kdone = false;  // the rotation stored the whole K region
  int64_t tok_base = 0;
  if (Lk != nullptr) {
    kpf = Lk->k_prefix;
    kbytes = Lk->nrows * Lk->row_bytes;
    tok_base = (int64_t)st.pl0 * Lk->page_size;
    kdone = Lk->tail_vecs == 0 && kbytes == st.rbytes && tok_base + (int64_t)st.npg * Lk->page_size <= st.len;
  }
  const uint32_t sbase = smem_addr(stage);
  for (int g = 0; g < st.npg; ++g) {
    if ((st.skipmask >> g) & 1) continue;
    for (int pf = 0; pf < st.nreg; ++pf) {
      const bool kreg = pf == kpf;
      if (kreg && kdone) continue;
      const uint32_t src = sbase + (uint32_t)((pf * PU + g) * st.rbytes);
      uint8_t* dst = st.base + (int64_t)pf * st.prefix_stride + (int64_t)st.blk[g] * st.page_stride;
      for (int v = tid; v < vecs; v += nthreads) {
        const int off = v << 4;
        if (kreg && off < kbytes) {
          const int row = off / Lk->row_bytes;
          const int col = (off - row * Lk->row_bytes) >> 4;
          if (col < Lk->rot_vecs && tok_base + (int64_t)g * Lk->page_size + row_slot(*Lk, row) < st.len) continue;
        }
        st_stream(dst + off, lds128(src + (uint32_t)off));
      }
    }
  }
}

// Warp-specialised pipeline. Warps 0..cwarps-1 rotate (in CG groups that
// take alternate units); the last warp is the producer. Its lanes prefetch
// the copy plans of one batch (up to 32 units) at a time; for the CTA's
// unit i the lane that prefetched it writes the stage metadata and arms
// full[i % NS], then the warp issues the unit's bulk loads (one region per
// lane). When no batch is left the producer arms one end marker (npg = -1)
// per consumer group instead of a unit. When every consumer warp has released the unit (empty[s]) the warp
// issues its bulk stores (one region per lane) and reuses the stage of the
// previous unit once those stores have read it.
// Units run page range by page range across the jobs of a group, so
// consecutive units share a factor block: the producer loads a block into a
// factor buffer (the other one of two, or the only one) only when the key
// changes (its bytes complete on the unit's full barrier; later units see it
// through their own, later, full waits), after the units that read that
// buffer's previous block have been released.
// Shared memory: [0,128) full/empty barriers | [128,kBulkHeader) stage meta |
// per-stage deviation slots | factor buffers | stages, plane-major
// (region pf of page g at (pf * pages_per_unit + g) * rbytes).
template <int KVT, bool NEOX, bool ROTATE, bool GATHER, bool SCORE, bool FC>
__global__ void __launch_bounds__(kBulkThreads, 1) bulk_pages_kernel(PageLaunch p, BulkGeom g) {
  using E = Elem<KVT>;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kMaxStages;
  StageMeta* meta = reinterpret_cast<StageMeta*>(smem + 128);
  float* devs = reinterpret_cast<float*>(smem + kBulkHeader);  // NS x dev_stride floats
  uint8_t* fbufs = smem + kBulkHeader + g.dev_bytes;
  uint8_t* stages = fbufs + (g.fac_off ? g.fac_nbuf * g.fac_buf : 0);
  const int NS = g.nstage;
  const int PU = g.pages_per_unit;
  const int dev_stride = g.dev_bytes / (4 * NS);
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int cwarps = (int)(blockDim.x >> 5) - 1;  // consumer warps of this CTA
  const bool producer = warp == cwarps;
  // consumer groups: group c rotates units c, c + CG, c + 2 CG, ... so CG
  // units are in the consumers' hands at once. NS is a multiple of CG, so a
  // stage is always rotated by the same group, which waits for its phases in
  // order (a parity wait must never run two phases ahead).
  const int CG = (g.cgroups > 1 && g.nstage % g.cgroups == 0) ? g.cgroups : 1;
  const int gwarps = cwarps / CG;

  // Region pf of job-local page pl (block blk): store side at
  // stg_off + (pf * n_sel + pl) * rbytes, layer side at
  // base + pf * prefix_stride + blk * page_stride.

  if (tid == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], gwarps);
    }
    mbar_init_fence();
  }
  if (SCORE)
    for (int q = tid; q < NS * dev_stride; q += blockDim.x) devs[q] = 0.f;
  __syncthreads();

  if (producer) {
    const unsigned FULL = 0xffffffffu;
    // the CTA's units: batch after batch, the current one is local units
    // [bbeg, bend) = global units [u0, u0 + bend - bbeg); n = the CTA's unit
    // count once a claim came back empty (-1 before)
    int64_t bbeg = 0, bend = 0, u0 = 0, n = -1;
    int nclaims = 0;
    StageMeta mine{};  // this lane's unit of the current batch
    // next batch: the first by CTA index, then from the work counter, about
    // half the units left per CTA (1 to 32); returns its size (0: none left)
    auto claim = [&]() -> int {  // all lanes
      const uint64_t total = (uint64_t)p.total_units;
      uint64_t start = 0;
      int m = 0;
      if (lane == 0) {
        uint64_t want = (uint64_t)p.first_batch;
        if (nclaims == 0) {
          start = (uint64_t)blockIdx.x * want;
        } else {
          const uint64_t cur = *reinterpret_cast<volatile unsigned long long*>(p.work);
          const uint64_t left = total > cur ? total - cur : 0;
          want = left / (2 * (uint64_t)gridDim.x);
          want = want < 1 ? 1 : (want > 32 ? 32 : want);
          start = atomicAdd(p.work, (unsigned long long)want);
        }
        m = start < total ? (int)(total - start < want ? total - start : want) : 0;
      }
      ++nclaims;
      u0 = (int64_t)__shfl_sync(FULL, (unsigned long long)start, 0);
      return __shfl_sync(FULL, m, 0);
    };
    auto prefetch = [&](int m) {  // all lanes: lane < m prefetches unit u0 + lane
      int64_t gi = find_group(p.groups, p.num_groups, u0);
      mine.npg = 0;
      mine.skipmask = 0;
      mine.sn = 0;
      mine.rot = 0;
      mine.fac = nullptr;
      mine.fac_bytes = 0;
      mine.fkey = -1;
      mine.len = 0;
      if (lane < m) {
        const int64_t u = u0 + lane;
        while (gi + 1 < p.num_groups && p.groups[gi + 1].unit_begin <= u) ++gi;
        const GroupDev G = p.groups[gi];
        const int64_t local = u - G.unit_begin;
        const int r = (int)(local / G.cnt);
        const int jl = (int)(local - (int64_t)r * G.cnt);
        JobDev jd;
        if (p.jobs != nullptr) {
          jd = p.jobs[G.j0 + jl];
        } else {  // chunk-level load: the job of (chunk, layer slot j0 + jl)
          const LayerDev& Lj = p.layers[G.j0 + jl];
          jd.stg_off = G.stg_off + (int64_t)G.n_sel * Lj.store_page_off;
          jd.idx_off = G.idx_off;
          jd.fac_tok = G.fac_tok;
          jd.n_sel = G.n_sel;
          jd.layer = G.j0 + jl;
          jd.meta = G.meta;
          jd.score_row = Lj.score_row;
        }
        const LayerDev& L = p.layers[jd.layer];
        const int pl0 = r * PU;
        const int npg = min(PU, jd.n_sel - pl0);
        mine.base = L.base;
        mine.stg_off = jd.stg_off;
        mine.page_stride = L.page_stride;
        mine.prefix_stride = L.prefix_stride;
        mine.layer = jd.layer;
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
        if (ROTATE && jd.meta >= 0) {
          const MetaDev m = p.metas[jd.meta];
          if (L.has_rot && m.rotate) {
            const int64_t tb = (int64_t)token_factor_bytes(L.half_rot, FC);
            mine.rot = 1;
            mine.len = m.len;
            mine.fac = reinterpret_cast<const uint8_t*>(p.fac) + (jd.fac_tok + (int64_t)pl0 * L.page_size) * tb;
            mine.fac_bytes = (int32_t)((size_t)npg * page_factor_bytes(L.page_size, L.half_rot, FC));
            mine.fkey = (gi << 24) | r;
          }
          if (SCORE && jd.score_row >= 0) {
            const int64_t tok0 = (int64_t)pl0 * L.page_size;
            const int64_t left = m.len - tok0;
            const int64_t cap = (int64_t)npg * L.page_size;
            mine.sn = (int32_t)(left < 0 ? 0 : (left < cap ? left : cap));
            mine.sout = p.scores + (int64_t)jd.score_row * p.score_ld + m.score_col + tok0;
          }
        }
      }
    };
    // factor buffers: the block each holds and the last unit that reads it
    // (scalar pairs: no local-memory arrays)
    long long fkey0 = -1, fkey1 = -1;
    int64_t last0 = -1, last1 = -1;
    int cur = 1;
    int64_t waited = -1;  // empty[] of every unit <= waited has completed
    // loads of unit i into stage i % NS (warp-synchronous: every lane calls);
    // false when a wait timed out
    auto issue = [&](int64_t i) -> bool {
      if (g.unarmed && i == 0) return true;  // test only: nothing arms unit 0
      if (n < 0 && i >= bend) {
        const int m = claim();
        if (m == 0) {
          n = i;
        } else {
          bbeg = i;
          bend = i + m;
          prefetch(m);
        }
      }
      const int s = (int)(i % NS);
      if (n >= 0 && i >= n) {  // end marker of consumer group (i - n)
        if (lane == 0) {
          meta[s].npg = -1;
          mbar_arrive(&full[s]);
        }
        __syncwarp();
        return true;
      }
      const int k = (int)(i - bbeg);
      const long long fkey = __shfl_sync(FULL, (long long)mine.fkey, k);
      const int npg = __shfl_sync(FULL, mine.npg, k);
      const int live = npg - __popc(__shfl_sync(FULL, mine.skipmask, k));
      int fbuf = 0;
      uint32_t fload = 0;
      if (g.fac_off && fkey >= 0 && live > 0) {
        if (fkey == (cur ? fkey1 : fkey0)) {
          fbuf = cur;
        } else {
          const int f = g.fac_nbuf == 2 ? cur ^ 1 : 0;
          const int64_t x = f ? last1 : last0;
          // units up to x may still read the buffer's old block: wait for
          // each of them (consumer groups release units out of order)
          for (int64_t y = waited + 1; y <= x; ++y) {
            const bool ok = mbar_wait(&empty[y % NS], (uint32_t)((y / NS) & 1), (uint64_t)g.wait_ns);
            if (__any_sync(FULL, !ok)) return false;
          }
          if (f) fkey1 = fkey; else fkey0 = fkey;
          cur = f;
          fbuf = f;
          fload = (uint32_t)__shfl_sync(FULL, mine.fac_bytes, k);
        }
        if (fbuf) last1 = i; else last0 = i;
      }
      if (lane == k) {
        mine.fbuf = fbuf;
        meta[s] = mine;
        // the arrival (with the byte count) precedes every copy; scatter
        // loads whole planes (skipped pages included), gather live regions
        const int pages = GATHER ? live : mine.npg;
        if (live == 0) mbar_arrive(&full[s]);
        else mbar_arrive_expect_tx(&full[s], (uint32_t)(pages * mine.nreg * mine.rbytes) + fload);
      }
      if (live == 0) return true;
      __syncwarp();
      // operands from the stage metadata (shared memory), read once before
      // the copies (which clobber memory)
      const StageMeta& sm = meta[s];
      const int nreg = sm.nreg, rbytes = sm.rbytes, pl0 = sm.pl0, skipm = sm.skipmask, nsel = sm.n_sel;
      const int npgs = sm.npg;
      // scatter: the unit's pages of a plane are contiguous in the store, one
      // copy per plane; gather: one copy per live region
      const int nops = GATHER ? npgs * nreg : nreg;
      uint8_t* const lbase = sm.base;
      const int64_t stg_off = sm.stg_off, pstride = sm.page_stride, fstride = sm.prefix_stride;
      const uint8_t* const fsrc = sm.fac;
      uint8_t* buf = stages + (size_t)s * g.stage_bytes;
      for (int o = lane; o < nops + (fload ? 1 : 0); o += 32) {
        uint8_t* dst;
        const uint8_t* src;
        uint32_t bytes;
        if (o == nops) {
          dst = fbufs + (size_t)fbuf * g.fac_buf;
          src = fsrc;
          bytes = fload;
        } else if (!GATHER) {
          dst = buf + (size_t)o * PU * rbytes;
          src = p.store + stg_off + ((int64_t)o * nsel + pl0) * rbytes;
          bytes = (uint32_t)(npgs * rbytes);
        } else {
          const int q = o / nreg, pf = o - q * nreg;
          if ((skipm >> q) & 1) continue;
          dst = buf + ((size_t)pf * PU + q) * rbytes;
          src = lbase + (int64_t)pf * fstride + (int64_t)sm.blk[q] * pstride;
          bytes = (uint32_t)rbytes;
        }
        bulk_load(dst, src, bytes, &full[s]);
      }
      return true;
    };
    bool ok = true;
    int64_t issued = 0;  // units whose loads are armed
    // with bulk stores a stage is refilled once the stores of its unit have
    // read it (NS - 1 units in flight); with consumer stores as soon as the
    // consumers release it (NS in flight)
    const bool cst = !GATHER && g.cstore;
    const int inflight = cst ? NS : NS - 1;
    // units and end markers still to arm
    auto more = [&]() { return n < 0 || issued < n + CG; };
    while (issued < inflight && more()) {
      if (!issue(issued)) {
        ok = false;
        break;
      }
      ++issued;
    }
    bool prev_stored = false;  // unit i-1 has a pending store group (every lane)
    int64_t i = 0;
    for (; ok && (n < 0 || i < n); ++i) {
      const int s = (int)(i % NS);
      const bool got = mbar_wait(&empty[s], (uint32_t)((i / NS) & 1), (uint64_t)g.wait_ns);
      if (__any_sync(FULL, !got)) {
        ok = false;
        break;
      }
      waited = i;
      // operands from the stage metadata, read once before the copies
      const StageMeta& sm = meta[s];
      const int nreg = sm.nreg, rbytes = sm.rbytes, pl0 = sm.pl0, skipm = sm.skipmask, nsel = sm.n_sel;
      const int nops = sm.npg * nreg;
      uint8_t* const lbase = sm.base;
      const int64_t stg_off = sm.stg_off, pstride = sm.page_stride, fstride = sm.prefix_stride;
      const int sn = sm.sn;
      float* const sout = sm.sout;
      const bool stored = !cst && sm.npg > __popc(skipm);
      if (stored) {
        // stores spread over the lanes; every lane commits a bulk group per
        // stored unit (empty for lanes without a region), so the groups of
        // all lanes stay in step for the waits below
        uint8_t* buf = stages + (size_t)s * g.stage_bytes;
        // gather without skipped pages: one store per plane (contiguous in
        // the store); else one per live region
        const bool whole = GATHER && skipm == 0;
        const int sops = whole ? nreg : nops;
        for (int o = lane; o < sops; o += 32) {
          uint8_t* dst;
          const uint8_t* src;
          uint32_t bytes;
          if (whole) {
            dst = p.store_mut + stg_off + ((int64_t)o * nsel + pl0) * rbytes;
            src = buf + (size_t)o * PU * rbytes;
            bytes = (uint32_t)(sm.npg * rbytes);
          } else {
            const int q = o / nreg, pf = o - q * nreg;
            if ((skipm >> q) & 1) continue;
            dst = GATHER ? p.store_mut + stg_off + ((int64_t)pf * nsel + pl0 + q) * rbytes
                         : lbase + (int64_t)pf * fstride + (int64_t)sm.blk[q] * pstride;
            src = buf + ((size_t)pf * PU + q) * rbytes;
            bytes = (uint32_t)rbytes;
          }
          bulk_store(dst, src, bytes);
        }
        bulk_commit();
      }
      if (SCORE) {
        float* dv = devs + s * dev_stride;
        for (int q = lane; q < sn; q += 32) sout[q] = dv[q];
        __syncwarp();
        for (int q = lane; q < dev_stride; q += 32) dv[q] = 0.f;
      }
      __syncwarp();
      // the next load goes into the stage of unit i-1 (bulk stores: they must
      // have read it; unit i's group, committed last, may still be pending)
      // or of unit i (consumer stores)
      if (more()) {
        if (prev_stored) {
          if (stored) bulk_wait_read<1>(); else bulk_wait_read<0>();
        }
        __syncwarp();
        if (issue(issued)) ++issued;
        else ok = false;
      }
      prev_stored = stored;
      __syncwarp();
    }
    // end markers the loop did not reach (consumer groups beyond the units in
    // flight): they write only stage metadata, and every unit that used
    // their stages has been released
    while (ok && more()) {
      issue(issued);
      ++issued;
    }
    if (!ok && lane == 0) {
      atomicOr(p.err, DEV_ERR_TIMEOUT);
      // drain the loads that may still be in flight into this CTA's stages
      // (units not yet released by the consumers)
      for (int64_t k = i; k < issued; ++k)
        if (!(g.unarmed && k == 0)) mbar_wait(&full[k % NS], (uint32_t)((k / NS) & 1));
    }
    bulk_wait_all();
    return;
  }

  // consumers
  const int grp = warp / gwarps;
  const int gtid = tid - grp * gwarps * 32;
  const bool cst = !GATHER && g.cstore;
  for (int64_t i = grp;; i += CG) {
    const int s = (int)(i % NS);
    if (!mbar_wait(&full[s], (uint32_t)((i / NS) & 1), (uint64_t)g.wait_ns)) {
      atomicOr(p.err, DEV_ERR_TIMEOUT);
      break;
    }
    const StageMeta& st = meta[s];
    if (st.npg < 0) break;  // end marker
    const bool live = st.npg > __popc(st.skipmask);
    uint8_t* stage = stages + (size_t)s * g.stage_bytes;
    const LayerDev* Lk = nullptr;
    if (ROTATE && st.rot && live) {
      Lk = &p.layers[st.layer];
      const bool staged = g.fac_off > 0;
      const uint8_t* fac_unit = staged ? fbufs + (size_t)st.fbuf * g.fac_buf : st.fac;
      rotate_unit_smem<E, NEOX, SCORE, FC>(*Lk, stage, PU, st, fac_unit, staged, st.len,
                                           devs + s * dev_stride, gtid, gwarps * 32, cst);
      if (!cst) fence_proxy_async();
    }
    if (cst && live) store_rest(Lk, st, stage, PU, gtid, gwarps * 32);
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
  const int grid = bulk_grid(p.total_units, sm_count, g.ctas_per_sm);
  if (p.work == nullptr || p.first_batch != bulk_first_batch(p.total_units, grid))
    throw Error(DARIC_ERR_INVALID, "internal: bulk launch without its work counter");
  const int threads = (g.cwarps + 1) * 32;
  kernel<<<grid, threads, smem, s>>>(p, g);
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
