// Internal definitions shared by the host side (capi.cpp) and the kernels.
//
// Device descriptors are uploaded once per call as one contiguous blob
// (layer table, job or chunk table, factor runs, unit groups) through a
// pinned ring (capi.cpp, class Upload); kernels read them through
// read-only-cached loads.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <stdexcept>
#include <string>

#include "../../include/daric_b200.h"

namespace daric {

// ---------------------------------------------------------------- errors --
// Errors are thrown inside the library and turned into status codes at the C
// boundary (capi.cpp). Messages follow the reference's TORCH_CHECK texts where
// a reference check exists.
struct Error : std::runtime_error {
  int code;
  Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

#define DARIC_CHECK(cond, msg)                                          \
  do {                                                                  \
    if (!(cond)) throw ::daric::Error(DARIC_ERR_INVALID, (msg));        \
  } while (0)

#define DARIC_CUDA(call)                                                         \
  do {                                                                           \
    cudaError_t e_ = (call);                                                     \
    if (e_ != cudaSuccess)                                                       \
      throw ::daric::Error(DARIC_ERR_CUDA, std::string("CUDA error at ") +       \
                                               __FILE__ + ":" +                  \
                                               std::to_string(__LINE__) + " - " + \
                                               cudaGetErrorString(e_));          \
  } while (0)

// ------------------------------------------------------- fast division --
// Division by a runtime-invariant positive divisor with one multiply-high
// (Granlund & Montgomery, "Division by Invariant Integers using
// Multiplication", PLDI 1994, round-up method). Valid for 0 <= n < 2^31.
struct FastDiv {
  uint32_t d;
  uint32_t mul;
  uint32_t shift;
};

inline FastDiv make_fastdiv(uint32_t d) {
  FastDiv f{d, 0, 0};
  uint32_t s = 0;
  while ((1ull << s) < d) ++s;
  f.shift = s;
  // mul = floor(2^32 * (2^s - d) / d) + 1
  f.mul = (uint32_t)(((1ull << 32) * ((1ull << s) - d)) / d + 1);
  return f;
}

__host__ __device__ __forceinline__ uint32_t fdiv(uint32_t n, FastDiv f) {
#ifdef __CUDA_ARCH__
  uint32_t hi = __umulhi(n, f.mul);
#else
  uint32_t hi = (uint32_t)(((uint64_t)n * f.mul) >> 32);
#endif
  return (uint32_t)(((uint64_t)hi + n) >> f.shift);
}

// ------------------------------------------------------------ layouts ----
// One registered KV layer as the kernels see it.
struct LayerDev {
  uint8_t* base;          // layer data
  int64_t page_stride;    // bytes between pages (blocks)
  int64_t prefix_stride;  // bytes between prefix entries (K/V planes)
  int64_t suffix;         // bytes of one (prefix, page) region (dense span)
  int32_t prefix_size;
  int32_t num_pages;
  // rotation geometry (valid when has_rot)
  int32_t has_rot;
  int32_t k_prefix;       // prefix index whose region holds the K rows
  int32_t nrows;          // K rows per page region
  int32_t row_bytes;      // distance between consecutive K rows
  int32_t row_vecs;       // row_bytes / 16
  int32_t rot_vecs;       // 16-byte vectors of a row that are rotated
  int32_t pair_vecs;      // rotation tasks per row (NeoX: rot_vecs/2, GPT-J: rot_vecs)
  int32_t page_size;      // tokens per page
  FastDiv pair_div;       // task -> row
  FastDiv tok_div;        // row -> token (before the modulo)
  FastDiv tok_mod;        // modulo page_size
  FastDiv tail_div;       // row_vecs - rot_vecs (non-rotated vectors per row)
  FastDiv page_div;       // nrows * pair_vecs (rotation tasks per page)
  int32_t tail_vecs;      // row_vecs - rot_vecs
  int32_t half_rot;       // rotary_dim / 2 (elements)
  const uint8_t* table;   // cos_sin_cache
  int64_t table_row;      // bytes per table row
  int64_t max_pos;        // rows of the table
  // chunk-level loads (daric_copier_load_chunks)
  int64_t store_page_off; // bytes per chunk page of the layers before this one in the store
  int32_t score_row;      // score row of the layer (-1 = no scores)
  int32_t pad2;
};

struct JobDev {
  int64_t stg_off;     // byte offset into the store buffer
  int64_t idx_off;     // first entry of this job's block ids in indices_flat
  int64_t unit_begin;  // first unit (page) of this job within the launch
  int64_t fac_tok;     // factor-buffer token of the chunk's token 0 (its table)
  int32_t n_sel;       // pages of this job
  int32_t layer;       // index into the launch's LayerDev table
  int32_t meta;        // chunk index (-1 = none)
  int32_t score_row;   // score row (-1 = no scores)
};

struct MetaDev {
  int64_t pos_a;      // FLEXIBLE: old start; DELTA: delta
  int64_t pos_b;      // FLEXIBLE: new start
  int64_t len;        // tokens to rotate
  int64_t score_col;  // first score column of the chunk
  int32_t rotate;     // 0 = copy only (old == new, or mode NONE)
  int32_t pad;
};

struct PageLaunch {
  const LayerDev* layers;
  const JobDev* jobs;
  const MetaDev* metas;
  const uint8_t* store;      // store (staging) base
  uint8_t* store_mut;        // same, writable (gather)
  const int32_t* indices;    // indices_flat
  int64_t indices_numel;
  int64_t num_jobs;
  int64_t total_units;
  int32_t mode;              // DARIC_ROPE_*
  float* scores;
  int64_t score_ld;
  int* err;                  // device error word
  const float4* fac;         // rotary factors (factor pre-pass output)
  const struct GroupDev* groups;  // bulk pipeline unit order
  int64_t num_groups;
  // bulk pipeline batches: CTA b's first batch is units [b * first_batch,
  // (b + 1) * first_batch); later ones are claimed from *work, which starts
  // at grid * first_batch (bulk_first_batch)
  unsigned long long* work;
  int64_t first_batch;
};

// Grid of a bulk-pipeline launch and its first batch per CTA: about half the
// units per CTA, at most 32 (the producer warp's prefetch width).
inline int bulk_grid(int64_t units, int sm_count, int ctas_per_sm) {
  const int64_t ctas = (int64_t)sm_count * ctas_per_sm;
  return (int)(units < ctas ? units : ctas);
}
inline int64_t bulk_first_batch(int64_t units, int grid) {
  const int64_t f = grid > 0 ? units / (2 * (int64_t)grid) : 1;
  return f < 1 ? 1 : (f > 32 ? 32 : f);
}

// Bulk pipeline unit order: consecutive jobs of one chunk with the same page
// count and factor run form a group; its units go page range by page range
// and, within a range, job by job (unit = range r of job j0 + l at
// unit_begin + r * cnt + l), so consecutive units share their factor block.
// Chunk-level loads (PageLaunch::jobs == nullptr): a group is one chunk and
// its jobs are the launch's layers [j0, j0 + cnt) (layer-table slots); job
// (chunk, layer l) reads the store at stg_off + n_sel * store_page_off(l)
// and the chunk's block ids at idx_off, for every layer.
struct GroupDev {
  int64_t unit_begin;
  int32_t j0, cnt;     // jobs [j0, j0 + cnt)
  int32_t n_sel;       // pages of each job
  int32_t nranges;     // ceil(n_sel / pages_per_unit)
  int64_t stg_off;     // chunk-level: store offset of the chunk
  int64_t idx_off;     // chunk-level: first block id of the chunk
  int64_t fac_tok;     // chunk-level: factor-buffer token of the chunk's token 0
  int32_t meta;        // chunk-level: chunk index
  int32_t pad;
};

// In-place rotation segments.
struct SegDev {
  int64_t blk_off;     // offset of the request's block table
  int64_t tok_start;   // first token position
  int64_t tok_len;     // tokens
  int64_t pos_a, pos_b;
  int64_t unit_begin;  // first unit (page-slice) of the segment
  int64_t fac_tok;     // factor-buffer token of the segment's token 0
  int32_t first_page;  // tok_start / page_size
  int32_t num_units;   // units of the segment (SIMT: pages touched; bulk: page ranges)
  int32_t num_pages;   // pages touched
  int32_t pad;
};

struct InplaceLaunch {
  const LayerDev* layers;
  int64_t num_layers;
  const SegDev* segs;
  int64_t num_segs;
  int64_t units_per_layer;   // sum over segments of pages touched
  const int32_t* block_table;
  int64_t block_table_numel;
  int32_t mode;
  int* err;
  const float4* fac;
};

// Copy-engine pipeline of the in-place rotation: NSTAGE stages of up to
// pages_per_unit pages' K regions (kbytes each, rows at their natural
// offsets), after the header.
struct InplaceGeom {
  int32_t nstage;
  int32_t stage_bytes;
  int32_t pages_per_unit;
  int32_t kbytes;       // largest K region of a page in the launch
  int32_t ctas_per_sm;
  int32_t cwarps;       // consumer warps per CTA (plus one producer warp)
  int32_t tab_dtype;    // rotary table dtype (factors are read from the table)
  int32_t wait_ns;      // limit of a pipeline wait (ns); the drain after a time-out keeps 200 ms
  int32_t unarmed;      // test only: each CTA's first unit is never armed, so its waits run out
  int32_t pad;
};

// Factor pre-pass: one run of tokens [0, len) of a chunk (or segment) with
// one rotary table, written at factor-buffer token out_tok.
struct FacJobDev {
  const uint8_t* table;
  int64_t table_row;   // bytes per table row
  int64_t pos_a, pos_b;
  int64_t len;
  int64_t out_tok;
  int64_t item_begin;  // first float4 of this run within the launch
  int32_t half_rot;
  int32_t P;           // rotation tasks per row (half_rot / fpv)
};

struct FactorLaunch {
  const FacJobDev* jobs;
  int64_t num_jobs;
  int64_t total_items;  // entry count (4 factors per entry)
  void* out;
  int32_t mode;
  int32_t fpv;          // factors per rotation task
  int32_t compact;      // entries are 4 x bf16 (8 bytes) instead of 4 x fp32
  int32_t contig;       // a task's entries are contiguous (c * NG + g) instead of strided (g * P + c)
};

// Factor bytes of one token (half_rot (cos, sin) pairs): fp32, or bf16 when
// the table is bf16 (its factors are bf16 values, so the narrow form is exact).
__host__ __device__ inline size_t token_factor_bytes(int half_rot, bool compact) {
  return (size_t)half_rot * (compact ? 4 : 8);
}
__host__ __device__ inline size_t page_factor_bytes(int page_size, int half_rot, bool compact = false) {
  return (size_t)page_size * token_factor_bytes(half_rot, compact);
}

struct SelSegDev {
  int64_t col_off, len, pos0, k, blk_off, out_off;
};

struct SelectLaunch {
  const float* scores;
  int64_t num_layers, score_ld, num_segs;
  const SelSegDev* segs;
  int32_t mode;
  float threshold;
  const int32_t* block_table;
  int64_t block_table_numel;
  int64_t block_size;
  int32_t* out_idx;
  int64_t* out_slot;
  int32_t* out_count;
  int64_t out_ld;
  int* err;
  int32_t cluster;    // CTAs per (segment, layer), a thread-block cluster
  int32_t smem_keys;  // keys of a slice staged in shared memory (capacity)
};

struct RangeDev {
  int64_t start, end, blk_off, out_begin;
};

struct RangeLaunch {
  const RangeDev* ranges;
  int64_t num_ranges, total;
  const int32_t* block_table;
  int64_t block_table_numel;
  int64_t block_size;
  int32_t* out_idx;
  int64_t* out_slot;
  int* err;
};

// Device error bits (OR-ed into the device error word).
enum : int {
  DEV_ERR_BLOCK_RANGE = 1,   // a block id outside [0, num_pages)
  DEV_ERR_TABLE_RANGE = 2,   // a rotary position outside [0, max_position)
  DEV_ERR_INDEX_RANGE = 4,   // a block-table index outside the given table
  DEV_ERR_TIMEOUT = 8,       // a bounded wait in a pipelined kernel gave up
};

// Geometry of the bulk-copy pipeline: NSTAGE shared-memory stages of
// stage_bytes each, after the header, a dev_bytes region of per-slot
// deviations and the factor buffers. A unit is up to pages_per_unit
// consecutive pages of one job, plane-major in its stage: region pf of page g
// at (pf * pages_per_unit + g) * rbytes. page_data = largest page of the
// launch (prefix_size x region bytes).
struct BulkGeom {
  int32_t nstage;
  int32_t stage_bytes;
  int32_t pages_per_unit;
  int32_t page_data;
  int32_t dev_bytes;
  int32_t fac_off;      // >0: offset of the factor buffers (one unit's factors each); 0: read from L2
  int32_t fac_buf;      // bytes of one factor buffer
  int32_t fac_nbuf;     // factor buffers: 2 (load the next block while the last is read) or 1
  int32_t fac_compact;  // factors stored as bf16 pairs (bf16 tables) instead of fp32
  int32_t ctas_per_sm;  // 1, 2 or 4 CTAs (each with its own producer warp) per SM
  int32_t cgroups;      // consumer-warp groups (1, 2 or 4) taking alternate units
  int32_t cwarps;       // consumer warps per CTA (plus one producer warp)
  int32_t cstore;       // scatter: consumer warps write the paged cache (no bulk stores)
  int32_t wait_ns;      // limit of a pipeline wait (ns); the drain after a time-out keeps 200 ms
  int32_t unarmed;      // test only: each CTA's first unit is never armed, so its waits run out
  int32_t pad;
};

// Limit of one bounded wait in the pipelined kernels (ns). DARIC_WAIT_NS
// sets a shorter limit for the waits of a launch (tests make a wait run out
// with it); the drain of in-flight copies after a time-out keeps this one.
constexpr int32_t kDefaultWaitNs = 200 * 1000 * 1000;

// Bytes of the bulk pipeline's shared-memory header (barriers + stage meta).
constexpr int kBulkHeader = 2048;

// [header | deviation slots | factor buffers | stages]
inline size_t bulk_smem_bytes(const BulkGeom& g) {
  return kBulkHeader + (size_t)g.dev_bytes + (g.fac_off ? (size_t)g.fac_nbuf * g.fac_buf : 0) +
         (size_t)g.nstage * g.stage_bytes;
}

// ------------------------------------------------------------ launchers --
// Kernel signature key for the rotating scatter.
struct RotKey {
  int kv_dtype, tab_dtype, neox;
};

void launch_plain_pages(const PageLaunch& p, bool gather, bool vec16, int sm_count, cudaStream_t s);
void launch_factors(const FactorLaunch& p, int tab_dtype, int sm_count, cudaStream_t s);
void launch_rotate_scatter(const PageLaunch& p, RotKey key, int sm_count, cudaStream_t s);
void launch_rotate_inplace(const InplaceLaunch& p, RotKey key, int sm_count, cudaStream_t s);
// Units of InplaceLaunch are page ranges of g.pages_per_unit pages.
void launch_bulk_inplace(const InplaceLaunch& p, const InplaceGeom& g, RotKey key, int sm_count, cudaStream_t s);
void launch_bulk_plain(const PageLaunch& p, const BulkGeom& g, bool gather, int sm_count, cudaStream_t s);
void launch_bulk_rotate(const PageLaunch& p, const BulkGeom& g, RotKey key, int sm_count, cudaStream_t s);
// max_len: longest segment of the call (picks the cluster size).
void launch_score_select(SelectLaunch p, int64_t max_len, int sm_count, cudaStream_t s);
void launch_ranges_to_slots(const RangeLaunch& p, cudaStream_t s);

int* device_error_word(int device);  // per-device error word (lazily created)

// Last-error hooks of the C boundary (capi.cpp) for entry points defined in
// other translation units.
void record_error(int code, const char* msg);
void clear_error();

}  // namespace daric
