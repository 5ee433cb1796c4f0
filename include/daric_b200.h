/*
 * daric_b200.h — C ABI of the B200-native reused-KV hot path.
 *
 * Every entry point takes plain pointers and sizes (no torch types) and
 * returns an int status: DARIC_OK (0) on success, otherwise an error code
 * whose message is available from daric_last_error() on the same thread.
 * Device pointers must live on the device named by the call; all GPU work is
 * enqueued on the given cudaStream_t (passed as void*; NULL = legacy default
 * stream) and nothing blocks the host except where a comment says so.
 *
 * The reference's native module is the pybind11 module `daric.cache_ops`
 * (csrc/cache_ops/bindings.cpp:7-31, typed in daric/cache_ops.pyi:6-53).
 * The Python package `daric_b200` binds this header through ctypes and
 * exposes the reference's names and argument meanings on top of it.
 */
#ifndef DARIC_B200_H
#define DARIC_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define DARIC_API __attribute__((visibility("default")))
#else
#define DARIC_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes -------------------------------------------------------- */
#define DARIC_OK 0
#define DARIC_ERR_INVALID 1 /* argument check failed (reference: TORCH_CHECK) */
#define DARIC_ERR_CUDA 2    /* CUDA runtime error (reference: CUDA_CHECK)    */
#define DARIC_ERR_STATE 3   /* object not ready, e.g. store not registered    */
#define DARIC_ERR_DEVICE 4  /* device-side check tripped (bad block id, ...)  */

/* ---- element type codes -------------------------------------------------- */
#define DARIC_DTYPE_F32 0
#define DARIC_DTYPE_F16 1
#define DARIC_DTYPE_BF16 2
#define DARIC_DTYPE_FP8_E4M3 3 /* uint8 storage viewed as e4m3 (adapter.py:370-371) */

/* ---- rotation modes ------------------------------------------------------ */
#define DARIC_ROPE_NONE 0     /* plain scatter, K untouched                         */
#define DARIC_ROPE_FLEXIBLE 1 /* rotate by new-old: C=n_c*o_c+n_s*o_s, S=n_s*o_c-n_c*o_s
                                 from table rows (old+t, new+t), one rounding per op in
                                 the table dtype (adapter.py:196-295)                */
#define DARIC_ROPE_DELTA 2    /* rotate by a fixed delta: C,S = table row delta
                                 (strict PIC, adapter.py:118-194)                    */

/* ---- selection modes ----------------------------------------------------- */
#define DARIC_SELECT_TOPK 0      /* k highest scores; ties -> lower token index   */
#define DARIC_SELECT_THRESHOLD 1 /* every token whose score >= threshold          */

/* Last error message of the calling thread ("" if none). Valid until the next
 * call into this library from the same thread. */
DARIC_API const char* daric_last_error(void);

/* Library ABI version (major*100 + minor). */
DARIC_API int daric_version(void);

/* Number of streaming multiprocessors of `device` (cached). */
DARIC_API int daric_device_sm_count(int device, int* out_sm_count);

/* Reads and clears the device-side error bits of `device`: 1 = a block id
 * outside [0, num_pages) was skipped, 2 = a rotary position outside the table
 * was skipped, 4 = a block-table index outside the given table was skipped,
 * 8 = a bounded wait inside a pipelined kernel gave up (its unit was dropped).
 * The kernels never fault on these; they skip the access and set the bit.
 * Synchronous (waits for the device's work to finish). */
DARIC_API int daric_device_errors(int device, int* out_bits);

/* ======================================================================== */
/* CacheCopier — replaces class CacheCopier (cache_ops.h:91-126,            */
/* copier.cpp:7-111, bindings.cpp:11-16).                                   */
/* ======================================================================== */
typedef struct daric_copier daric_copier;

/* Replaces `CacheCopier()` (bindings.cpp:12). */
DARIC_API int daric_copier_create(daric_copier** out);
/* Releases the handle. Pending GPU work that uses registered memory must be
 * finished by the caller first (the reference relies on tensor refcounts). */
DARIC_API void daric_copier_destroy(daric_copier* copier);

/* Replaces `CacheCopier.register_layer(name, tensor, is_page_first)`
 * (copier.cpp:7-11). The tensor is described by its data pointer, device,
 * sizes/strides (in elements) and element size; the page-copy shape is
 * derived as in get_page_copy_shape (helpers.cu:94-148) and rejected with
 * DARIC_ERR_INVALID on the same conditions. Re-registering a name replaces
 * the previous entry (insert_or_assign, copier.cpp:10). */
DARIC_API int daric_copier_register_layer(daric_copier* copier, const char* name, void* data, int device,
                                int ndim, const int64_t* sizes, const int64_t* strides,
                                int64_t element_size, int is_page_first);

/* Replaces `CacheCopier.register_store(buffer)` (copier.cpp:13-25): a 1-D
 * contiguous uint8 device buffer of `nbytes` bytes. */
DARIC_API int daric_copier_register_store(daric_copier* copier, void* data, int64_t nbytes, int device);

/* Replaces `CacheCopier.gather_pages(...)` (copier.cpp:41-76,
 * kernels.cu:127-217): paged KV -> store. Job i copies the pages
 * indices_flat[indices_offsets[i] .. indices_offsets[i+1]) of layer
 * layer_names[i] into store[offsets[i] .. offsets[i]+byte_sizes[i]),
 * byte_sizes[i] must equal prefix*n_sel*suffix (kernels.cu:151-161).
 * Pages whose block id is 0 are skipped (kernels.cu:25-26).
 * indices_flat is a device int32 array of indices_numel entries on
 * indices_device; indices_offsets has num_jobs+1 host entries. */
DARIC_API int daric_copier_gather_pages(daric_copier* copier, int64_t num_jobs, const char* const* layer_names,
                              const int64_t* offsets, const int64_t* byte_sizes,
                              const int32_t* indices_flat, int64_t indices_numel, int indices_device,
                              const int64_t* indices_offsets, void* stream);

/* Replaces `CacheCopier.scatter_pages(...)` (copier.cpp:78-111,
 * kernels.cu:219-292, 86-123): store -> paged KV, same argument meaning as
 * gather_pages. Bit-identical bytes to the reference; 16-byte vectorised when
 * every job is 16-byte aligned, byte-granular otherwise. */
DARIC_API int daric_copier_scatter_pages(daric_copier* copier, int64_t num_jobs, const char* const* layer_names,
                               const int64_t* offsets, const int64_t* byte_sizes,
                               const int32_t* indices_flat, int64_t indices_numel, int indices_device,
                               const int64_t* indices_offsets, void* stream);

/* Attaches the rotary table of a registered layer. Replaces
 * `Adapter.register_rotary_embed(layer_name, rotary_emb)` (adapter.py:109-113)
 * together with the stride resolution of `_launch_triton_rerotate`
 * (adapter.py:311-368): the K rows of the layer are located from the sizes
 * and strides given at register_layer:
 *   5-D non-page-first (2, nb, bs, H, D)  : K = prefix 0, rows (bs, H)
 *   5-D page-first     (nb, 2, bs, H, D)  : K = first half of the page
 *   4-D page-first     (nb, H, bs, 2*D)   : K = first D elements of each row
 *   3-D                (nb, bs, hidden)   : one head of `hidden` elements
 * cos_sin_cache: device [max_position, rotary_dim] array of table_dtype
 * (cos in the first rotary_dim/2 columns, sin in the rest), 16-byte aligned.
 * kv_dtype: element type of the KV layer (BF16, F16, F32 or FP8_E4M3). */
DARIC_API int daric_copier_register_rotary(daric_copier* copier, const char* layer_name, int kv_dtype,
                                 const void* cos_sin_cache, int table_dtype, int64_t max_position,
                                 int64_t rotary_dim, int is_neox);

/* Fused re-rotate + scatter: store -> paged KV with K rotated in fp32.
 * Fuses scatter_pages (kernels.cu:86-123) with the re-rotation that the
 * reference runs afterwards in a second process (adapter.py:196-295 flexible,
 * 118-194 strict, kernel adapter.py:30-88). Job arrays as in scatter_pages;
 * in addition every job belongs to one chunk ("meta"):
 *   job_meta[i]      : chunk index of job i, in [0, num_metas)
 *   meta_pos_a[m]    : FLEXIBLE: saved (old) start position of chunk m
 *                      DELTA   : rotation delta of chunk m
 *   meta_pos_b[m]    : FLEXIBLE: new start position of chunk m (NULL for DELTA)
 *   meta_len[m]      : tokens of chunk m to rotate (token t = page*bs + slot;
 *                      tokens >= meta_len are copied unrotated)
 * FLEXIBLE chunks with old == new are copied unrotated (adapter.py:212).
 * Every job's layer must have register_rotary. Optional deviation scores:
 * when scores != NULL, for job i the kernel writes
 *   scores[job_score_row[i]*score_ld + meta_score_col[m] + t] =
 *       sum over heads and rotary elements of (K'(t) - K(t))^2   (fp32)
 * for every rotated token t of the chunk (unrotated tokens get 0).
 * Host arrays: job_meta, job_score_row (num_jobs); meta_* (num_metas). */
DARIC_API int daric_copier_rerotate_scatter_pages(
    daric_copier* copier, int64_t num_jobs, const char* const* layer_names, const int64_t* offsets,
    const int64_t* byte_sizes, const int32_t* indices_flat, int64_t indices_numel, int indices_device,
    const int64_t* indices_offsets, const int64_t* job_meta, int mode, int64_t num_metas,
    const int64_t* meta_pos_a, const int64_t* meta_pos_b, const int64_t* meta_len, float* scores,
    int64_t score_ld, const int64_t* job_score_row, const int64_t* meta_score_col, void* stream);

/* Chunk-level fused load: the copy plan of KVIOManager._build_copy_plan
 * (management/service/gpu_kv_io.py:334-379: per chunk, per layer, offsets,
 * byte sizes and a block-id list repeated for every layer) built on the
 * device from one descriptor per chunk. layer_names lists every layer of a
 * chunk in store order (the store's sorted layer order,
 * gpu_kv_io.py:355-373); chunk m's region at chunk_stg_off[m] holds, for
 * layer j, [prefix][chunk_pages[m] pages][page bytes] after the layers
 * before it (chunk_pages[m] x their bytes per page). Every layer of chunk m
 * uses the block ids block_ids[chunk_blk_off[m] .. + chunk_pages[m])
 * (device int32). The call loads layers [layer_begin, layer_end) only
 * (layer-wise loading). mode, pos_a/pos_b/len per chunk as meta_* of
 * daric_copier_rerotate_scatter_pages (DARIC_ROPE_NONE: plain scatter);
 * with scores, layer j writes row j at column score_col[m] + t. The layers
 * of one call share one rotary table, KV dtype and rotary style. Same bytes
 * as rerotate_scatter_pages on the expanded plan. */
DARIC_API int daric_copier_load_chunks(daric_copier* copier, int64_t num_layers, const char* const* layer_names,
                                       int64_t layer_begin, int64_t layer_end, int64_t num_chunks,
                                       const int64_t* chunk_stg_off, const int64_t* chunk_blk_off,
                                       const int64_t* chunk_pages, const int32_t* block_ids,
                                       int64_t block_ids_numel, int block_ids_device, int mode,
                                       const int64_t* pos_a, const int64_t* pos_b, const int64_t* len,
                                       float* scores, int64_t score_ld, const int64_t* score_col, void* stream);

/* In-place re-rotation of K in paged caches, all layers in one launch.
 * Replaces the per-layer `_launch_triton_rerotate` / `_fused_rerotate_kernel`
 * loop (adapter.py:174-194, 268-295, 297-396). Work is given per segment
 * (a run of tokens of one request):
 *   seg_blk_off[s]  : offset of the segment's block table in block_table
 *   seg_tok_start[s]: first token position (request-relative) to rotate
 *   seg_tok_len[s]  : number of tokens to rotate
 *   seg_pos_a[s], seg_pos_b[s]: as meta_pos_a/b of rerotate_scatter_pages,
 *        with token t of the segment using positions (a + t, b + t) in
 *        FLEXIBLE mode and a in DELTA mode
 * Token position p lives in slot block_table[seg_blk_off + p / bs]*bs + p % bs
 * (adapter.py:163-171, 258-265). block_table: device int32.
 * The layers are registered layers of `copier`, each with register_rotary.
 * Block id 0 is rotated like any other block, as the reference does. */
DARIC_API int daric_copier_rerotate_inplace(daric_copier* copier, int64_t num_layers,
                                  const char* const* layer_names, int mode, int64_t num_segs,
                                  const int32_t* block_table, int64_t block_table_numel,
                                  const int64_t* seg_blk_off, const int64_t* seg_tok_start,
                                  const int64_t* seg_tok_len, const int64_t* seg_pos_a,
                                  const int64_t* seg_pos_b, void* stream);

/* ======================================================================== */
/* Batched copy-engine DMA — replaces batched_memcpy_d2h / _h2d             */
/* (helpers.cu:187-248, bindings.cpp:18-30): one cudaMemcpyAsync per region. */
/* `host` must be page-locked for the copy to be asynchronous.              */
/* ======================================================================== */
DARIC_API int daric_batched_memcpy_d2h(const void* staging, void* host, int64_t n, const int64_t* stg_offsets,
                             const int64_t* host_offsets, const int64_t* sizes, int device,
                             void* stream);
DARIC_API int daric_batched_memcpy_h2d(const void* host, void* staging, int64_t n,
                             const int64_t* host_offsets, const int64_t* stg_offsets,
                             const int64_t* sizes, int device, void* stream);

/* ======================================================================== */
/* Recompute selection                                                      */
/* ======================================================================== */

/* Score-driven recompute selection with the slot mapping vLLM derives for the
 * selected tokens (integration/vllm/worker.py:310-346: slot =
 * block_ids[p // bs]*bs + p % bs). No reference counterpart computes the
 * scores (the reference's policy is positional, policy.py:45-103); this
 * entry point is the radix select over them.
 *   scores      : device fp32, layer l, token column c at scores[l*score_ld + c]
 *   segments    : request s owns columns [seg_col_off[s], seg_col_off[s]+seg_len[s]);
 *                 its token j is request position seg_pos0[s] + j
 *   TOPK        : selects seg_k[s] tokens (clamped to seg_len) per (layer, s):
 *                 score descending, ties -> lower j; NaN ranks above +inf
 *   THRESHOLD   : selects every j with score >= threshold (NaN never)
 *   outputs (row l, request s): out_idx[l*out_ld + out_off[s] + n] = position,
 *                 out_slot[... same ...] = slot (int64), ascending position
 *                 order; out_count[l*num_segs + s] = number selected.
 *                 Capacity per (l, s) is seg_len[s] for THRESHOLD, seg_k[s]
 *                 for TOPK; out_off must leave that room.
 *   block_table : device int32; request s's table starts at seg_blk_off[s].
 * Host arrays: seg_* and out_off (num_segs entries). */
DARIC_API int daric_score_select(const float* scores, int64_t num_layers, int64_t score_ld, int64_t num_segs,
                       const int64_t* seg_col_off, const int64_t* seg_len, const int64_t* seg_pos0,
                       const int64_t* seg_k, int mode, float threshold, const int32_t* block_table,
                       int64_t block_table_numel, const int64_t* seg_blk_off, int64_t block_size,
                       int32_t* out_idx, int64_t* out_slot, int32_t* out_count, int64_t out_ld,
                       const int64_t* out_off, int device, void* stream);

/* Largest number of requests (segments) one daric_score_select_noalloc call
 * accepts: the size of its fixed scratch. */
#define DARIC_NOALLOC_MAX_SEGMENTS 1024

/* Recompute selection that allocates no device memory. No counterpart in the
 * reference. Same arguments, checks and results as daric_score_select, for
 * callers that must not call cudaMalloc once they are running: a serving
 * process that gave all free device memory to its KV cache at start-up (any
 * later device allocation fails or breaks that budget), or a host whose
 * memory pool owns every device allocation. The per-request descriptors go
 * to a fixed device array inside the library (48 KiB + 256 B, held by every
 * GPU that loads the library until exit) instead of library-allocated
 * scratch, so at most DARIC_NOALLOC_MAX_SEGMENTS requests per call; more are
 * rejected with DARIC_ERR_INVALID. The caller still passes the inputs and
 * outputs. The first call on each device looks up that array's device
 * address and sets the kernel's shared-memory limit; make that first call
 * before any stream capture. All calls share the one array: calls that
 * overlap on the GPU (other streams or threads) race on it and must be
 * serialised by the caller. A block-table index outside the table yields
 * slot -1 (the device error bits of daric_device_errors are not used). */
DARIC_API int daric_score_select_noalloc(const float* scores, int64_t num_layers, int64_t score_ld,
                                         int64_t num_segs, const int64_t* seg_col_off, const int64_t* seg_len,
                                         const int64_t* seg_pos0, const int64_t* seg_k, int mode, float threshold,
                                         const int32_t* block_table, int64_t block_table_numel,
                                         const int64_t* seg_blk_off, int64_t block_size, int32_t* out_idx,
                                         int64_t* out_slot, int32_t* out_count, int64_t out_ld,
                                         const int64_t* out_off, int device, void* stream);

/* DARIC-policy ranges -> recompute index list + slot mapping. Expands the
 * [start, end) ranges of DARICPolicy.get_recompute_ptrs (policy.py:45-103) the
 * way the recompute sub-requests do (worker.py:324-344, utils.py:406-465):
 * range r of request range_req... uses the block table at range_blk_off[r].
 * Output n-th position of the concatenated ranges (in range order):
 *   out_idx[n] = position, out_slot[n] = slot. Host arrays of num_ranges. */
DARIC_API int daric_ptrs_to_slots(int64_t num_ranges, const int64_t* range_start, const int64_t* range_end,
                        const int64_t* range_blk_off, const int32_t* block_table,
                        int64_t block_table_numel, int64_t block_size, int32_t* out_idx,
                        int64_t* out_slot, int device, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* DARIC_B200_H */
