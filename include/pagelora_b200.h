/*
 * pagelora_b200.h -- C ABI of the B200 (sm_100a) PageLoRA decode hot path.
 *
 * Every entry point takes raw device pointers, sizes, strides (in elements)
 * and a CUDA stream (`void *stream` is a cudaStream_t; NULL = legacy default
 * stream).  Nothing here allocates device memory, synchronises the stream or
 * throws: every function returns a pl_status and kernels that detect bad
 * input at run time (a page id outside the pool, a malformed span) write a
 * pl_status code into the caller-owned device word `status_dev` (an int32
 * the caller zeroes once and reads whenever it wants to check).  All
 * launches are capturable in a CUDA graph.
 *
 * Tensor dtypes: bf16 activations / weights / KV, fp32 partial states,
 * int32 page-table metadata, matching the reference's defaults.
 *
 * Each declaration names the reference interface it replaces
 * (paths relative to the PageLoRA project root).
 */
#ifndef PAGELORA_B200_H_
#define PAGELORA_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PL_ABI_VERSION 1

typedef enum pl_status {
  PL_OK = 0,
  PL_ERR_INVALID_ARGUMENT = 1,   /* null pointer, negative size, bad stride        */
  PL_ERR_UNSUPPORTED = 2,        /* head_dim / page_size / group / K not compiled   */
  PL_ERR_PAGE_OUT_OF_RANGE = 3,  /* device: a page id >= num_pages (access skipped)  */
  PL_ERR_WORKSPACE_TOO_SMALL = 4,
  PL_ERR_SPAN_START = 5,         /* "page spans must start at page offset 0"        */
  PL_ERR_SPAN_LENGTH = 6,        /* "page span length is out of range"              */
  PL_ERR_SPAN_NOT_FULL = 7,      /* "non-last page spans must be full pages"        */
  PL_ERR_CUDA = 8,               /* a CUDA runtime call failed (see pl_last_cuda_error) */
  PL_ERR_TIMEOUT = 9,            /* device: a bounded wait ran out (kernel returned) */
  PL_ERR_NO_DEVICE = 10
} pl_status;

/* ---------------------------------------------------------------- library */

/* ABI version (PL_ABI_VERSION) of the loaded library. */
int32_t pl_abi_version(void);

/* Human-readable name of a status code. */
const char *pl_status_string(int32_t status);

/* cudaGetErrorString of the last CUDA failure seen by this library on the
 * calling thread ("" if none). */
const char *pl_last_cuda_error(void);

/* Number of SMs of the current device (cached per device), or -1. */
int32_t pl_device_sm_count(void);

/* ------------------------------------------------------------ page tables */

/*
 * Build CSR page tables from per-row KV block spans, on the device.
 * Replaces model/kvcache/flashinfer_page_table.py:137-181
 * (build_flashinfer_page_table / build_flashinfer_batch_page_table) and
 * the buffer updates at :40-59 and :89-121, including the coalescing of
 * adjacent slices of one page (:184-197) and the validation (:200-221).
 *
 * Input (device, int32): spans of row r are span_* [row_indptr[r],
 * row_indptr[r+1]).  Output (device, int32): out_indptr[num_rows+1],
 * out_indices[<= num_spans], out_last_page_len[num_rows].
 * On a malformed span nothing is written; *status_dev receives
 * PL_ERR_SPAN_START / _LENGTH / _NOT_FULL of the first failing coalesced
 * span in row order and *err_row_dev (nullable) its row.
 * Single launch; num_rows <= 4096, num_spans < 2^31.
 */
int32_t pl_page_table_build(const int32_t *span_block_id,
                            const int32_t *span_start,
                            const int32_t *span_length,
                            const int32_t *row_indptr,
                            int32_t num_rows, int32_t page_size,
                            int32_t *out_indptr, int32_t *out_indices,
                            int32_t *out_last_page_len,
                            int32_t *status_dev, int32_t *err_row_dev,
                            void *stream);

/*
 * Advance a device-resident page table by one decode token per row without
 * any host work (graph-replayable).  Row r keeps its pages in
 * row_pages[r*row_capacity + 0 .. row_num_pages[r]); the row grows by one
 * slot and, when it is empty or its last page is full, the page
 * new_page_ids[r] is appended first.  Writes the append slot of the new
 * token (slot_page_id[r], slot_offset[r]) and, when positions_out is not
 * NULL, its position (tokens in the row - 1), updates row_num_pages and
 * last_page_len in place, and rebuilds the contiguous CSR page table
 * (out_indptr[num_rows+1], out_indices) that pl_paged_decode reads.
 * No reference counterpart as a kernel: it replaces the per-token host
 * rebuild of model/flashinfer/generation.py:188-247 (_plan_decode*) and
 * paged_kvcache_manager.py:195-213 (reserve_chunk) for one-token chunks.
 * Single launch; num_rows <= 4096.
 */
int32_t pl_page_table_advance(int32_t *row_num_pages, int32_t *last_page_len,
                              int32_t *row_pages, const int32_t *new_page_ids,
                              int32_t num_rows, int32_t row_capacity,
                              int32_t page_size, int32_t *out_indptr,
                              int32_t *out_indices, int32_t *slot_page_id,
                              int32_t *slot_offset, int32_t *positions_out,
                              int32_t *status_dev, void *stream);

/* ------------------------------------------------------- decode attention */

typedef struct pl_decode_plan_t {
  int32_t num_splits;        /* KV splits per (row, kv head); 1 = no merge      */
  int32_t ctas;              /* grid size = batch * num_kv_heads * num_splits   */
  int64_t workspace_bytes;   /* bytes of workspace pl_paged_decode needs         */
} pl_decode_plan_t;

/*
 * Host planning of one decode step (no device access, no sync).
 * Replaces model/flashinfer/attention_backend.py:63-118 (plan_decode) and
 * the FlashInfer plan() it calls (:229-285): picks the split-KV factor so
 * that batch*num_kv_heads*num_splits fills the device.  total_pages is an
 * upper bound of the pages of all rows (e.g. indices.numel()).
 */
int32_t pl_decode_plan(int32_t batch, int32_t num_qo_heads,
                       int32_t num_kv_heads, int32_t head_dim,
                       int32_t page_size, int64_t total_pages,
                       int32_t max_splits, pl_decode_plan_t *plan_out);

/*
 * Paged GQA decode attention, one query token per row.
 * Replaces attention_backend.py:120-131 (run_decode) and FlashInfer's
 * BatchDecodeWithPagedKVCacheWrapper.run it wraps.
 *
 *   q        bf16 [batch, num_qo_heads, head_dim], strides (q_stride_b, q_stride_h)
 *   kv_cache bf16 NHD pool of ONE layer [num_pages, 2, page_size, num_kv_heads, head_dim]
 *            (K at [:,0], V at [:,1]), contiguous (paged_kv_store.py:559-570)
 *   indptr/indices/last_page_len int32 CSR page table (device)
 *   out      bf16 [batch, num_qo_heads, head_dim] (strides as q's, o_stride_*)
 *   out_lse  fp32 [batch, num_qo_heads] natural-log LSE, nullable
 *   sm_scale softmax scale applied to q.k (the reference's
 *            (q / 16) * (16 / sqrt(D)) == q / sqrt(D))
 *   num_splits from pl_decode_plan; with num_splits > 1 the partial states
 *            go to `workspace` and the last CTA of each (row, kv head) merges
 *            them (no second launch).  The first 4*batch*num_kv_heads bytes of
 *            the workspace are arrival counters that must be zero before the
 *            first call; every call leaves them zero again.  The partials
 *            follow the counters, so a workspace serves calls of one
 *            batch x num_kv_heads; give calls of other shapes their own.
 * Supported: head_dim 64 or 128, page_size 16 or 32, group (qo/kv) <= 16.
 * A row with no pages yields O = 0 and LSE = -inf.
 */
int32_t pl_paged_decode(const void *q, int64_t q_stride_b, int64_t q_stride_h,
                        const void *kv_cache, int64_t num_pages,
                        const int32_t *indptr, const int32_t *indices,
                        const int32_t *last_page_len,
                        int32_t batch, int32_t num_qo_heads,
                        int32_t num_kv_heads, int32_t head_dim,
                        int32_t page_size, float sm_scale,
                        int32_t num_splits,
                        void *out, int64_t o_stride_b, int64_t o_stride_h,
                        float *out_lse,
                        void *workspace, int64_t workspace_bytes,
                        int32_t *status_dev, void *stream);

/*
 * RoPE table of one decode step: cos_sin[r][i] = (cos, sin) of
 * positions[r] * theta^(-2i / head_dim), i < head_dim / 2, fp32 (the
 * non-interleaved rotation of model/flashinfer/projection.py:155-190, as
 * FlashInfer's apply_rope_pos_ids computes it).  The positions are those of
 * every layer of the step, so one launch serves them all
 * (pl_paged_decode_qkv's rope_cos_sin).  head_dim % 32 == 0; cos_sin
 * 16-byte aligned.
 */
int32_t pl_rope_cos_sin(const int32_t *positions, int32_t rows,
                        int32_t head_dim, float rope_theta, float *cos_sin,
                        void *stream);

/*
 * One decoder layer's attention from the packed q/k/v projection row:
 * per-head LoRA-B expand, Qwen3 q/k RMSNorm (HF rounding), RoPE, the paged
 * append of the new token's K/V and the paged decode, in one launch.
 * Replaces model/flashinfer/layer_runner.py:283-337 (projection split, head
 * norms, RoPE via model/flashinfer/projection.py:34-190), :399-412
 * (_append_decode_kv_static) and attention_backend.py:120-131 (run_decode).
 *   qkv .. rope_theta  as pl_qkv_rope_append (rows = batch rows)
 *   rope_cos_sin       nullable: the step's RoPE table from pl_rope_cos_sin
 *                      ([batch][head_dim / 2] (cos, sin) fp32, 16-byte
 *                      aligned); without it every launch evaluates the
 *                      angles itself (the same values)
 *   slot_page/offset   where row b's new token goes; it must be the last
 *                      slot of the row's last page in the page table
 *                      (pl_page_table_advance writes both); a row whose slot
 *                      is elsewhere (a split-KV shard that does not hold the
 *                      tail) appends nothing
 *   q_out              nullable: the rotated q [batch, Hq, D] bf16
 *   kv_cache .. out_lse, workspace  as pl_paged_decode; flags
 *                      PL_DECODE_OUT_F32: `out` is fp32 (a split-KV partial)
 */
#define PL_DECODE_OUT_F32 1
int32_t pl_paged_decode_qkv(const void *qkv, int64_t qkv_stride,
                            const float *lora_down, int64_t down_stride,
                            const void *lora_b, int32_t lora_rank,
                            float lora_scale, const int32_t *tok_adapter,
                            const void *q_norm_w, const void *k_norm_w,
                            float norm_eps, const int32_t *positions,
                            float rope_theta, const float *rope_cos_sin,
                            const int32_t *slot_page,
                            const int32_t *slot_offset, void *q_out,
                            void *kv_cache, int64_t num_pages,
                            const int32_t *indptr, const int32_t *indices,
                            const int32_t *last_page_len, int32_t batch,
                            int32_t num_qo_heads, int32_t num_kv_heads,
                            int32_t head_dim, int32_t page_size, float sm_scale,
                            int32_t num_splits, void *out, int64_t o_stride_b,
                            int64_t o_stride_h, float *out_lse, int32_t flags,
                            void *workspace, int64_t workspace_bytes,
                            int32_t *status_dev, void *stream);

/*
 * Paged decode of query rows that share page lists: row b attends to the
 * pages of page-table row b / fold (the CSR has ceil(batch / fold) rows).
 * The `fold` rows of a page-table row sit in one tensor-core tile (fold x
 * group <= 16 query heads), so each shared page is read once per `fold`
 * rows.  Used for the shared prefix of a branch batch (the reference repeats
 * the prefix pages in every branch's table, model/flashinfer/generation.py
 * :872-1132); otherwise as pl_paged_decode (flags PL_DECODE_OUT_F32: fp32
 * out for a partial state merged with pl_merge_states_strided).
 */
int32_t pl_paged_decode_shared(const void *q, int64_t q_stride_b,
                               int64_t q_stride_h, const void *kv_cache,
                               int64_t num_pages, const int32_t *indptr,
                               const int32_t *indices,
                               const int32_t *last_page_len, int32_t batch,
                               int32_t fold, int32_t num_qo_heads,
                               int32_t num_kv_heads, int32_t head_dim,
                               int32_t page_size, float sm_scale,
                               int32_t num_splits, void *out,
                               int64_t o_stride_b, int64_t o_stride_h,
                               float *out_lse, int32_t flags, void *workspace,
                               int64_t workspace_bytes, int32_t *status_dev,
                               void *stream);

/*
 * Split merge of pl_paged_decode (and its variants): with `enable` (the
 * default) the num_splits CTAs of one (row, kv head) run as a thread-block
 * cluster and merge their states through distributed shared memory when
 * num_splits <= 16 and every cluster of the launch fits on the device at
 * once; otherwise, or with enable = 0, through the workspace.  The result is
 * the same up to fp32 summation order.  No reference counterpart (a
 * process-wide switch).
 */
int32_t pl_decode_set_cluster_merge(int32_t enable);

/* Clusters of num_splits decode CTAs (2..16) the current device can hold at
 * once for this head_dim / page_size (0: none); a diagnostic. */
int32_t pl_decode_cluster_capacity(int32_t head_dim, int32_t page_size,
                                   int32_t num_splits);

/*
 * pl_paged_decode with the attention output in fp32 (`out` float, 16-byte
 * aligned): the partial state of a split-KV shard, merged across GPUs with
 * its LSE (pl_merge_states_strided).  No reference counterpart: the
 * cross-GPU split-KV decode of long contexts is new on this path.
 */
int32_t pl_paged_decode_f32(const void *q, int64_t q_stride_b, int64_t q_stride_h,
                            const void *kv_cache, int64_t num_pages,
                            const int32_t *indptr, const int32_t *indices,
                            const int32_t *last_page_len,
                            int32_t batch, int32_t num_qo_heads,
                            int32_t num_kv_heads, int32_t head_dim,
                            int32_t page_size, float sm_scale,
                            int32_t num_splits,
                            float *out, int64_t o_stride_b, int64_t o_stride_h,
                            float *out_lse,
                            void *workspace, int64_t workspace_bytes,
                            int32_t *status_dev, void *stream);

/*
 * pl_paged_decode without a caller workspace.  No counterpart in the
 * reference: FlashInfer's wrapper takes a caller-allocated workspace.
 * The split partials and arrival counters live in a fixed device array of
 * PL_FIXED_SCRATCH_BYTES per device, inside the library; nothing is
 * allocated.  Arguments and results are those of pl_paged_decode.
 *   - The array's first 64 KiB are arrival counters for up to 16384
 *     (row, kv head) pairs whatever the shape, so calls of different shapes
 *     may follow one another; the split partials use the rest.
 *   - Returns PL_ERR_WORKSPACE_TOO_SMALL, launching nothing, when
 *     batch * num_kv_heads exceeds 16384 or the partials (batch *
 *     num_qo_heads * num_splits * (head_dim + 1) * 4 bytes) exceed the
 *     remaining ~4 MiB.
 *   - The first call on each device (that device current) looks up the
 *     array's address and clears it on `stream`; make that first call
 *     before any stream capture.  The array of a freshly loaded library is
 *     zero already, so the clear is a defensive reset.  The address is
 *     looked up again (and the array cleared) when the device's current
 *     context changes, e.g. after cudaDeviceReset.
 *   - One array per device: calls that overlap on a device (two streams,
 *     two host threads) race on it.  Serialise them.
 *   - Every completed call leaves the counters at zero.  A call whose
 *     kernel gave up a bounded wait (status word PL_ERR_TIMEOUT) may leave
 *     a partial count; call pl_fixed_scratch_clear before the next call.
 */
#define PL_FIXED_SCRATCH_BYTES (4 * 1024 * 1024)
int32_t pl_paged_decode_fixed_scratch(const void *q, int64_t q_stride_b,
                                      int64_t q_stride_h, const void *kv_cache,
                                      int64_t num_pages, const int32_t *indptr,
                                      const int32_t *indices,
                                      const int32_t *last_page_len,
                                      int32_t batch, int32_t num_qo_heads,
                                      int32_t num_kv_heads, int32_t head_dim,
                                      int32_t page_size, float sm_scale,
                                      int32_t num_splits, void *out,
                                      int64_t o_stride_b, int64_t o_stride_h,
                                      float *out_lse, int32_t *status_dev,
                                      void *stream);

/*
 * Re-zero the arrival counters of this device's fixed scratch array on
 * `stream` (no reference counterpart; it belongs to
 * pl_paged_decode_fixed_scratch).  Needed only after a call whose status
 * word reported PL_ERR_TIMEOUT; allocates nothing.  Same first-call rule as
 * pl_paged_decode_fixed_scratch.
 */
int32_t pl_fixed_scratch_clear(void *stream);

/*
 * Merge S partial attention states per (row, head) by log-sum-exp.
 * No reference counterpart in the project (FlashInfer merges internally);
 * it is the merge step of split-KV decode and of the cross-GPU split-KV
 * path (partials gathered over NCCL).
 *   v_partial   fp32 [num_rows, num_states, head_dim] (row = (batch, head))
 *   lse_partial fp32 [num_rows, num_states] natural log; -inf = empty state
 *   out         bf16 [num_rows, head_dim] (row stride out_stride), out_lse nullable
 */
int32_t pl_merge_states(const float *v_partial, const float *lse_partial,
                        int32_t num_rows, int32_t num_states,
                        int32_t head_dim, void *out, int64_t out_stride,
                        float *out_lse, void *stream);

/*
 * pl_merge_states over partials with explicit element strides: state s of
 * row r is v_partial[r * v_row_stride + s * v_state_stride + d] and
 * lse_partial[r * lse_row_stride + s * lse_state_stride], e.g. the
 * [gpus][rows][D] result of an all-gather.  No reference counterpart.
 */
int32_t pl_merge_states_strided(const float *v_partial, int64_t v_row_stride,
                                int64_t v_state_stride, const float *lse_partial,
                                int64_t lse_row_stride, int64_t lse_state_stride,
                                int32_t num_rows, int32_t num_states,
                                int32_t head_dim, void *out, int64_t out_stride,
                                float *out_lse, void *stream);

/*
 * pl_paged_decode merged with a prior attention state of the same query
 * rows: out[r, h] = the log-sum-exp merge of (prior_o[r, h], prior_lse[r, h])
 * and this launch's state, with the arithmetic of pl_merge_states_strided
 * over [prior, this], so the bf16 result equals writing this launch's fp32
 * state and merging the two in a separate launch.  prior_o fp32 [batch,
 * num_qo_heads, head_dim] contiguous, 16-byte aligned; prior_lse fp32
 * [batch, num_qo_heads], natural log.  Used for the second pass of a
 * shared-prefix decode (the rows' suffixes after the shared prefix), which
 * the reference runs as one attention over repeated prefix pages
 * (model/flashinfer/generation.py:872-1132).  bf16 out only.
 */
int32_t pl_paged_decode_merge_prior(const void *q, int64_t q_stride_b,
                                    int64_t q_stride_h, const void *kv_cache,
                                    int64_t num_pages, const int32_t *indptr,
                                    const int32_t *indices,
                                    const int32_t *last_page_len, int32_t batch,
                                    int32_t num_qo_heads, int32_t num_kv_heads,
                                    int32_t head_dim, int32_t page_size,
                                    float sm_scale, int32_t num_splits,
                                    void *out, int64_t o_stride_b,
                                    int64_t o_stride_h, const float *prior_o,
                                    const float *prior_lse, void *workspace,
                                    int64_t workspace_bytes, int32_t *status_dev,
                                    void *stream);

/* ------------------------------------------------- split-KV peer exchange */
/*
 * Split-KV decode over GPUs (one process per GPU): every GPU computes a
 * partial (O fp32, LSE) over its page range, and the states are merged by
 * log-sum-exp.  pl_splitkv_exchange_merge does the exchange and the merge in
 * one kernel over NVLink peer memory, instead of an all-gather collective
 * followed by pl_merge_states_strided.  No reference counterpart (the
 * reference runs on one GPU).
 *
 * Set-up, once per GPU, on buffers the caller allocates (nothing here
 * allocates):
 *   gather  fp32 [2][world][slot] (slot = pl_splitkv_exchange_slot_floats),
 *           zeroed;
 *   flags   int32 [world][ctas] (ctas = pl_splitkv_exchange_ctas), zeroed;
 *   epochs  int32 [ctas], zeroed.
 * Export gather and flags with pl_ipc_export, share the handle bytes and
 * offsets with the other GPUs (e.g. an all-gather at start-up), map the
 * peers' buffers with pl_ipc_import, and put the world gather pointers and
 * the world flag pointers (this GPU's own ones at index rank) into two
 * device arrays.  Peer access needs GPUs that reach each other over NVLink
 * or PCIe P2P.
 *
 *   part    this GPU's partial, packed: O [rows_h][head_dim] fp32, then LSE
 *           [rows_h] (natural log, as pl_paged_decode_f32's out_lse);
 *           16-byte aligned; head_dim % 4 == 0
 *   out     bf16 [rows_h][head_dim]: the merged output, bit-identical to
 *           pl_merge_states_strided over the all-gathered partials, and the
 *           same on every GPU
 * Every GPU must make the same sequence of calls (same rows_h, head_dim,
 * rows_per_cta).  Each CTA waits (bounded, ~2 s) for the same CTA of every
 * other GPU; a wait that runs out writes PL_ERR_TIMEOUT to *status_dev and
 * the CTA returns without merging.
 */
int32_t pl_ipc_handle_bytes(void);
int32_t pl_ipc_export(const void *dev_ptr, void *handle_out,
                      int64_t *offset_out);
int32_t pl_ipc_import(const void *handle, int64_t offset, void **dev_ptr_out);
int32_t pl_ipc_close(void *dev_ptr, int64_t offset);
int64_t pl_splitkv_exchange_slot_floats(int32_t rows_h, int32_t head_dim);
int32_t pl_splitkv_exchange_ctas(int32_t rows_h, int32_t rows_per_cta);
int32_t pl_splitkv_exchange_merge(const float *part,
                                  void *const *peer_gather_dev,
                                  int32_t *const *peer_flags_dev,
                                  const int32_t *flags_local, int32_t *epochs,
                                  int32_t rank, int32_t world, int32_t rows_h,
                                  int32_t head_dim, int32_t rows_per_cta,
                                  void *out, int32_t *status_dev,
                                  void *stream);

/* ------------------------------------------------------ prefill attention */
/*
 * Ragged paged prefill attention on the tcgen05 tensor cores.  Replaces
 * model/flashinfer/attention_backend.py:133-190 (plan_prefill + run_prefill:
 * FlashInfer BatchPrefillWithPagedKVCacheWrapper, NHD, pos_encoding NONE,
 * sm_scale = query_rescale / sqrt(D) applied to q / query_rescale, which is
 * sm_scale = 1/sqrt(D) on q itself).  Nothing is planned on the host: the
 * kernel finds each CTA's (request, query tile) from qo_indptr, so the call
 * depends on the shapes only and can be captured once per total_q.
 *   q           bf16, token t / head h at q + t*q_stride_t + h*q_stride_h
 *               (strides in elements, multiples of 8; 16-byte aligned)
 *   qo_indptr   int32 [batch+1]: request b owns tokens [qo_indptr[b], qo_indptr[b+1])
 *   kv_*        the request's pages, as for pl_paged_decode; the queries are
 *               the LAST qo_len positions of the kv_len keys (causal: query i
 *               sees keys 0 .. kv_len - qo_len + i)
 *   total_q     >= qo_indptr[batch]; sizes the grid and bounds every q/out access
 *   out         bf16 like q; out_lse nullable fp32 [total_q, num_qo_heads], natural log
 * head_dim 64 or 128, page_size 16/32/64/128, num_qo_heads / num_kv_heads
 * <= 128.  Rows with no visible key get O = 0 (LSE -inf).  Device errors
 * (PL_ERR_PAGE_OUT_OF_RANGE: the page reads as zeros; PL_ERR_INVALID_ARGUMENT:
 * qo_indptr outside [0, total_q]) go to *status_dev.
 */
int32_t pl_paged_prefill(const void *q, int64_t q_stride_t, int64_t q_stride_h,
                         const void *kv_cache, int64_t num_pages,
                         const int32_t *qo_indptr, const int32_t *kv_indptr,
                         const int32_t *kv_indices,
                         const int32_t *kv_last_page_len, int32_t batch,
                         int32_t total_q, int32_t num_qo_heads,
                         int32_t num_kv_heads, int32_t head_dim,
                         int32_t page_size, float sm_scale, int32_t causal,
                         void *out, int64_t out_stride_t, int64_t out_stride_h,
                         float *out_lse, int32_t *status_dev, void *stream);

/* --------------------------------------------------------------- LoRA path */

/*
 * Segment-grouped LoRA shrink: down[t, :] = x[t, :] . A[adapter(seg(t))]^T
 * Replaces the x.A^T half of multilora/linear.py:226-227 and
 * model/flashinfer/packed_ops.py:324 (F.linear(hidden, packed.a)).
 *   x      bf16 [num_tokens, in_features] (row stride x_stride)
 *   a      bf16 [num_adapters, rank, in_features] (stacked, contiguous)
 *   seg_indptr int32 [num_segments+1] token ranges, seg_adapter int32
 *          [num_segments] adapter index (-1 = no LoRA: writes zeros)
 *   down   fp32 [num_tokens, rank] (row stride down_stride)
 */
int32_t pl_lora_shrink_seg(const void *x, int64_t x_stride,
                           const void *a, int32_t num_adapters,
                           int32_t rank, int32_t in_features,
                           const int32_t *seg_indptr,
                           const int32_t *seg_adapter, int32_t num_segments,
                           int32_t num_tokens,
                           float *down, int64_t down_stride, void *stream);

/*
 * Per-token LoRA shrink with an optional RMSNorm in front, one launch:
 *   xn[t]      = bf16(x[t] * rsqrt(mean(x[t]^2) + eps) * norm_w)  (norm_w != NULL;
 *                bit-identical to pl_rmsnorm; written to xn_out when it is
 *                not NULL)
 *   down[t, j] = xn[t] . A[adapter(t)][j, :]  (fp32; x[t] itself without norm_w)
 * adapter(t) = tok_adapter[t] (device, NULL = adapter 0); an adapter
 * outside [0, num_adapters) gives zeros.  A is bf16 [num_adapters, rank,
 * k_in].  Replaces the x . A^T of multilora/linear.py:226-227 and
 * model/flashinfer/packed_ops.py:324 (F.linear(hidden, packed.a)) for
 * per-row adapters, and with norm_w also the RMSNorm of
 * model/flashinfer/norm.py in front of the packed q/k/v projection.  One
 * CTA per (token, 4 rank rows): k_in % 8 == 0 and k_in <= 8192
 * (PL_ERR_UNSUPPORTED otherwise).
 */
int32_t pl_lora_shrink_rows(const void *x, int64_t x_stride,
                            int32_t num_tokens, int32_t k_in,
                            const void *norm_w, float norm_eps, void *xn_out,
                            int64_t xn_stride, const void *a,
                            int32_t num_adapters, int32_t rank,
                            const int32_t *tok_adapter, float *down,
                            int64_t down_stride, void *stream);

/* Epilogue/prologue selectors of pl_linear_lora_expand_fused. */
#define PL_PROLOGUE_NONE 0     /* x used as given                                    */
#define PL_PROLOGUE_RMSNORM 1  /* x <- bf16(x * rsqrt(mean(x^2)+eps) * norm_w)       */
#define PL_PROLOGUE_SILU_MUL 2 /* x[t] <- bf16(silu(x[t,:K]) * x[t,K:2K]) (gate_up)  */
#define PL_FLAG_WEIGHTS_STATIC 1
#define PL_FLAG_DOWN_FROM_X 2  /* lora_down unused: the kernel computes the LoRA   */
                               /* down x . A^T itself; shrink_a = A stack          */
                               /* [n_shrink adapters][lora_rank][k_in] (token t   */
                               /* uses tok_adapter[t], or 0), lora_rank <= 64,    */
                               /* one slice; no shrink rows are produced          */

/*
 * Base projection with the LoRA expand and residual fused into its epilogue:
 *   base   = x . W^T (+ bias)                              (W bf16 [n_out, K])
 *   delta  = bf16( bf16( B[adapter(t)][o, :] . bf16(down[t, roff(o) : roff(o)+rank]) ) * lora_scale )
 *   y      = bf16( bf16(base) + delta )                     (lora_b != NULL)
 *   y      = bf16( residual + bf16(y) )                     (residual != NULL)
 * roff(o) = rank * (slice of o), slices are [0, slice_end[0]), [slice_end[0],
 * slice_end[1]), ... (up to 4, e.g. q/k/v) -- the packed block-diagonal B of
 * packed_ops.py:328-384 without its zero blocks.  B is bf16
 * [num_adapters, n_out, rank]; pass B * scale with lora_scale = 1 for the
 * packed path (packed_ops.py:371-373 folds the scale into B) or the plain B
 * with lora_scale = alpha/rank for LoRALinear.forward (linear.py:230-231
 * scales the rounded product).  adapter(t) = tok_adapter[t] (device, -1 =
 * none) or 0 when tok_adapter is NULL.
 * Optionally extra "shrink rows": rows n_out .. n_out+n_shrink of the
 * weight stream are taken from shrink_a (bf16 [n_shrink, K]) and their
 * fp32 results x . shrink_a^T are written to shrink_out[t, :] (row stride
 * shrink_stride) -- the LoRA shrink of the NEXT stage fused into this pass.
 * Replaces packed_ops.py:105-165 (project_qkv_packed), :251-265
 * (project_linear), :314-325 (_packed_lora_delta) and
 * multilora/linear.py:200-231 (LoRALinear.forward) for num_tokens <= 8.
 * The input prologue (PL_PROLOGUE_*) folds the preceding RMSNorm
 * (model/flashinfer/norm.py:15-24) or SiLU-and-mul (packed_ops.py:230-239).
 * Requires K % 16 == 0; x rows are read with stride x_stride.
 * slice_end is a HOST array (num_slices-1 row bounds, read during the call).
 * flags: PL_FLAG_WEIGHTS_STATIC lets the kernel stream w / shrink_a before
 * the preceding kernel on the stream has finished (programmatic dependent
 * launch); pass it only when no upstream kernel writes those weights.
 * PL_FLAG_DOWN_FROM_X folds the LoRA shrink of multilora/linear.py:226-227
 * (x . A^T, fp32) into the launch: every CTA computes the down values of
 * its tokens from the staged x, so no separate pl_lora_shrink_seg runs.
 */
int32_t pl_linear_lora_expand_fused(
    const void *x, int64_t x_stride, int32_t num_tokens, int32_t k_in,
    int32_t prologue, const void *norm_w, float norm_eps,
    const void *w, int32_t n_out, const void *bias,
    const float *lora_down, int64_t down_stride, const void *lora_b,
    int32_t lora_rank, float lora_scale, const int32_t *slice_end,
    int32_t num_slices,
    const int32_t *tok_adapter,
    const void *residual, int64_t res_stride,
    void *y, int64_t y_stride,
    const void *shrink_a, int32_t n_shrink, float *shrink_out,
    int64_t shrink_stride, int32_t flags,
    int32_t *status_dev, void *stream);

/*
 * One projection of pl_linear_lora_chain: the arguments of
 * pl_linear_lora_expand_fused, with the slice bounds held in the struct.
 */
typedef struct PlGemvPhase {
  const void *x;
  int64_t x_stride;
  int32_t num_tokens, k_in, prologue;
  const void *norm_w;
  float norm_eps;
  const void *w;
  int32_t n_out;
  const void *bias;
  const float *lora_down;
  int64_t down_stride;
  const void *lora_b;
  int32_t lora_rank;
  float lora_scale;
  int32_t slice_end[3];
  int32_t num_slices;
  const int32_t *tok_adapter;
  const void *residual;
  int64_t res_stride;
  void *y;
  int64_t y_stride;
  const void *shrink_a;
  int32_t n_shrink;
  float *shrink_out;
  int64_t shrink_stride;
  int32_t flags;
} PlGemvPhase;

/*
 * The projection that the next pl_linear_lora_phase call on the stream will
 * run: its weight rows (w [n_out, k_in], then shrink_a [n_shrink, k_in]),
 * its token count, and how many of its first ring stages (16 rows x up to
 * 2048 columns each) every CTA should find in L2.
 */
typedef struct PlGemvPrefetch {
  const void *w;
  int32_t n_out;
  const void *shrink_a;
  int32_t n_shrink;
  int32_t k_in;
  int32_t num_tokens;
  int32_t units;
} PlGemvPrefetch;

/*
 * pl_linear_lora_expand_fused with its arguments in a PlGemvPhase, plus an
 * optional hand-over to the next projection: once a CTA has issued the
 * copies of its own weight rows, it asks for the first `next->units` ring
 * stages that the same CTA of the `next` launch will read to be fetched into
 * L2 (no destination, no wait).  The next launch's first stages then arrive
 * from L2 while DRAM is still busy with this launch's last rows.  next may
 * be NULL (or units 0): no prefetch.  No reference counterpart: a schedule
 * of this build for the o_proj / mlp / qkv_proj sequence of
 * model/flashinfer/layer_runner.py:283-396.  The next launch is expected to
 * have the same number of CTAs per SM (pl_linear_set_tuning).
 */
int32_t pl_linear_lora_phase(const PlGemvPhase *phase,
                             const PlGemvPrefetch *next, int32_t *status_dev,
                             void *stream);

/*
 * Consecutive projections of one decoder layer in ONE launch, each with the
 * semantics and rounding of pl_linear_lora_expand_fused, e.g. o (LoRA
 * expand + residual) -> gate_up (RMSNorm) -> down (SiLU-and-mul + residual)
 * -> the next layer's packed q/k/v (RMSNorm + LoRA shrink rows): the
 * o_proj / mlp / next qkv_proj sequence of
 * model/flashinfer/layer_runner.py:338-396 for num_tokens <= 8.
 * Phase p reads what phase p-1 wrote: the launch is persistent (one CTA
 * per SM, all resident), the weights of every phase stream through one
 * shared-memory ring without waiting for the activations, and the CTAs meet
 * at a grid barrier between phases.
 *   phases       host array of num_phases (1..6) projections, all with the
 *                same num_tokens; read during the call
 *   grid_barrier device int32, zero before the first call; every call leaves
 *                it zero again.  After a call whose status word reports
 *                PL_ERR_TIMEOUT it may be left non-zero: zero it before the
 *                next call.  Only needed when num_phases > 1.
 * A phase's lora_down must not be the shrink output of an earlier phase of
 * the same call (PL_ERR_UNSUPPORTED): it is read through L1.  x / residual
 * of a later phase may be any earlier phase's y (read from L2).  Weights are
 * streamed before the preceding kernel on the stream has finished, as with
 * PL_FLAG_WEIGHTS_STATIC: no upstream kernel may write them.  Bounded waits
 * report PL_ERR_TIMEOUT through *status_dev.
 */
int32_t pl_linear_lora_chain(const PlGemvPhase *phases, int32_t num_phases,
                             int32_t *grid_barrier, int32_t *status_dev,
                             void *stream);

/*
 * Kernel variant and pipeline shape of pl_linear_lora_expand_fused for this
 * process.  No reference counterpart (a tuning knob).
 *   mode -1: restore the built-in defaults (tuning and L2 prefetch).
 *   mode 0: by size -- register-direct for launches of <= 64 MiB of weights
 *           (shapes as last set for mode 2), TMA ring above (as last set for
 *           mode 1); the other arguments are checked but unused.
 *   mode 1: TMA ring -- stages x (16 rows x cols_per_stage) bulk copies,
 *           consumer_warps (4 or 8) mma warps, ctas_per_sm (1..4) CTAs per SM;
 *           the ring is made shallower when tokens x K does not fit.
 *   mode 2: register-direct loads -- consumer_warps (4 or 8) warps per CTA,
 *           grid of ctas_per_sm (1..16) CTAs per SM (stages / cols_per_stage
 *           are checked but unused).
 */
int32_t pl_linear_set_tuning(int32_t mode, int32_t stages,
                             int32_t cols_per_stage, int32_t consumer_warps,
                             int32_t ctas_per_sm);

/*
 * Register-direct variant (tuning mode 2) with PL_FLAG_WEIGHTS_STATIC: bytes
 * of weights per launch (whole 16-row tiles, the first ones of each CTA)
 * that are prefetched into L2 before the upstream grid completes.  0 (the
 * default) disables it; at most 1 GiB.  No reference counterpart.
 */
int32_t pl_linear_set_l2_prefetch(int64_t max_bytes);

/* ------------------------------------------- multi-token linear (tcgen05) */

typedef struct pl_gemm_plan_t {
  int32_t ctas;              /* grid size (one CTA per SM unless capped)        */
  int32_t max_slots;         /* most CTAs sharing one 128-row weight tile       */
  int64_t workspace_bytes;   /* bytes of workspace pl_linear_lora_gemm needs   */
} pl_gemm_plan_t;

/*
 * Work split of pl_linear_lora_gemm for T tokens (1..128), K inputs and
 * n_out rows over num_ctas CTAs (0: one per SM of the current device).
 */
int32_t pl_linear_gemm_plan(int32_t num_tokens, int32_t k_in, int32_t n_out,
                            int32_t num_ctas, pl_gemm_plan_t *plan);

/*
 * Whether pl_linear_lora_gemm with these sizes and a rank-16 LoRA (16-byte
 * aligned B) computes the LoRA terms of a CTA's last tile ahead, while the
 * weights stream (1), or expands them in the final merge (0); negative on
 * invalid sizes.  CTAs owning fewer than half a tile of units expand in the
 * merge either way.  No reference counterpart (a query of this library's
 * plan, for tests and tuning).
 */
int32_t pl_linear_gemm_lora_precompute(int32_t num_tokens, int32_t k_in,
                                       int32_t n_out, int32_t num_ctas,
                                       int32_t lora_rank, int32_t num_slices);

/*
 * Multi-token LoRA linear on the tcgen05 tensor cores (TMA-fed, accumulator
 * in tensor memory, persistent grid sharing 128-row x 256-column units
 * evenly over the SMs): the batched-decode / prefill-chunk counterpart of
 * pl_linear_lora_expand_fused for 1..128 tokens.  Replaces
 * multilora/linear.py:200-231 (LoRALinear.forward: F.linear + the LoRA
 * delta) and model/flashinfer/packed_ops.py:105-165, 251-265
 * (project_qkv_packed / project_linear) for a multi-sequence batch.
 *   x           bf16 [T, K] (row stride x_stride), already normalised
 *               (pl_rmsnorm / pl_silu_mul); 16-byte aligned, K % 8 == 0
 *   w           bf16 [n_out, K] row-major
 *   epilogue    bias, LoRA expand and residual exactly as in
 *               pl_linear_lora_expand_fused; tok_adapter[t] selects token
 *               t's adapter (-1: none), so a batch mixes adapters
 *               (segment-grouped shrink: pl_lora_shrink_seg)
 *   num_ctas    grid size (0: one per SM); the result does not depend on it
 *               beyond fp32 summation order, and is deterministic for a
 *               given value
 *   workspace   256-byte aligned, pl_linear_gemm_plan's workspace_bytes for
 *               the same num_ctas; its first 4 * ceil(n_out / 128) bytes
 *               are arrival counters: zero before the first call, left zero.
 *   flags       PL_FLAG_WEIGHTS_STATIC as for the GEMV; PL_FLAG_SILU_PAIRS:
 *               w is a gate/up stack interleaved in blocks of 64 rows (rows
 *               128j .. 128j+63 = gate rows 64j .. 64j+63, the next 64 = the
 *               same up rows) and y gets the SiLU-and-mul instead,
 *               y[t, c] = bf16(silu(bf16(g)) * bf16(u)) for c < n_out / 2:
 *               the gate_up projection and pl_silu_mul of
 *               model/flashinfer/packed_ops.py:168-239 in one launch, with the
 *               same rounding.  Needs n_out % 128 == 0, y_stride % 4 == 0, y
 *               8-byte aligned, and no bias, LoRA or residual.
 */
#define PL_FLAG_SILU_PAIRS 8
int32_t pl_linear_lora_gemm(const void *x, int64_t x_stride, int32_t num_tokens,
                            int32_t k_in, const void *w, int32_t n_out,
                            const void *bias, const float *lora_down,
                            int64_t down_stride, const void *lora_b,
                            int32_t lora_rank, float lora_scale,
                            const int32_t *slice_end, int32_t num_slices,
                            const int32_t *tok_adapter, const void *residual,
                            int64_t res_stride, void *y, int64_t y_stride,
                            int32_t num_ctas, void *workspace,
                            int64_t workspace_bytes, int32_t flags,
                            int32_t *status_dev, void *stream);

/*
 * FlashInfer RMSNorm over T rows (one bf16 rounding):
 * y = bf16(x * rsqrt(mean(x^2) + eps) * w).  Replaces model/norm.py:51-54
 * (flashinfer rmsnorm, called at model/norm.py:51-65) on the decode path.
 * K % 8 == 0.
 */
int32_t pl_rmsnorm(const void *x, int64_t x_stride, int32_t num_tokens,
                   int32_t k_in, const void *w, float eps, void *y,
                   int64_t y_stride, void *stream);

/*
 * Hugging Face RMSNorm over rows (two bf16 roundings, as LlamaRMSNorm /
 * Qwen3RMSNorm compute it): y = bf16(w * bf16(x * rsqrt(mean(x^2) + eps))).
 * With one row per (token, head) and K = head_dim it is the Qwen3 q/k head
 * norm of model/flashinfer/projection.py:248-262 (_apply_optional_head_norm,
 * the module call when the FlashInfer norm is off).  K % 8 == 0.
 */
int32_t pl_rmsnorm_hf(const void *x, int64_t x_stride, int32_t num_rows,
                      int32_t k_in, const void *w, float eps, void *y,
                      int64_t y_stride, void *stream);

/*
 * SwiGLU activation over packed [gate | up] rows: y[t, k] =
 * bf16(silu(x[t, k]) * x[t, K + k]), k < K = k_out.  Replaces
 * model/flashinfer/packed_ops.py:237 (flashinfer silu_and_mul).
 */
int32_t pl_silu_mul(const void *x, int64_t x_stride, int32_t num_tokens,
                    int32_t k_out, void *y, int64_t y_stride, void *stream);

/*
 * Merged ("effective") weight builder: w_out = w_in + sign * scale * (B @ A)
 * with the reference's rounding points (bf16 tensors):
 *   mode 0: bf16(w + bf16(bf16(B@A) * scale))  -- linear.py:143-146,166-172
 *                                                 and effective_weights.py:70-72
 *   mode 1: bf16(w + scale * bf16(B@A))        -- effective_weights.py:111-113
 *   sign -1 is unmerge (linear.py:157-159).  w_out may alias w_in.
 *   w bf16 [n_out, k_in]; a bf16 [rank, k_in]; b bf16 [n_out, rank].
 */
int32_t pl_lora_merge_weight(const void *w_in, void *w_out, const void *a,
                             const void *b, int32_t n_out, int32_t k_in,
                             int32_t rank, float scale, int32_t sign,
                             int32_t mode, void *stream);

/* ------------------------------------------------- decode-step glue kernels */

/*
 * Scatter one token per row into the paged KV pool (NHD layout).
 * Replaces model/flashinfer/layer_runner.py:399-412 (_append_decode_kv_static)
 * and paged_kv_append.py:45-118 for single-token rows.
 *   k, v bf16 [num_tokens, num_kv_heads, head_dim] (row strides k_stride/v_stride)
 *   page_id/page_offset int32 [num_tokens]
 */
int32_t pl_kv_append(const void *k, int64_t k_stride, const void *v,
                     int64_t v_stride, void *kv_cache, int64_t num_pages,
                     const int32_t *page_id, const int32_t *page_offset,
                     int32_t num_tokens, int32_t num_kv_heads,
                     int32_t head_dim, int32_t page_size,
                     int32_t *status_dev, void *stream);

/*
 * Post-projection step of one decode token: optional LoRA expand (when
 * lora_down != NULL, same rounding and lora_scale rule as
 * pl_linear_lora_expand_fused; a module without LoRA has zero B rows),
 * optional per-head RMSNorm of q and k (Qwen3 q_norm / k_norm with the HF
 * module's rounding), RoPE (non-interleaved, theta, positions) on q and k,
 * then K/V appended to the paged pool and q written for attention.
 * Replaces model/flashinfer/projection.py:34-190 (head norms +
 * apply_rope_pos_ids) and layer_runner.py:310-329 (static append).
 *   qkv bf16 [num_tokens, (Hq+2*Hkv)*D] row stride qkv_stride
 *   lora_b bf16 [num_adapters, (Hq+2*Hkv)*D, rank] (scale folded), slices q/k/v
 *   positions int32 [num_tokens]; q_out bf16 [num_tokens, Hq, D]
 */
int32_t pl_qkv_rope_append(const void *qkv, int64_t qkv_stride,
                           const float *lora_down, int64_t down_stride,
                           const void *lora_b, int32_t lora_rank,
                           float lora_scale,
                           const int32_t *tok_adapter,
                           const void *q_norm_w, const void *k_norm_w,
                           float norm_eps, const int32_t *positions,
                           float rope_theta, void *q_out, void *kv_cache,
                           int64_t num_pages, const int32_t *page_id,
                           const int32_t *page_offset, int32_t num_tokens,
                           int32_t num_qo_heads, int32_t num_kv_heads,
                           int32_t head_dim, int32_t page_size,
                           int32_t *status_dev, void *stream);

/* out[t, :] = table[token_ids[t], :] (bf16 rows of width dim). */
int32_t pl_embed(const int64_t *token_ids, const void *table, int64_t vocab,
                 int32_t dim, int32_t num_tokens, void *out,
                 int32_t *status_dev, void *stream);

/* First-index argmax over bf16 rows: out_ids[t] = argmax(logits[t, :vocab])
 * (torch.argmax order: NaN wins, ties to the smaller index).
 * Replaces model/flashinfer/sampling.py:8-15 (greedy_argmax_token).  Up to one
 * CTA per SM scans each row; the workspace (16-byte aligned, >= 4*num_tokens +
 * 8*num_tokens*148 bytes) holds the candidates and per-row arrival tickets,
 * whose first 4*num_tokens bytes must be zero before the first call (every
 * call leaves them zero). */
int32_t pl_argmax(const void *logits, int64_t stride, int32_t vocab,
                  int32_t num_tokens, int64_t *out_ids, void *workspace,
                  int64_t workspace_bytes, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* PAGELORA_B200_H_ */
