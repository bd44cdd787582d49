/* C ABI of the B200 beam-search decode kernels (libgrs_b200.so).
 *
 * Every entry point takes device pointers, element strides, sizes and a
 * cudaStream_t passed as void*, enqueues its kernels on that stream and
 * returns GRS_OK or a negative grs_status.  Nothing here allocates device
 * memory unless it says so; nothing synchronises the stream.  Errors found by
 * kernels (cache exhausted, bad page, refcount underflow) are written to a
 * caller-provided device status word (int32, 0 = ok) that the host reads once
 * per step.  Each entry point names the reference interface it replaces.
 */
#ifndef GRS_B200_H
#define GRS_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define GRS_API __attribute__((visibility("default")))
#else
#define GRS_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  GRS_OK = 0,
  GRS_ERR_EXHAUSTED = -1,    /* "paged KV cache exhausted" (paged_cache.py:87) */
  GRS_ERR_BAD_PAGE = -2,     /* "retaining an unallocated page" (paged_cache.py:96) */
  GRS_ERR_REFCOUNT = -3,     /* "negative page reference count" (paged_cache.py:103) */
  GRS_ERR_SHAPE = -4,        /* bad shape / unsupported layout */
  GRS_ERR_CUDA = -5,         /* a launch failed */
  GRS_ERR_CORRUPT = -6,      /* "free-list corruption" (paged_cache.py:90) */
  GRS_ERR_LENGTH = -7,       /* "prefix handle length/block table mismatch" (paged_cache.py:228) */
  GRS_ERR_WORKSPACE = -8,    /* caller workspace too small */
  GRS_ERR_TOO_LARGE = -9,    /* inputs exceed a fixed internal scratch capacity */
  GRS_ERR_TIMEOUT = -10,     /* a bounded in-kernel wait ran out (device status word) */
  GRS_ERR_ORDER = -11        /* ranked records out of order or inconsistent (sharded search) */
} grs_status;

enum { GRS_DTYPE_BF16 = 0, GRS_DTYPE_F32 = 1 };

/* Library version string. */
GRS_API const char* grs_version(void);

/* Number of kernels this library has launched in the process so far (every
 * launch site counts itself; library kernels such as CUB sorts do not). */
GRS_API int64_t grs_launch_count(void);
/* Add n to that counter: the library kernels a replay of a captured CUDA
 * graph launches (counted once at capture time, not by the replay). */
GRS_API void grs_count_launches(int64_t n);

/* ---- paged attention: paged_attention.py:217-306 (paged_attention) ------
 * query [B,H,Q,D] (strides q_sb,q_sh,q_sq; D contiguous); key/value cache
 * [pages,page,H,D] (strides kc_sp,kc_st,kc_sh; D contiguous); block_table
 * int32 [B, >=1] (row stride bt_stride, max_blocks columns); lengths int32 [B];
 * optional current_key/value [B,H,D] + current_valid uint8 [B] (all or none,
 * paged_attention.py:230-232); optional shared_key/value [num_shared,H,D]
 * contiguous, attended by every beam before its pages (not in the
 * reference; the shared-prefix decode microbenchmark).  Rows with no valid
 * key are written as zeros.  Block-table entries outside [0, num_pages) are
 * not read (such a token is treated as absent). */
GRS_API int grs_paged_attention(int dtype, const void* query, int64_t q_sb, int64_t q_sh, int64_t q_sq,
                        const void* key_cache, const void* value_cache, int64_t kc_sp,
                        int64_t kc_st, int64_t kc_sh, const int32_t* block_table,
                        int64_t bt_stride, const int32_t* lengths, const void* current_key,
                        const void* current_value, int64_t ck_sb, int64_t ck_sh,
                        const uint8_t* current_valid, const void* shared_key,
                        const void* shared_value, int64_t num_shared, void* output,
                        int64_t o_sb, int64_t o_sh, int64_t o_sq, int batch, int heads,
                        int query_len, int head_width, int page_size, int max_blocks,
                        int num_pages, void* stream);

/* Causal one-token decode (bf16, head width 32, one query, heads <= 16): the
 * causal action layers' attention (paged_attention.py:18-159 with the current
 * token, :101-132; paged_model.py:66-94) with grs_paged_attention's
 * semantics for query_len 1 and no shared prefix.  One CTA per beam stages
 * the beam's pages with one bulk copy per page of K and of V; needs pages
 * contiguous in the arena (kc_sh == 32, kc_st == heads * 32, kc_sp == page *
 * kc_st, the value arena with the same strides), page dividing 64, 16-byte
 * aligned query / cache / current tensors and strides that are multiples of
 * 8 elements; GRS_ERR_SHAPE otherwise (nothing launched).  current_key may
 * be null (no current token); current_valid may be null (all valid).  Page
 * ids outside [0, num_pages) set GRS_ERR_BAD_PAGE in `status` and their
 * tokens are skipped; a bounded wait that gives up sets GRS_ERR_TIMEOUT. */
GRS_API int grs_decode_causal(const void* query, int64_t q_sb, int64_t q_sh,
                              const void* key_cache, const void* value_cache, int64_t kc_sp,
                              int64_t kc_st, int64_t kc_sh, const int32_t* block_table,
                              int64_t bt_s, const int32_t* lengths, int num_pages,
                              const void* current_key, const void* current_value, int64_t ck_sb,
                              int64_t ck_sh, const uint8_t* current_valid, void* out,
                              int64_t o_sb, int64_t o_sh, int batch, int heads, int page,
                              int32_t* status, void* stream);

/* Shared-prefix decode (bf16, head width 32, one query, heads <= 8): the
 * same semantics as grs_paged_attention with query_len 1 (token order:
 * shared prefix, pages, current token).  One CTA per 32 consecutive beams
 * and head holds every key those beams see: the head's slice of the shared
 * prefix (staged once per CTA), each distinct page of each 16-beam tile
 * (deduplicated per block-table column) and the current tokens, so no
 * partial leaves the CTA.  block_table rows hold max_blocks (<= 32)
 * entries.  Requires 16-byte aligned query, cache, current and shared
 * tensors, heads adjacent in the cache and current rows (head stride 32)
 * and strides that are multiples of 8 elements; returns GRS_ERR_SHAPE
 * otherwise (the caller then uses grs_paged_attention).  The kernel has no
 * in-kernel waits and leaves `status` untouched. */
GRS_API int grs_decode_attention_shared(const void* query, int64_t q_sb, int64_t q_sh,
                                        const void* key_cache, const void* value_cache,
                                        int64_t kc_sp, int64_t kc_st, int64_t kc_sh,
                                        const int32_t* block_table, int64_t bt_stride,
                                        int max_blocks, const int32_t* lengths, int num_pages,
                                        const void* current_key, const void* current_value,
                                        int64_t ck_sb, int64_t ck_sh,
                                        const uint8_t* current_valid, const void* shared_key,
                                        const void* shared_value, int num_shared, void* output,
                                        int64_t o_sb, int64_t o_sh, int batch, int heads,
                                        int page_size, int32_t* status, void* stream);

/* The same decode in one launch of 8-CTA clusters of 16 beams (the earlier
 * design, kept for comparison): each cluster reads every distinct page of
 * its beams once, shared and page keys are split across the cluster and the
 * partials are combined through distributed shared memory.  Same arguments
 * and shape rules as grs_decode_attention_shared.  `status` (device int32,
 * may be null) receives GRS_ERR_TIMEOUT if an in-kernel wait gives up; it is
 * left untouched otherwise. */
GRS_API int grs_decode_attention_shared_cluster(const void* query, int64_t q_sb, int64_t q_sh,
                                                const void* key_cache, const void* value_cache,
                                                int64_t kc_sp, int64_t kc_st, int64_t kc_sh,
                                                const int32_t* block_table, int64_t bt_stride,
                                                int max_blocks, const int32_t* lengths, int num_pages,
                                                const void* current_key, const void* current_value,
                                                int64_t ck_sb, int64_t ck_sh,
                                                const uint8_t* current_valid, const void* shared_key,
                                                const void* shared_value, int num_shared, void* output,
                                                int64_t o_sb, int64_t o_sh, int batch, int heads,
                                                int page_size, int32_t* status, void* stream);

/* ---- PagedKVCache device state: paged_cache.py:16-105 -------------------
 * refcounts int32 [capacity], free_list int32 [capacity] with its length in
 * free_count (device int32), last_pos int32 [capacity] release scratch.
 * grs_cache_init sets refcounts 0, free_list [capacity-1 .. 0]
 * (paged_cache.py:74-75), last_pos -1. */
GRS_API int grs_cache_init(int32_t* refcounts, int32_t* free_list, int32_t* free_count,
                           int32_t* last_pos, int capacity, void* stream);

/* Allocate n pages for rows copied in from another cache (a beam moved
 * between GPUs of a sharded search): pop them from the top of the free list
 * as the append path does, refcount 1 each, page ids into out_pages int32 [n].
 * GRS_ERR_EXHAUSTED in status when the free list is too short. */
GRS_API int grs_cache_alloc(int32_t* refcounts, const int32_t* free_list, int32_t* free_count,
                            int capacity, int n, int32_t* out_pages, int32_t* status,
                            void* stream);

/* paged_cache.py:107-208 (PagedKVCache.append_batch): for each of n parents
 * (block-table rows + lengths) retain the shared pages, allocate the child
 * page from the top of the free list (parent order), COW-copy the valid rows
 * of a partial tail page and write one new row into every arena.  Arenas are
 * contiguous: keys/values [layers, capacity, page, H*D], actions [capacity,
 * page, W], readout keys/values [capacity, page, H*D] (nullable together with
 * new_readout_*).  New rows: keys/values [layers, n, H*D], actions [n, W],
 * readout [n, H*D], in the arena dtype (elem_bytes 2 = bf16, 4 = fp32).
 * Writes child rows (child_cols columns, zero padded) and lengths. */
GRS_API int grs_cache_append(int elem_bytes, int32_t* refcounts, int32_t* free_list,
                             int32_t* free_count, int capacity, const int32_t* parent_table,
                             int64_t parent_stride, const int32_t* parent_lengths, int n,
                             int page_size, int32_t* child_table, int64_t child_stride,
                             int32_t* child_lengths, int child_cols, void* keys, void* values,
                             int layers, int heads_x_width, const void* new_keys,
                             const void* new_values, void* actions, int model_width,
                             const void* new_actions, void* readout_keys, void* readout_values,
                             const void* new_readout_keys, const void* new_readout_values,
                             int32_t* status, void* stream);

/* paged_cache.py:99-105 (PagedKVCache.release) for n handles in order: pages
 * reaching refcount 0 are appended to the free list in scan order. */
GRS_API int grs_cache_release(int32_t* refcounts, int32_t* free_list, int32_t* free_count,
                              int32_t* last_pos, int capacity, const int32_t* table,
                              int64_t stride, const int32_t* lengths, int n, int cols,
                              int page_size, int32_t* status, void* stream);

/* paged_cache.py:223-228: flags GRS_ERR_LENGTH when ceil(length/page) differs
 * from a handle's block count. */
GRS_API int grs_cache_check_lengths(const int32_t* nblocks, const int32_t* lengths, int n,
                                    int page_size, int32_t* status, void* stream);

/* ---- proposals: gpu_proposals.py:69-192 (build_gpu_proposals) -----------
 * Candidates (int64 batch_ids, sources; float32 probabilities; a source < 0
 * marks a padding row that expands to nothing) expand through
 * the CSR rule index (GpuRuleIndex, gpu_proposals.py:20-50; int32 arrays);
 * the stable per-parent cap and global rank select <= global_cap expanded
 * actions: out_row (candidate row), out_xfer, out_next_gate (int64
 * [global_cap], -1 padded), out_count (device int64), out_metrics
 * (device int64 [2] = predicted_actions, eligible_actions).  max_expanded is
 * an upper bound of the expansion size; workspace from
 * grs_proposals_workspace_bytes(num_candidates, max_expanded). */
GRS_API int64_t grs_proposals_workspace_bytes(int64_t max_candidates, int64_t max_expanded);
GRS_API int grs_proposals_rank(const int64_t* batch_ids, const int64_t* sources,
                               const float* probabilities, int64_t num_candidates,
                               const int64_t* parent_gate_counts, int64_t num_parents,
                               const int32_t* xfer_offsets, const int32_t* xfer_counts,
                               const int32_t* xfer_ids, const int32_t* gate_deltas,
                               const int32_t* all_xfer_counts, int num_sources,
                               int64_t max_expanded, int per_parent_cap, int64_t global_cap,
                               int64_t* out_row, int64_t* out_xfer, int64_t* out_next_gate,
                               int64_t* out_count, int64_t* out_metrics, void* workspace,
                               int64_t workspace_bytes, int32_t* status, void* stream);

/* Parent-grouped form of grs_proposals_rank (gpu_proposals.py:69-155 with the
 * same ordering and tie rules) for candidates laid out [parents, k] with the
 * rows of parent b at [b*k, (b+1)*k) and absent rows marked source < 0: the
 * per-parent cap is taken per parent in shared memory (expansion of one
 * parent <= 4096 actions, gate deltas in [-8, 7]) and one stable radix sort
 * ranks the <= parents*cap survivors.  Outputs as grs_proposals_rank (rows
 * index the [parents*k] candidate table); workspace from
 * grs_proposals_grouped_workspace_bytes(parents, per_parent_cap). */
GRS_API int64_t grs_proposals_grouped_workspace_bytes(int64_t parents, int per_parent_cap);
GRS_API int grs_proposals_rank_grouped(const int64_t* sources, const float* probabilities,
                                       int64_t parents, int k, const int64_t* parent_gate_counts,
                                       const int32_t* xfer_offsets, const int32_t* xfer_counts,
                                       const int32_t* xfer_ids, const int32_t* gate_deltas,
                                       const int32_t* all_xfer_counts, int num_sources,
                                       int per_parent_cap, int64_t global_cap, int64_t* out_row,
                                       int64_t* out_xfer, int64_t* out_next_gate,
                                       int64_t* out_count, int64_t* out_metrics, void* workspace,
                                       int64_t workspace_bytes, int32_t* status, void* stream);

/* Proposals from two models' candidates with a per-parent exploration quota
 * (build_legacy_proposals, paged_rollout_benchmark.py:101-210; used while
 * the search runs a second, exploration model, :917-919, 937-961).  The
 * candidate table holds the primary model's rows [0, num_primary) then the
 * exploration model's (source < 0: absent row).  Per parent, each model's
 * allowed actions are ranked (next gate, probability desc, xfer, expansion
 * order); the parent keeps the first cap - quota primary actions, then
 * exploration actions whose (xfer, anchor, binding) is not yet kept
 * (appending before checking the cap, as the reference), then the other
 * primary actions that no kept one repeats, up to the cap; all kept actions
 * are ranked (next gate, probability desc, parent gate) with ties in the
 * parent's list order (next gate, probability desc, xfer, kept position),
 * first global_cap.  Outputs as grs_proposals_rank (rows index the
 * concatenated table); out_metrics int64 [5] = primary predicted, primary
 * eligible, exploration predicted, exploration eligible, selected
 * exploration proposals.  Workspace from
 * grs_proposals_exploration_workspace_bytes. */
GRS_API int64_t grs_proposals_exploration_workspace_bytes(int64_t num_candidates,
                                                          int64_t num_primary,
                                                          int64_t max_expanded,
                                                          int64_t num_parents);
GRS_API int grs_proposals_rank_exploration(
    const int64_t* batch_ids, const int64_t* sources, const int64_t* anchors,
    const float* probabilities, int64_t num_candidates, int64_t num_primary,
    const int64_t* parent_gate_counts, int64_t num_parents, const int32_t* xfer_offsets,
    const int32_t* xfer_counts, const int32_t* xfer_ids, const int32_t* gate_deltas,
    const int32_t* all_xfer_counts, int num_sources, int64_t max_expanded, int per_parent_cap,
    int exploration_per_parent, int64_t global_cap, int64_t* out_row, int64_t* out_xfer,
    int64_t* out_next_gate, int64_t* out_count, int64_t* out_metrics, void* workspace,
    int64_t workspace_bytes, int32_t* status, void* stream);

/* Allocation-free variant of grs_proposals_rank (no counterpart in the
 * reference).  For callers that cannot allocate device memory when they rank
 * proposals (a runtime whose device memory is all pre-reserved by its own
 * pool, a foreign-language binding without access to the framework's
 * allocator, a loop where cudaMalloc would stall the device): the scratch
 * comes from a fixed GRS_PROPOSALS_STATIC_SCRATCH_BYTES array inside the
 * library, held on every GPU that loads it until exit.  Inputs whose
 * workspace (grs_proposals_workspace_bytes) exceeds it return
 * GRS_ERR_TOO_LARGE without launching anything.  The first call on a device
 * resolves the array's device address; make it before any stream capture.
 * Calls share the array: calls that overlap on the GPU race.  Same
 * arguments and outputs as grs_proposals_rank minus the workspace. */
#define GRS_PROPOSALS_STATIC_SCRATCH_BYTES (8ll << 20)
GRS_API int grs_proposals_rank_static(const int64_t* batch_ids, const int64_t* sources,
                                      const float* probabilities, int64_t num_candidates,
                                      const int64_t* parent_gate_counts, int64_t num_parents,
                                      const int32_t* xfer_offsets, const int32_t* xfer_counts,
                                      const int32_t* xfer_ids, const int32_t* gate_deltas,
                                      const int32_t* all_xfer_counts, int num_sources,
                                      int64_t max_expanded, int per_parent_cap,
                                      int64_t global_cap, int64_t* out_row, int64_t* out_xfer,
                                      int64_t* out_next_gate, int64_t* out_count,
                                      int64_t* out_metrics, int32_t* status, void* stream);

/* ---- paged action model: row-wise fused kernels ---------------------------
 * Activation dtype GRS_DTYPE_F32 or GRS_DTYPE_BF16; parameters fp32; rows are
 * B*S slot rows (rows_per_beam = S) or B token rows (rows_per_beam = 1).
 *
 * grs_add_layernorm: residual + LayerNorm with the masks of the reference:
 *   s = x + scale[row]*y; zc = zero_row && zero_beam; wc = where_row &&
 *   where_beam && where_len>0; zero_before: s = zc ? s : 0; sum_out = s;
 *   ln_out = wc ? LN(s) : x, then (if !zero_before) zc ? . : 0.
 *   Covers InitialGraphLayer's norm (model.py:52-53), the node readout
 *   (paged_model.py:375-379), _update_live_nodes (paged_model.py:239-241) and
 *   the causal residual/norm chain (paged_model.py:77-93, 555-558). */
GRS_API int grs_add_layernorm(int dtype, const void* x, int64_t x_stride, const void* y,
                              int64_t y_stride, const float* scale, const float* gamma,
                              const float* beta, void* sum_out, int64_t sum_stride, void* ln_out,
                              int64_t ln_stride, const uint8_t* zero_row,
                              const uint8_t* zero_beam, const uint8_t* where_row,
                              const uint8_t* where_beam, const int32_t* where_len, int64_t rows,
                              int rows_per_beam, int width, float eps, int zero_before,
                              void* stream);
/* y = GELU(y + bias) in place (exact erf GELU, nn.GELU()); GELU optional. */
GRS_API int grs_bias_gelu(int dtype, void* y, int64_t rows, int cols, int64_t stride,
                          const float* bias, int apply_gelu, void* stream);
/* s0 embedding (paged_model.py:246-250). */
GRS_API int grs_embed_initial(int dtype, const int64_t* types, int64_t rows, int width,
                              const float* gate_emb, const float* marker, void* states,
                              int64_t stride, uint8_t* live, void* stream);
/* InitialGraphLayer aggregation (model.py:36-51) over port arrays
 * in/out_node, in/out_port int32 [B, port_slots, 4] (port_slots >= slots);
 * fb = [forward | backward] messages [B*slots, 2W]; rel fp32 [32, W]; writes
 * the degree-normalised sum. */
GRS_API int grs_graph_aggregate(int dtype, const void* fb, int64_t fb_stride, const float* rel,
                                const int32_t* in_node, const int32_t* in_port,
                                const int32_t* out_node, const int32_t* out_port, int64_t rows,
                                int slots, int port_slots, int width, void* agg,
                                int64_t agg_stride, void* stream);
/* Bound-slot gather, pooling and action-context input (paged_model.py:494-523). */
GRS_API int grs_action_inputs(int dtype, const void* states, int64_t state_stride, int slots,
                              const int64_t* xfer_ids, const int64_t* source_ids,
                              const int64_t* source_slots, int pattern, int width,
                              const float* xfer_emb, const float* source_reps, void* bound,
                              void* ctx_in, uint8_t* source_mask, uint8_t* active, int batch,
                              void* stream);
/* token = (raw + action_position[length]) * active (paged_model.py:524-525). */
GRS_API int grs_position_token(int dtype, const void* raw, const float* position,
                               const int32_t* lengths, const uint8_t* active, void* token,
                               int batch, int width, void* stream);
/* _update_live_nodes bound-key attention + action_delta hidden layer
 * (paged_model.py:223-238) for every slot row; writes the GELU hidden
 * [rows, 2W] and the affinity sigmoid(max logit) [rows]. */
GRS_API int grs_update_live_hidden(int dtype, const void* qxa, int64_t qxa_stride,
                                   const void* keys, const void* vw, const void* cvec,
                                   const uint8_t* source_mask, int pattern, int64_t rows,
                                   int slots, int width, void* hidden, int64_t hidden_stride,
                                   float* affinity, void* stream);
/* destination_state hidden layer per (beam, destination) (paged_model.py:592-601). */
GRS_API int grs_destination_hidden(int dtype, const void* r, const float* type_table,
                                   const float* pos_table, const int64_t* dest_slots,
                                   const int64_t* dest_types, const uint8_t* active, int pattern,
                                   int batch, int hidden_width, void* hidden, void* stream);
/* Kill source slots, create destination slots (paged_model.py:569-604). */
GRS_API int grs_apply_slots(int dtype, void* states, int64_t state_stride, uint8_t* live,
                            int64_t* types, int slots, const int64_t* source_slots,
                            const uint8_t* source_mask, int spattern, const int64_t* dest_slots,
                            const int64_t* dest_types, const uint8_t* active, int dpattern,
                            const void* created, int width, int batch, void* stream);
/* match_logits epilogue (model.py:382-389): fp32 logits + eligible mask. */
GRS_API int grs_match_logits(int dtype, const void* acc, int64_t acc_stride,
                             const float* source_bias, const int64_t* first_types,
                             const uint8_t* live, const int64_t* types, int64_t rows,
                             int num_sources, float inv_sqrt_r, float* logits, uint8_t* eligible,
                             void* stream);
/* Beam reindex (index_select of the beam dimension, paged_rollout_benchmark.py
 * :497-499 / :1192-1195) with slot padding: out row i = in row index[i]
 * (in_bytes), tail up to out_bytes filled with fill_byte. */
GRS_API int grs_gather_beams(const void* in, void* out, const int64_t* index, int64_t rows,
                             int64_t in_bytes, int64_t out_bytes, int fill_byte, void* stream);
/* Port arrays from an edge list (model.py:402-418); arrays pre-filled with -1. */
GRS_API int grs_edges_to_ports(const int64_t* edge_batch, const int64_t* edge_src,
                               const int64_t* edge_dst, const int64_t* edge_relation,
                               int64_t edges, int slots, int32_t* out_node, int32_t* out_port,
                               int32_t* in_node, int32_t* in_port, void* stream);

/* ---- candidates: threshold_inference.py:208-297, model.py:391-478 --------
 * grs_select_candidates: per beam row, near/far calibration by rewrite
 * distance (near = distance <= 2), raw-logit threshold, eligibility, then the
 * k best calibrated scores sorted (score desc, flat index asc).  Outputs
 * [batch, k] rows: out_batch (row), out_source (-1 = no candidate),
 * out_anchor, out_prob = sigmoid(score), optional out_score.
 * logits fp32 / eligible uint8 [batch, slots, num_sources]; distance int32
 * [batch, slots]; k <= 2048. */
GRS_API int grs_select_candidates(const float* logits, const uint8_t* eligible,
                                  const int32_t* distance, int batch, int slots, int num_sources,
                                  int k, float near_scale, float near_bias, float near_thr,
                                  float far_scale, float far_bias, float far_thr,
                                  int64_t* out_batch, int64_t* out_source, int64_t* out_anchor,
                                  float* out_prob, float* out_score, void* stream);
/* grs_structural_decode: complete ordered bindings by port following
 * (model.py:391-478) for `count` candidates (sources < 0 are skipped);
 * bindings int64 [count, max_pattern] (-1 padded), valid uint8 [count];
 * clear_invalid sets sources[c] = -1 for invalid candidates.  Port arrays
 * int32 [B, slots, 4]; rule tables are the model's buffers. */
GRS_API int grs_structural_decode(const int64_t* types, const uint8_t* live, int slots,
                                  const int32_t* out_node, const int32_t* out_port,
                                  const int32_t* in_node, const int32_t* in_port,
                                  const int64_t* source_types, const int64_t* source_lengths,
                                  const int64_t* child, const int64_t* parent,
                                  const int64_t* parent_port, const int64_t* child_port,
                                  const int64_t* direction, const int64_t* pattern_edges,
                                  int max_edges, int max_pattern, const int64_t* batch_ids,
                                  int64_t* sources, const int64_t* anchors, int64_t count,
                                  int64_t* bindings, uint8_t* valid, int clear_invalid,
                                  void* stream);

/* ---- lazy topology: lazy_rollout_benchmark.py:105-485 and the accept loop
 * paged_rollout_benchmark.py:1013-1046 --------------------------------------
 * Per beam: types int64 [B, S] (-1 dead), port arrays out/in node/port int32
 * [B, S, 4] (-1 none), touch step int32 [B, S] (-1 never), previous-preferred
 * uint8 [B, S], rewrite distance int32 [B, S], next_slot/streak int32 [B],
 * gate count int64 [B], fingerprint uint64 [B] (XOR of splitmix64 node and
 * edge components).  `table` is the per-xfer rewrite table of width
 * grs_topology_table_width() built by the host from the patterns. */
GRS_API int grs_topology_table_width(void);
/* Plan every ranked proposal (rows/xfers/next_gate from grs_proposals_rank,
 * device count): validity and child fingerprint (plan_indexed_rewrite). */
GRS_API int grs_topology_plan(int64_t count_cap, const int64_t* count, const int64_t* rows,
                              const int64_t* xfers, const int64_t* next_gate,
                              const int64_t* cand_batch, const int64_t* cand_bindings,
                              int cand_pattern, const int32_t* table, const int64_t* types,
                              int32_t* out_node, int32_t* out_port, int32_t* in_node,
                              int32_t* in_port, int slots, const int32_t* next_slot,
                              const uint64_t* fingerprint, uint8_t* valid, uint64_t* fp_out,
                              int32_t* status, void* stream);
/* Accept loop: first occurrence by rank among valid, unseen fingerprints;
 * the first beam_size are accepted, inserted into the seen set and stably
 * sorted by next gate count into child_proposal.  summary int64 [6] =
 * accepted, attempted, invalid, duplicates, max child next slot, best
 * (smallest) child gate count; with rows == NULL the next-slot extent is not
 * computed (summary[4] = 0: a sharded search ranks records from several GPUs
 * and takes the extent from the gathered records instead).  Hash
 * tables are power-of-two open-addressing arrays (uint64 keys, 0 = empty). */
GRS_API int grs_topology_accept(int64_t count_cap, const int64_t* count, const uint8_t* valid,
                                const uint64_t* fp, const int64_t* next_gate, int beam_size,
                                uint64_t* step_keys, int32_t* step_first, int64_t step_capacity,
                                uint64_t* seen, int64_t seen_capacity, uint8_t* classes,
                                int64_t* child_proposal, int64_t* summary, const int64_t* rows,
                                const int64_t* xfers, const int64_t* cand_batch,
                                const int32_t* table, const int32_t* next_slot, int32_t* status,
                                void* stream);
GRS_API int grs_topology_seen_insert(const uint64_t* fp, int64_t n, uint64_t* seen,
                                     int64_t seen_capacity, int32_t* status, void* stream);
/* Build every accepted child (materialize_indexed_rewrite, dense_last_touched,
 * previous_preferred, local_streak, BFS rewrite distance) into the child
 * buffers (row stride `slots`, parents read with row stride `p_slots`) and
 * emit the per-child action tensors of the model advance. */
GRS_API int grs_topology_materialize(
    int max_children, const int64_t* child_proposal, const int64_t* summary, const int64_t* rows,
    const int64_t* xfers, const int64_t* next_gate, const uint64_t* fp, const int64_t* cand_batch,
    const int64_t* cand_anchor, const int64_t* cand_bindings, int cand_pattern,
    const int32_t* table, const int64_t* xfer_to_source, int p_slots, int slots,
    const int64_t* p_types, const int32_t* p_out_node, const int32_t* p_out_port, const int32_t* p_in_node,
    const int32_t* p_in_port, const int32_t* p_touched, const uint8_t* p_pref,
    const int32_t* p_next_slot, const int32_t* p_streak, int64_t* c_types, int32_t* c_out_node,
    int32_t* c_out_port, int32_t* c_in_node, int32_t* c_in_port, int32_t* c_touched,
    uint8_t* c_pref, int32_t* c_distance, int32_t* c_next_slot, int32_t* c_streak,
    int64_t* c_gate, uint64_t* c_fp, int64_t* a_parent, int64_t* a_xfer, int64_t* a_source,
    int64_t* a_src_slots, int src_pattern, int64_t* a_dst_slots, int64_t* a_dst_types,
    int dst_pattern, int depth, int32_t* status, void* stream);
/* XOR fingerprint of beam rows from their types and out-ports (indexed_topology). */
GRS_API int grs_topology_fingerprint(const int64_t* types, const int32_t* out_node,
                                     const int32_t* out_port, const int32_t* in_node,
                                     const int32_t* in_port, int batch, int slots, uint64_t* fp,
                                     void* stream);

/* ---- tensor-core GEMM with a fused epilogue (sm_100a tcgen05) -------------
 * out[M, N] = (A[M, K] . B[N, K]^T (+ bias[N])) then GELU when `gelu`, bf16 in
 * and out, fp32 accumulation: the readout graph layers' u0 projection and its
 * GELU (paged_model.py:381-436, model.py:26-53) in one pass.  A row-major with
 * row stride lda, B K-major (a Linear weight [out, in]) with row stride ldb,
 * out row stride ldo (elements).  Requires K % 64 == 0, N % 256 == 0, strides
 * multiples of 8 elements and 16-byte aligned pointers; GRS_ERR_SHAPE
 * otherwise (the caller then uses a library GEMM).  `status` (device int32,
 * may be null) receives GRS_ERR_TIMEOUT if an in-kernel wait gives up. */
GRS_API int grs_gemm_bf16_epilogue(const void* a, int64_t lda, const void* b, int64_t ldb, int M,
                                   int N, int K, const float* bias, int gelu, void* out,
                                   int64_t ldo, int32_t* status, void* stream);
/* The general form of the tensor-core GEMM used for every bf16 projection of
 * the paged action model (paged_model.py:36-94, 213-241, 338-436, 513-604;
 * model.py:26-53): out = (A . B^T (+ bias) (+ residual)) then GELU when
 * `gelu`, rows with zero_row[r] == 0 written as zeros (the residual + dead-row
 * mask is the readout graph output's add, paged_model.py:434-436).  N a
 * multiple of 128, K of 64; residual bf16 [M, N] with row stride ldr, or
 * null; zero_row may be null.  GRS_ERR_SHAPE for shapes or alignments the
 * kernel does not take (nothing launched). */
GRS_API int grs_gemm_bf16(const void* a, int64_t lda, const void* b, int64_t ldb, int M, int N,
                          int K, const float* bias, int gelu, const void* residual, int64_t ldr,
                          const uint8_t* zero_row, void* out, int64_t ldo, int32_t* status,
                          void* stream);
/* The same tensor-core GEMM with N = 256 and a residual + LayerNorm epilogue
 * (the readout graph layers' u2 projection and their add+LayerNorm,
 * model.py:26-53):  s = residual[M, 256] + A . B^T + bias;  out = (s - mean(s))
 * / sqrt(var(s) + eps) * gamma + beta, rows with zero_row[r] == 0 written as
 * zeros (zero_row may be null).  fp32 statistics, two-pass variance; bias,
 * gamma, beta fp32 [256]; residual bf16 with row stride ldr.  GRS_ERR_SHAPE
 * for shapes or alignments the kernel does not take. */
GRS_API int grs_gemm_bf16_layernorm(const void* a, int64_t lda, const void* b, int64_t ldb, int M,
                                    int K, const float* bias, const void* residual, int64_t ldr,
                                    const float* gamma, const float* beta, const uint8_t* zero_row,
                                    float eps, void* out, int64_t ldo, int32_t* status,
                                    void* stream);
/* grs_gemm_bf16_layernorm with N = 256 or 128 and the masks of the model's
 * other add+LayerNorm passes: s = residual + row_scale[r] * (A . B^T + bias) (row_scale may be
 * null: 1), rows whose where_row[r], where_beam[r / rows_per_beam] is 0 or
 * whose where_len[r / rows_per_beam] <= 0 keep the residual unchanged, rows
 * with zero_row[r] == 0 are zeroed (each mask may be null).  These are the
 * node readout's output projection + norm (paged_model.py:373-379: rows of
 * beams with no action history keep their state) and the live-node update's
 * action_delta output + norm (paged_model.py:236-241: the update scaled by
 * the affinity, only live slots of active beams change). */
GRS_API int grs_gemm_bf16_layernorm_ex(const void* a, int64_t lda, const void* b, int64_t ldb,
                                       int M, int N, int K, const float* bias,
                                       const float* row_scale,
                                       const void* residual, int64_t ldr, const float* gamma,
                                       const float* beta, const uint8_t* zero_row,
                                       const uint8_t* where_row, const uint8_t* where_beam,
                                       const int32_t* where_len, int rows_per_beam, float eps,
                                       void* out, int64_t ldo, int32_t* status, void* stream);
/* One InitialGraphLayer update on the tensor cores, width 256 (model.py:26-53):
 * out = LayerNorm(residual + GELU(A . U0^T + b0) . U2^T + b2) * gamma + beta,
 * rows with zero_row[r] == 0 zeroed.  A = [states | aggregated messages] bf16
 * [M, 512] (row stride lda), U0 [512, 512] and U2 [256, 512] K-major bf16,
 * b0 [512], b2, gamma, beta [256] fp32, residual bf16 [M, 256] (the states:
 * usually the first 256 columns of A), out bf16 [M, 256].  The [M, 512] GELU
 * activation stays in shared memory: one launch, no intermediate tensor.
 * GRS_ERR_SHAPE for strides or alignments the kernel does not take. */
GRS_API int grs_graph_mlp_bf16(const void* a, int64_t lda, const void* u0, int64_t ldu0,
                               const float* b0, const void* u2, int64_t ldu2, const float* b2,
                               int M, const void* residual, int64_t ldr, const float* gamma,
                               const float* beta, const uint8_t* zero_row, float eps, void* out,
                               int64_t ldo, int32_t* status, void* stream);
/* Match logits on the tensor cores (model.py:375-389): logits[r, v] =
 * (x[r] . w[v]) * scale + bias[v] where the slot is live and its gate type
 * equals first_types[v], else -1e4; eligible[r, v] the same condition.  w is
 * the bf16 product of the source vectors and the retrieval_node weight
 * ([32, K], rows >= num_sources zero), so the node projection and the
 * source product are one GEMM with N = 32; num_sources <= 32, K % 64 == 0;
 * live uint8 [M], types int64 [M], logits fp32 [M, num_sources], eligible
 * uint8 [M, num_sources]. */
GRS_API int grs_match_logits_bf16(const void* x, int64_t ldx, const void* w, int64_t ldw, int M,
                                  int K, int num_sources, const float* bias,
                                  const int64_t* first_types, const uint8_t* live,
                                  const int64_t* types, float scale, float* logits,
                                  uint8_t* eligible, int32_t* status, void* stream);

/* ---- beam search sharded over the GPUs of a node ---------------------------
 * The reference ranks a level's proposals globally
 * (paged_rollout_benchmark.py:967-1005) and accepts in that order
 * (:1013-1046) on one GPU.  Sharded, every GPU ranks its own beams and packs
 * the ranked list into records (int64, field-major: KEY1, KEY2, FP, AUX rows
 * of `width`, then 4 metrics: ranked count, predicted, eligible, allocated
 * pages).  KEY1 = next_gate << 44 | (0xffffffff - prob_bits) << 12 |
 * parent_gate, KEY2 = global_parent << 27 | xfer << 11 | candidate row within
 * the parent, AUX = child next slot | valid << 32; rows past the ranked count
 * have KEY1 = INT64_MAX.  Lexicographic (KEY1, KEY2) order is the reference
 * ranking order.  Fields that overflow their bits flag GRS_ERR_TOO_LARGE. */
GRS_API int grs_shard_records(int64_t width, const int64_t* count, const int64_t* rows,
                              const int64_t* xfers, const int64_t* next_gate, const float* probs,
                              const int64_t* cand_batch, int64_t k, const int64_t* gate,
                              const int64_t* global_index, const int32_t* next_slot,
                              const int32_t* table, const uint8_t* valid, const int64_t* fp,
                              const int64_t* ranked_metrics, const int32_t* free_count,
                              int64_t capacity, int64_t* out, int32_t* status, void* stream);
/* Merge `world` gathered record blocks (block r at gathered + r * stride, each
 * sorted) into the first `cap` (<= world * width) records of the global
 * ranking: valid (uint8), fp, next gate, source GPU, index in its source
 * list and child next slot per merged position; rows past the merged count
 * are zero with source = world.  count[0] = min(cap, records present),
 * metrics[4] = the summed metrics.  An unsorted block flags GRS_ERR_ORDER. */
GRS_API int grs_shard_merge(const int64_t* gathered, int world, int64_t width, int64_t stride,
                            int64_t cap, int64_t* count, int64_t* metrics, uint8_t* valid,
                            int64_t* fp, int64_t* next_gate, int64_t* src, int64_t* index,
                            int64_t* child_next, int32_t* status, void* stream);
/* Place the summary[0] accepted children (child_proposal: merged positions,
 * global order) on GPUs: each GPU keeps its own children up to an even share
 * (A / world, one more for the first A % world GPUs), the rest go in order to
 * the GPUs with room, lowest first.  Writes pairs[world * world] (children
 * moving from GPU s to d; diagonal: kept), extent[0] (largest child next
 * slot), and for GPU `me`: keep_local / keep_global (its kept children's
 * source-list index and global child index, global order), out_local (source
 * indices of its leaving children by destination, global order within) and
 * in_global (global indices of the children it receives by source GPU,
 * global order within).  world <= 64, beam_size <= 8192. */
GRS_API int grs_shard_route(const int64_t* child_proposal, const int64_t* summary,
                            const int64_t* src, const int64_t* index, const int64_t* child_next,
                            int64_t cap, int beam_size, int world, int me, int64_t* pairs,
                            int64_t* extent, int64_t* keep_local, int64_t* keep_global,
                            int64_t* out_local, int64_t* in_global, int32_t* status,
                            void* stream);
/* Multi-segment row copy (at most 40 segments).  `segments` is a HOST array
 * of 10 int64 words per segment: src address, src row stride, src unit
 * stride, src index address (0 = none), dst address, dst row stride, dst unit
 * stride, dst index address (0 = none), unit bytes, units per row.  Unit k of
 * row i is read from src + src_index[i * units + k] * src_unit_stride (or src
 * + i * src_row_stride + k * src_unit_stride without an index) and written
 * likewise.  Rows: min(*n_dev, n_max) when n_dev is given, else n_max.  Packs
 * the fields and cache pages of beams that change GPU into send rows,
 * unpacks received rows, and reorders beams, each in one launch. */
GRS_API int grs_rows_copy(int nseg, const int64_t* segments, const int64_t* n_dev,
                          int64_t n_max, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* GRS_B200_H */
