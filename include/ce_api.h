/*
 * ce_api.h -- C ABI of the B200 (sm_100a) decode-time KV eviction path.
 *
 * One shared library, libce_b200.so, exports these symbols.  Every pointer
 * argument is caller-owned DEVICE memory unless the comment says "host".
 * Every entry point:
 *   - enqueues its kernels on `stream` (a cudaStream_t passed as void*);
 *   - never synchronises the device and never allocates memory; scratch comes
 *     from the caller through (workspace, workspace_bytes), sized with the
 *     matching *_workspace_bytes() query;
 *   - returns CE_OK or a negative CE_ERR_* status for host-detectable errors
 *     (bad sizes, unsupported shapes, launch failures) and never throws;
 *   - reports data-dependent errors found on the device (an index outside the
 *     pool, a capacity overflow, a bounded wait that gave up) by OR-ing
 *     CE_EW_* bits into the optional device word `err` (may be NULL).
 *
 * Vocabulary (the reference's, at page granularity):
 *   unit      one KV page of `page_size` tokens (page_size 1 = the reference's
 *             token slots).  Pools hold [units, kv_heads, page_size, head_dim]
 *             bf16 per layer; at page_size 1 that is the reference's
 *             [slots, kv_heads, head_dim] (SGLang MHATokenToKVPool).
 *   row       a request row (SGLang req_pool_idx).
 *   table     [rows, width] compacted resident units of each row, shared by
 *             every layer and KV head (reference State.table).
 *   req_to_unit [rows, width] logical position (in units) -> pool unit
 *             (reference req_to_token).
 *   frontier  [rows] logical length (units) below which residents live in
 *             `table`; count [rows] = number of compacted residents.
 *   pos       [rows, layers, kv_heads, pos_cap] logical unit position that
 *             column c of `table` holds for (layer, head) (reference
 *             entry["pos"]).
 *   scores    [layers, kv_heads, pool_units] fp32 H2O scores, one per
 *             (layer, KV head, unit) (reference State.scores).
 *
 * Reference citations are file:line inside tonghuikang/cache-eviction,
 * e.g. code/cache_eviction/sglang_evict_runtime.py:136 (written
 * "runtime:136" below).
 */
#ifndef CE_API_H
#define CE_API_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes (return values) ------------------------------------- */
#define CE_OK               0
#define CE_ERR_ARG         -1   /* a size/pointer argument is invalid        */
#define CE_ERR_UNSUPPORTED -2   /* shape outside what the kernels implement  */
#define CE_ERR_CUDA        -3   /* a CUDA runtime call or launch failed      */
#define CE_ERR_WORKSPACE   -4   /* workspace smaller than the query returned */

/* ---- device error-word bits (OR-ed into *err) -------------------------- */
#define CE_EW_INDEX      0x01  /* a unit index outside [0, pool_units)           */
#define CE_EW_CAPACITY   0x02  /* a CSR / column / output capacity was exceeded  */
#define CE_EW_TIMEOUT    0x04  /* a bounded device wait gave up (kernel returned) */
#define CE_EW_MODE       0x08  /* a row's score mode had no workspace (flags)    */
#define CE_EW_PROTECTED  0x10  /* protected counts differ between heads          */
#define CE_EW_SWA        0x20  /* a freed unit still maps to a sliding-window slot */
#define CE_EW_PACK       0x40  /* packed ownership overlaps the sliding-window region */
#define CE_EW_SHAPE      0x80  /* per-row sizes inconsistent with the arguments  */

/* ---- policies (reference POLICIES, runtime:45-46, plus H2O global) ----- */
#define CE_POLICY_PREFIX_SLIDING 0  /* prefix_sliding_2048: keep exactly P u R   */
#define CE_POLICY_RANDOM         1  /* random_2048: caller-supplied uniforms      */
#define CE_POLICY_RESERVOIR      2  /* random_reservoir_2048: splitmix64 scores   */
#define CE_POLICY_HEAD_SUM       3  /* head_sum_2048: per-head score buffer       */
#define CE_POLICY_HEAD_MAX       4  /* head_max_sum_2048: per-head score buffer   */
#define CE_POLICY_H2O_GLOBAL     5  /* h2o_global_2048: sum of all KV heads' scores */

/* decode score modes per row (reference State.mode, runtime:45-46,162-164) */
#define CE_MODE_NONE 0
#define CE_MODE_SUM  1
#define CE_MODE_MAX  2

/* score / uniform element types */
#define CE_DTYPE_NONE 0
#define CE_DTYPE_F32  1
#define CE_DTYPE_F64  2
#define CE_DTYPE_BF16 3

/* per-boundary parameters, all in units (reference _boundary cfg + n + cursor,
 * runtime:415-437).  32 bytes, device array. */
typedef struct ce_row_params {
  int32_t n;        /* logical length at the boundary                         */
  int32_t budget;   /* retained units per (layer, head)                       */
  int32_t prefix;   /* protected prefix P                                     */
  int32_t recent;   /* protected recent window R                              */
  int32_t cursor;   /* sliding-window guard (pos >= cursor protected); -1 = none */
  int32_t policy;   /* CE_POLICY_*                                            */
  uint64_t seed;    /* reservoir seed (reference cfg["seed"])                 */
} ce_row_params;

/* ---- library info -------------------------------------------------------- */
const char* ce_version(void);
const char* ce_status_string(int status);
/* Detail of the last failing call made by this host thread. */
const char* ce_last_error(void);

/* Load the decode, selection / boundary, CSR and unit-pool kernels on the
 * current device and set their launch attributes, which their entry points
 * otherwise do on first use.  Under lazy module loading (the CUDA 12 default)
 * a first ce_boundary call spends ~5 ms loading its kernels; a server calls
 * this once per device at start-up so no decode step pays that.  Launches
 * nothing and allocates no workspace. */
int ce_prepare_device(void);

/* ---- K4: ragged CSR page table -------------------------------------------
 * Replaces gstar_evict.fill (runtime:136-152) and the two
 * create_flashinfer_kv_indices_triton launches it makes.  For batch entry b
 * (row = rows[b], L = seq_lens[b] tokens):
 *   kv_indptr[b+1] = kv_indptr[b] + count[row] + ceil(L/page) - frontier[row]
 *   kv_indices     = table[row, :count[row]] ++ req_to_unit[row, frontier:ceil(L/page)]
 *   kv_tokens[b]   = count[row]*page + L - frontier[row]*page  (valid tokens)
 * kv_indices is int32 or int64 (indices_i64).  Entries beyond kv_capacity are
 * dropped and flag CE_EW_CAPACITY. */
int ce_fill(const int32_t* table, int64_t table_stride,
            const int32_t* req_to_unit, int64_t r2u_stride,
            const int32_t* frontier, const int32_t* count,
            const int64_t* rows, const int64_t* seq_lens, int32_t bs,
            int32_t page_size,
            int32_t* kv_indptr, void* kv_indices, int32_t indices_i64,
            int64_t kv_capacity, int32_t* kv_tokens,
            int32_t* err, void* stream);

/* ---- unit pool of a continuous batch ---------------------------------------
 * A device-resident stack of free units, units[0 .. *top) (top: a device
 * int32), standing in for SGLang's token allocator on the decode path: the
 * new token's slot (alloc), a boundary's leftovers (allocator.free_full,
 * runtime:476-482) and a finished request's units (release, runtime:719-742).
 * Graph-capturable, no host sync; entries and rows are served in batch order,
 * so assignments are deterministic.
 *
 * ce_pool_alloc: for every batch entry b whose newest token (position
 * seq_lens[b] - 1) starts a unit, pop one unit and write it to
 * req_to_unit[rows[b], (seq_lens[b] - 1) / page_size].  An empty stack (or a
 * slot at or beyond r2u_width) flags CE_EW_CAPACITY and writes unit 0 there. */
int ce_pool_alloc(int32_t* units, int32_t* top, int32_t* req_to_unit, int64_t r2u_stride,
                  int64_t r2u_width, const int64_t* rows, const int64_t* seq_lens, int32_t bs,
                  int32_t page_size, int32_t* err, void* stream);

/* ce_pool_push: push lists[r * list_stride .. + counts[r * count_stride]) for
 * r = 0 .. nrows-1, in row order, onto the stack (capacity entries).  A list
 * longer than list_stride flags CE_EW_SHAPE and is skipped; units beyond the
 * capacity flag CE_EW_CAPACITY.  ce_boundary's freed / result arrays can be
 * passed directly (counts = result + 3, count_stride = 4). */
int ce_pool_push(int32_t* units, int32_t* top, int64_t capacity, const int32_t* lists,
                 int64_t list_stride, const int32_t* counts, int64_t count_stride, int32_t nrows,
                 int32_t* err, void* stream);

/* ---- K1: fused paged GQA decode attention + H2O score --------------------
 * Replaces SGLang decode_attention_fwd (stage 1 + stage 2, call shape
 * code/tests/test_sglang_evict.py:59-61) AND gstar_evict.after_decode /
 * _decode_scores (runtime:155-224) with one pass over K and V.
 *   q       [bs, H, 64] bf16 (strides q_sb, q_sh in elements, last dim dense)
 *   k_pool, v_pool  one layer, [pool_units, G, page_size, 64] bf16, dense
 *   kv_indptr/kv_indices/kv_tokens  the CSR from ce_fill (int32 indices)
 *   sinks   [H] fp32 natural-log sink logits, or NULL (no sink)
 *   mode_of_row [rows] CE_MODE_* and rows [bs] (mode = mode_of_row[rows[b]]);
 *           mode_of_row NULL = no scores for any row
 *   scores  [G, pool_units] fp32 of this layer (stride score_sg), receives
 *           per unit: CE_MODE_SUM  sum over tokens in the unit and over the
 *           group's query heads of p;  CE_MODE_MAX  sum over tokens of the
 *           max over the group's query heads of p, where
 *           p = exp(scale*q.k - logsumexp(all logits, sink)).
 *   zero_new  1: a unit whose first token is the newest token of the row is
 *           overwritten instead of accumulated (the reference zeroes the new
 *           slot's score first, runtime:211-212)
 *   out     [bs, H, 64] bf16 (out_f32 = 0) or fp32 (out_f32 = 1)
 *   lse_out [bs, H] fp32 natural-log normalizer incl. sink, or NULL
 *   score_flags bit0: CE_MODE_SUM rows may occur, bit1: CE_MODE_MAX rows may
 *           occur (sizes the workspace; a row whose mode has no workspace
 *           flags CE_EW_MODE and gets no score); CE_SCORE_DEFER: compute the
 *           outputs and lse only, leave the scores to ce_decode_scores
 * Supported: head_dim 64, H/G == 8, page_size 1 (G == 8) or 16 (any G). */
#define CE_SCORE_DEFER 4
int64_t ce_decode_workspace_bytes(int32_t bs, int64_t kv_capacity,
                                  int32_t num_q_heads, int32_t num_kv_heads,
                                  int32_t page_size, int32_t score_flags);
int ce_decode_attn_score(const void* q, int64_t q_sb, int64_t q_sh,
                         const void* k_pool, const void* v_pool, int64_t pool_units,
                         const int32_t* kv_indptr, const int32_t* kv_indices,
                         const int32_t* kv_tokens, int64_t kv_capacity,
                         const float* sinks,
                         const int32_t* mode_of_row, const int64_t* rows,
                         float sm_scale, int32_t bs, int32_t num_q_heads,
                         int32_t num_kv_heads, int32_t head_dim, int32_t page_size,
                         float* scores, int64_t score_sg, int32_t zero_new,
                         void* out, int32_t out_f32, int64_t o_sb, int64_t o_sh,
                         float* lse_out, int32_t score_flags,
                         void* workspace, int64_t workspace_bytes,
                         int32_t* err, void* stream);

/* ---- K1's score part, deferred ----------------------------------------------
 * After ce_decode_attn_score(..., score_flags | CE_SCORE_DEFER, workspace, ...)
 * adds the H2O page masses that call left out, from the normalisers and
 * per-page log-masses it kept in its workspace.  The arguments are that
 * call's (the same CSR, rows, modes, scores, score_flags and workspace), and
 * the two calls must be ordered (same stream, or an event between streams);
 * the CSR and the workspace must not be rewritten before this call has run.
 * The scores equal those of the undeferred call bit for bit.  No reference
 * counterpart: it lets a layer's page scoring run on a second stream beside
 * the next layer's attention. */
int ce_decode_scores(const int32_t* kv_indptr, const int32_t* kv_indices,
                     const int32_t* kv_tokens, int64_t kv_capacity, int64_t pool_units,
                     const int32_t* mode_of_row, const int64_t* rows, int32_t bs,
                     int32_t num_q_heads, int32_t num_kv_heads, int32_t page_size,
                     float* scores, int64_t score_sg, int32_t zero_new, int32_t score_flags,
                     const void* workspace, int64_t workspace_bytes, int32_t* err,
                     void* stream);

/* ---- K1 without a caller workspace ------------------------------------------
 * No counterpart in the reference.  For callers that cannot allocate device
 * memory when they decode (an engine that gave all HBM to its KV pool, a host
 * that forbids allocations after start-up, a global-mode graph capture):
 * identical to ce_decode_attn_score except that its scratch is a static
 * device array of CE_DECODE_STATIC_SCRATCH_BYTES inside the library, and that
 * CE_SCORE_DEFER is refused (CE_ERR_ARG).
 *   - Set-up: the first call on a device (and the first after cudaDeviceReset
 *     replaced its context) looks up the array's device address
 *     (cudaGetSymbolAddress) and loads the decode kernels.  A call with
 *     bs == 0 does only this and launches nothing.  Under lazy module loading
 *     (the CUDA 12 default) the array's 32 MiB are placed on the device at
 *     this point, so make the set-up call before handing the rest of HBM to a
 *     pool, and before any stream capture; the array then stays until the
 *     process exits (with eager loading it is placed when the context is
 *     created).  Calls after the set-up take no device memory.
 *   - A call whose ce_decode_workspace_bytes() exceeds the maximum returns
 *     CE_ERR_WORKSPACE and launches nothing.
 *   - Every call on a device shares the one array: calls that may overlap on
 *     the GPU (different streams without ordering) race and must be
 *     serialised by the caller.  No part of the array needs to start at zero.
 * Allocates nothing (no cudaMalloc/cudaFree, no allocating library call). */
#define CE_DECODE_STATIC_SCRATCH_BYTES (32u << 20)
int ce_decode_attn_score_static(const void* q, int64_t q_sb, int64_t q_sh,
                                const void* k_pool, const void* v_pool, int64_t pool_units,
                                const int32_t* kv_indptr, const int32_t* kv_indices,
                                const int32_t* kv_tokens, int64_t kv_capacity,
                                const float* sinks,
                                const int32_t* mode_of_row, const int64_t* rows,
                                float sm_scale, int32_t bs, int32_t num_q_heads,
                                int32_t num_kv_heads, int32_t head_dim, int32_t page_size,
                                float* scores, int64_t score_sg, int32_t zero_new,
                                void* out, int32_t out_f32, int64_t o_sb, int64_t o_sh,
                                float* lse_out, int32_t score_flags,
                                int32_t* err, void* stream);

/* ---- K5: prefill / extend H2O scores --------------------------------------
 * Replaces the scoring in gstar_evict.after_extend (runtime:277-311):
 * _prefill_scores with _probabilities (runtime:314-340), for a ragged batch
 * of extend chunks of one layer.
 *   q       [total_q, H, 64] bf16 (strides q_st, q_sh in elements, multiples
 *           of 8; last dim dense); entry b's chunk is rows
 *           qo_indptr[b] .. qo_indptr[b+1]  (nq_b queries)
 *   k_pool  [pool_units, G, page_size, 64] bf16 of this layer, dense
 *   kv_indptr/kv_indices/kv_tokens  entry b's key list: units
 *           kv_indices[kv_indptr[b] ..] holding kv_tokens[b] tokens, the
 *           resident prefix then the chunk's own tokens (the reference's
 *           prefix ++ new slots, runtime:330); kv_tokens[b] >= nq_b and the
 *           list has at least ceil(kv_tokens[b] / page_size) entries below
 *           kv_capacity
 *   mask    list token t is visible to chunk query i iff
 *           t <= kv_tokens[b] - nq_b + i  (key_pos > query_pos masked,
 *           runtime:334-336)
 *   sinks   [H] fp32 natural-log sink logits, or NULL
 *   mode_of_row, rows  as for ce_decode_attn_score (rows NULL: mode_of_row
 *           is indexed by b); entries whose mode is not SUM/MAX are skipped
 *   scores  [G, pool_units] fp32 of this layer (stride score_sg): per unit
 *           += sum over its tokens of sum over the chunk's queries of
 *           (sum (SUM) or max (MAX) over the group's query heads of p),
 *           p = exp(scale*q.k - logaddexp(logsumexp(visible logits), sink));
 *           zero_new 1: a unit whose first token is one of the chunk's is
 *           written instead of accumulated (the reference zeroes new slots
 *           first, runtime:293-294)
 *   total_q  rows of q (workspace size); max_q, max_tokens  host bounds on
 *           nq_b and kv_tokens[b] (grid sizes); an entry above either, or
 *           with ranges outside total_q / kv_capacity, flags CE_EW_SHAPE
 *           and is skipped
 * Supported: head_dim 64, H == 8*G, page_size dividing 64, sm_scale > 0.
 * No scratch beyond the workspace ([total_q, H] fp32 row normalizers). */
int64_t ce_prefill_workspace_bytes(int32_t total_q, int32_t num_q_heads);
int ce_prefill_scores(const void* q, int64_t q_st, int64_t q_sh,
                      const void* k_pool, int64_t pool_units,
                      const int32_t* qo_indptr, const int32_t* kv_indptr,
                      const int32_t* kv_indices, const int32_t* kv_tokens,
                      int64_t kv_capacity, const float* sinks,
                      const int32_t* mode_of_row, const int64_t* rows,
                      float sm_scale, int32_t bs, int32_t num_q_heads,
                      int32_t num_kv_heads, int32_t head_dim, int32_t page_size,
                      int32_t total_q, int32_t max_q, int32_t max_tokens,
                      float* scores, int64_t score_sg, int32_t zero_new,
                      void* workspace, int64_t workspace_bytes,
                      int32_t* err, void* stream);

/* ---- K5 variant: lost-mass diagnostic --------------------------------------
 * The reference's regret diagnostic (_diagnose, runtime:587-613): for ONE
 * entry's prefill chunk (qo_indptr/kv_indptr/kv_indices/kv_tokens as for
 * ce_prefill_scores, bs = 1, all keys visible to the causal mask) and
 * S <= 8 eviction specs, lost[s][i] += lost_scale * sum over the group's query
 * heads h and the keys t the spec evicted for head g of
 *   p = exp(scale*q_i,h . k_t - logaddexp(logsumexp(visible logits), sink_h)).
 * evicted_bits [S][G][bits_words] uint32, bit t set = key t evicted by spec s
 * for KV head g (bits_words * 32 >= max_tokens); lost [S][lost_stride] fp32
 * (lost_stride >= max_q), accumulated (atomically, over calls and KV heads).
 * The reference averages over query heads and layers: lost_scale =
 * 1 / (H * full layers).  Same workspace and shapes as ce_prefill_scores. */
int ce_prefill_lost(const void* q, int64_t q_st, int64_t q_sh,
                    const void* k_pool, int64_t pool_units,
                    const int32_t* qo_indptr, const int32_t* kv_indptr,
                    const int32_t* kv_indices, const int32_t* kv_tokens,
                    int64_t kv_capacity, const float* sinks, float sm_scale,
                    int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                    int32_t page_size, int32_t total_q, int32_t max_q, int32_t max_tokens,
                    const uint32_t* evicted_bits, int32_t num_specs, int64_t bits_words,
                    float* lost, int64_t lost_stride, float lost_scale,
                    void* workspace, int64_t workspace_bytes,
                    int32_t* err, void* stream);

/* ---- K5 variant: replay layer error ---------------------------------------
 * Replaces the reference's _replay_layer_difference (runtime:520-546) with
 * _visible (241-247): one prefill chunk of one request, queries at logical
 * positions start .. start+count-1 attending causally to the unevicted
 * keys/values 0 .. start+count-1 kept by position (the reference's shadow,
 * 227-238).  With a_i the full attention output of query i and b_i the
 * output restricted to each KV head's visible positions (both with the sink
 * in the normaliser),
 *   error[i] = ||b_i - a_i|| / max(||a_i||, 1e-12)   over all H x 64 values.
 *   q          [count, H, 64] bf16, strides q_st, q_sh (elements, multiples of 8)
 *   k, v       [kv_rows, G, 64] bf16 by position, kv_rows >= start + count
 *   visible    [G, bits_words] uint32, bit t of row g = position t visible to
 *              KV head g (bits_words * 32 >= start + count); NULL = all visible
 *   error      [count] fp32, written
 *   out_masked NULL or [count, H, 64] fp32: b (the masked output), written
 * Workspace: ce_replay_workspace_bytes(count, H). */
int64_t ce_replay_workspace_bytes(int32_t count, int32_t num_q_heads);
int ce_replay_error(const void* q, int64_t q_st, int64_t q_sh,
                    const void* k, const void* v, int64_t kv_rows,
                    const uint32_t* visible, int64_t bits_words,
                    const float* sinks, float sm_scale,
                    int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                    int32_t start, int32_t count, float* error, float* out_masked,
                    void* workspace, int64_t workspace_bytes,
                    int32_t* err, void* stream);

/* ---- K2: ragged per-head selection ---------------------------------------
 * Replaces gstar_evict.choose + _scores + reservoir_scores (runtime:358-412)
 * for `problems` independent boundaries, each over `segs` = layers*heads
 * segments of up to n_cols columns (ncols[i] valid, NULL = all):
 *   pos    [problems, segs, n_cols] int32 logical unit positions (unique per segment)
 *   score  [problems, segs, n_cols] f32/f64 (score_dtype) or NULL; ignored by
 *          prefix_sliding and reservoir; for h2o_global the key of (l, g, c) is
 *          the fp32 sum over the layer's heads in ascending head order
 *   params [problems] ce_row_params
 * protected = pos < prefix | pos >= n - recent | (cursor >= 0 & pos >= cursor);
 * the rest of the budget goes to the largest keys, ties to the larger pos.
 * Every position must lie in [0, max_n) with max_n >= every problem's n.
 * Outputs: kept [problems, segs, kept_stride] columns of the kept set sorted
 * by ascending pos (min(budget, ncols) of them; the protected count for
 * prefix_sliding); status [problems]: 0 chosen, 2 deferred (protected >
 * budget, kept not written), 3 protected counts differ between heads;
 * protected_count [problems]. */
int64_t ce_choose_workspace_bytes(int32_t problems, int32_t segs, int32_t n_cols);
int ce_choose(const int32_t* pos, const int32_t* ncols, int32_t n_cols,
              const void* score, int32_t score_dtype,
              const ce_row_params* params, int32_t problems, int32_t max_n,
              int32_t layers, int32_t heads, int32_t head_offset,
              int32_t* kept, int32_t kept_stride, int32_t* status,
              int32_t* protected_count,
              void* workspace, int64_t workspace_bytes,
              int32_t* err, void* stream);

/* ---- K2+K3: one eviction boundary for a batch of rows --------------------
 * Replaces gstar_evict._boundary (runtime:415-507): choose per (layer, KV
 * head), move every head's j-th middle survivor (ascending pos) into the j-th
 * non-protected candidate unit for K, V and scores of every layer, write
 * table/count/frontier/pos; when live != 0 also zero the leftover units'
 * scores, pack the req_to_unit row (runtime:476-491) and return the leftover
 * units in candidate order for the caller's allocator (free_full).
 *   k_layers/v_layers  device arrays [layers] of pool base addresses (uint64)
 *   marks   [pool_units] int32 scratch owned by the caller (zero-initialised
 *           once); epoch >= 1 must grow by one per call (the call tags real
 *           slots with epoch and freed units with -epoch)
 *   swa_mapping [pool_units] int64 or NULL (reference
 *           allocator.full_to_swa_index_mapping, runtime:477-479)
 *   uniforms [num_rows, layers, heads, max_cols] f32/f64 for random rows
 *           (a random row without them gets status 6)
 *   global_scores [num_rows, layers, global_heads, max_cols] fp32 or NULL:
 *           dense per-column scores of ALL KV heads (tensor-parallel ranks
 *           all-gather them); when NULL h2o_global sums the local heads
 *   max_cols >= count[row] + n - frontier[row] for every row
 *   max_width >= every row's middle width (budget - protected; <= 0 means
 *            max_cols): sizes the relocation scratch and the item space
 *   max_n    >= every row's n (positions are ranked in a max_n-bit bitmap)
 *   result  [num_rows, 4]: status (0 evicted, 1 nothing to do, 2 deferred,
 *           3 protected mismatch, 4 packing error, 5 sliding-window error,
 *           6 row sizes outside max_cols/max_n/pos_cap, or no uniforms for a
 *           random row), columns before,
 *           residents after (the protected count when deferred), units freed
 *   freed_units [num_rows, freed_stride] leftover units (live only)
 *   record_delta, record_counts  retention record (runtime:465-467, 500-507),
 *           or NULL: for every evicted row and (layer, head) the positions of
 *           the columns this boundary evicts, ascending and delta-coded (the
 *           first value is the position itself), at
 *           record_delta[(row * layers + layer) * kv_heads + head][...]
 *           (row stride record_stride >= max_cols), and their number in
 *           record_counts[(row * layers + layer) * kv_heads + head] (0 for
 *           rows that did not evict)
 * hazard_bytes bounds the relocation scratch; rows and layers are processed
 * in groups that fit it (at least one row of one layer, the minimum). */
int64_t ce_boundary_workspace_bytes(int32_t num_rows, int32_t layers, int32_t kv_heads,
                                    int32_t head_dim, int32_t page_size,
                                    int32_t max_cols, int32_t max_width,
                                    int32_t global_heads, int64_t hazard_bytes);
int ce_boundary(int32_t* table, int64_t table_stride, int32_t table_width,
                int32_t* req_to_unit, int64_t r2u_stride, int32_t r2u_width,
                int32_t* frontier, int32_t* count,
                int32_t* pos, int64_t pos_row_stride, int32_t pos_cap,
                float* scores, int64_t score_layer_stride, int64_t score_head_stride,
                int64_t pool_units,
                const uint64_t* k_layers, const uint64_t* v_layers,
                int32_t layers, int32_t kv_heads, int32_t head_dim, int32_t page_size,
                int32_t head_offset,
                int32_t* marks, int32_t epoch, const int64_t* swa_mapping,
                const int32_t* rows, const ce_row_params* params, int32_t num_rows,
                const void* uniforms, int32_t uniform_dtype,
                const float* global_scores, int32_t global_heads,
                int32_t live, int32_t max_cols, int32_t max_width, int32_t max_n,
                int32_t* result, int32_t* freed_units, int64_t freed_stride,
                void* workspace, int64_t workspace_bytes, int64_t hazard_bytes,
                uint32_t* record_delta, int64_t record_stride, int32_t* record_counts,
                int32_t* err, void* stream);

/* Dense per-column scores of the boundary rows, [num_rows, layers, heads,
 * max_cols] fp32 (zero beyond each row's columns), for the tensor-parallel
 * all-gather that h2o_global needs before ce_boundary. */
int ce_gather_row_scores(const int32_t* table, int64_t table_stride,
                         const int32_t* req_to_unit, int64_t r2u_stride,
                         const int32_t* frontier, const int32_t* count,
                         const float* scores, int64_t score_layer_stride,
                         int64_t score_head_stride, int64_t pool_units,
                         int32_t layers, int32_t kv_heads,
                         const int32_t* rows, const ce_row_params* params,
                         int32_t num_rows, int32_t max_cols, float* out,
                         int32_t* err, void* stream);

/* reservoir_scores (runtime:358-373) / core.reservoir_score (core.py:23-30):
 * out[l, g, c] = splitmix64(seed, l, head_offset + g, pos[l, g, c]) >> 11 as
 * the 53-bit integer (divide by 2^53 for the reference's double). */
int ce_reservoir_scores(const int32_t* pos, int32_t layers, int32_t heads,
                        int32_t n_cols, int32_t head_offset, uint64_t seed,
                        uint64_t* out, void* stream);

/* ---- self-test of the bounded device waits --------------------------------
 * Every pipelined kernel waits on mbarrier phases with a bound (2 s): a wait
 * that runs out flags CE_EW_TIMEOUT, tells the CTA's other warps to stop and
 * lets the kernel return.  This entry point runs that machinery alone: with
 * complete = 0 one warp waits limit_ns ([1 us, 2 s]) on a phase nothing
 * completes and a second warp waits on the same phase polling the abort flag;
 * status [3] int32 (device) receives {first wait gave up, second left through
 * the abort, block reached its end}.  With complete = 1 the phase completes
 * and status = {0, 0, 1}.  No reference counterpart. */
int ce_selftest_wait(int32_t complete, int64_t limit_ns, int32_t* err, int32_t* status, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* CE_API_H */
