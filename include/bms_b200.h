/*
 * bms_b200.h -- C ABI of the B200 (sm_100a) masked-selection library.
 *
 * Drop-in boundary for the native module of karthikeyansura/bitmask-speculation
 * (csrc/bindings.cpp:10-17 exports runtime_version, mask_count, masked_argmax,
 * masked_reduce_batch and masked_sample).  Every entry point takes plain device
 * pointers and sizes, no framework types:
 *
 *   - inputs are read-only; outputs are caller-allocated device buffers that the
 *     call overwrites (the library allocates no device or host memory);
 *   - work is enqueued on `stream` (a cudaStream_t; NULL = legacy default
 *     stream) of CUDA device `device`; nothing synchronises with the host;
 *   - every pointer must be device (or managed) memory of `device`, checked with
 *     cudaPointerGetAttributes before anything is launched;
 *   - contract violations return a nonzero BMS_ERROR_* code with a message from
 *     bms_last_error() (thread-local) and launch nothing; row-level data errors
 *     (empty mask, NaN, ...) are reported per row through the status outputs,
 *     exactly like the reference's device status codes (csrc/sample.cu:24-25).
 *
 * Masks are packed int32 words, token t allowed iff bit (t % 32) of word t / 32
 * is set; bits at or beyond the vocabulary are ignored.  Logits are float32,
 * bfloat16 or float16 (the reference accepted float32 only, csrc/checks.h:21).
 */
#ifndef BMS_B200_H
#define BMS_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define BMS_API __attribute__((visibility("default")))
#else
#define BMS_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Logit element types. */
enum { BMS_FLOAT32 = 0, BMS_BFLOAT16 = 1, BMS_FLOAT16 = 2 };

/* Return codes of the entry points. */
enum {
    BMS_SUCCESS = 0,
    BMS_ERROR_INVALID_ARGUMENT = 1, /* the reference raised RuntimeError (TORCH_CHECK) */
    BMS_ERROR_CUDA = 2,             /* a CUDA runtime call or launch failed */
    BMS_ERROR_UNSUPPORTED = 3       /* valid input beyond a documented limit */
};

/* Per-row status codes written by the kernels (csrc/sample.cu:24-25, argmax.cu:77). */
enum {
    BMS_STATUS_OK = 0,
    BMS_STATUS_EMPTY = 1,       /* mask has no valid token */
    BMS_STATUS_NAN = 2,         /* a logit of the row is NaN (valid or not) */
    BMS_STATUS_BAD_UNIFORM = 3, /* sampler uniform not in [0, 1) */
    BMS_STATUS_NO_MASS = 4,     /* every valid logit is -inf (sampler) */
    BMS_STATUS_POS_INF = 5,     /* a valid logit is +inf (sampler) */
    BMS_STATUS_BAD_LENGTH = 6,  /* verification: proposal count outside [0, K] */
    BMS_STATUS_TIMEOUT = 7,     /* a bounded device wait expired; row result undefined */
    BMS_STATUS_BAD_MASK_ROW = 8 /* verification with a mask table: index outside the table */
};

/* Draft budget policy.  kind 0: decoding/scheduling.py:21-46 DensityPolicy
 * (density < low -> max; < high -> (min + max) / 2; else min).  kind 1: linear
 * (density < low -> max; > high -> min; else max - floor((max - min) *
 * ((density - low) / (high - low))), all in IEEE double).  density is
 * count / vocab, correctly rounded. */
typedef struct bms_policy {
    int32_t kind;
    int32_t min_budget;
    int32_t max_budget;
    int32_t reserved;
    double low_density;
    double high_density;
} bms_policy;

/* Message of the last failed call on this thread ("" if none). */
BMS_API const char *bms_last_error(void);

/* Replaces csrc/runtime.cu:4-8 cuda_runtime_version. */
BMS_API int bms_runtime_version(int32_t *version);

/* Replaces csrc/popcount.cu:28-37 mask_count_cuda: *count = number of allowed
 * tokens in one row of ceil(vocab / 32) words (count is a device int64). */
BMS_API int bms_mask_count(const int32_t *mask, int64_t vocab, int64_t *count, int32_t device, void *stream);

/* Replaces csrc/argmax.cu:117-125 masked_argmax_cuda: lowest-index valid
 * maximum of one row; *token = -1 unless *status == BMS_STATUS_OK. */
BMS_API int bms_masked_argmax(const void *logits, int32_t dtype, const int32_t *mask, int64_t vocab,
                      int64_t *token, int32_t *status, int32_t device, void *stream);

/* Workspace of the batched entry points' dynamic and flat schedules (no reference counterpart):
 * bytes for `device` (-1 if invalid; about 11 MB on a 148-SM B200).  A workspace is device memory
 * of at least this size, 256-byte aligned, zeroed once before its first use; every call leaves it
 * ready for the next.  Calls that may run concurrently (different streams) need different
 * workspaces.  With a workspace, rows of at most 64 chunks (8,192 tokens per chunk for 16-bit
 * logits, 4,096 for float32) are handed to CTAs dynamically and the last rows are split across
 * CTAs; small sampler batches (fewer than 1.5 rows per resident CTA) stream as chunk blocks taken
 * by every CTA, followed by a second launch that merges each row.  Without a workspace (NULL),
 * each group of CTAs owns a fixed block of rows. */
BMS_API int64_t bms_workspace_bytes(int32_t device);

/* Replaces csrc/argmax.cu:127-137 masked_reduce_batch_cuda: per row of a
 * contiguous [rows, vocab] logits / [rows, ceil(vocab/32)] mask batch, the
 * masked argmax, the valid count and a status.  `counts` may be NULL; `workspace`
 * may be NULL (see bms_workspace_bytes).  No row limit (the reference stopped at
 * 65,535 rows, csrc/checks.h:36). */
BMS_API int bms_masked_reduce_batch(const void *logits, int32_t dtype, const int32_t *masks, int64_t rows,
                            int64_t vocab, int64_t *tokens, int64_t *counts, int32_t *status,
                            void *workspace, int64_t workspace_bytes, int32_t device, void *stream);

/* bms_masked_reduce_batch on the dynamic schedule with a workspace that is a file-scope device
 * array (about 1.8 MB per device, held until the process exits) instead of caller memory: the call
 * allocates nothing, for callers that may not allocate device memory (an engine whose allocator
 * owns the free HBM, a binding without a device allocator).  No reference counterpart.  Rows of at most 64 chunks (524,288 16-bit or 262,144 float32 tokens;
 * longer rows fail with BMS_ERROR_UNSUPPORTED).  Calls that overlap in time on one device (other
 * streams or threads) share the array and race: serialize them.  The first call on a device
 * resolves the array's address and clears its counters; make it before any stream capture. */
BMS_API int bms_masked_reduce_batch_noalloc(const void *logits, int32_t dtype, const int32_t *masks, int64_t rows,
                                            int64_t vocab, int64_t *tokens, int64_t *counts, int32_t *status,
                                            int32_t device, void *stream);

/* Replaces csrc/sample.cu:116-132 masked_sample_cuda: inverse-CDF sample of
 * the masked softmax at `temperature` with the device float64 scalar
 * `uniform` in [0, 1).  temperature == 0 is the masked argmax (uniform unused). */
BMS_API int bms_masked_sample(const void *logits, int32_t dtype, const int32_t *mask, int64_t vocab,
                      double temperature, const double *uniform, int64_t *token, int32_t *status,
                      int32_t device, void *stream);

/* Batched form of bms_masked_sample with one uniform per row (no reference
 * counterpart; the reference sampled one row per launch).  `counts` and
 * `workspace` may be NULL. */
BMS_API int bms_masked_sample_batch(const void *logits, int32_t dtype, const int32_t *masks, int64_t rows,
                            int64_t vocab, double temperature, const double *uniforms,
                            int64_t *tokens, int64_t *counts, int32_t *status, void *workspace,
                            int64_t workspace_bytes, int32_t device, void *stream);

/* Device form of grammar/density.py:23-53 (packed_mask_count / density) and
 * decoding/scheduling.py:40-46 (DensityPolicy.budget) for a [rows, words]
 * batch.  Any of counts / density / budget may be NULL; policy may be NULL when
 * budget is NULL. */
BMS_API int bms_mask_budget(const int32_t *masks, int64_t rows, int64_t vocab, const bms_policy *policy,
                    int64_t *counts, double *density, int32_t *budget, int32_t device, void *stream);

/* Compact upload form of mask rows (no reference counterpart; the reference copied every 31 KB
 * bitmap row to the device, kernels/dispatch.py:95).  Writes `lists` packed mask rows to `out`
 * (row l at out + l * ceil(vocab / 32), bits of the listed tokens set, every other bit clear) from
 * token-ID lists: list l is ids[offsets[l], offsets[l + 1]) (int32 device arrays; `offsets` has
 * lists + 1 entries; entries are clamped to [0, n_ids], so no offsets reach outside `ids`).  IDs may
 * repeat or come unsorted; an ID outside [0, vocab) sets nothing and sets bad[l] to 1 (else 0;
 * `bad` may be NULL).  Sparse rows sent this way plus dense rows sent as bitmaps form a mask table
 * for bms_verify_batch's `mask_rows`. */
BMS_API int bms_expand_token_lists(const int32_t *ids, int64_t n_ids, const int32_t *offsets, int64_t lists,
                                   int64_t vocab, int32_t *out, int32_t *bad, int32_t device, void *stream);

/* Like bms_expand_token_lists for rows given as byte-coded gap streams (no reference counterpart):
 * row l's stream is bytes[offsets[l], offsets[l + 1]) (`offsets` int32, rows + 1 entries, clamped to
 * [0, n_bytes]).  Starting before token 0, a byte b > 0 advances b tokens and allows the token it
 * reaches; a byte 0 advances 255 tokens and allows nothing.  About one byte per allowed token for
 * rows of 0.4 - 12 % density, against 4 bytes per token for ID lists and 4 * ceil(vocab / 32) for a
 * bitmap.  Tokens at or past `vocab` set nothing and set bad[l] to 1 (`bad` may be NULL). */
BMS_API int bms_expand_token_gaps(const uint8_t *bytes, int64_t n_bytes, const int32_t *offsets, int64_t rows,
                                  int64_t vocab, int32_t *out, int32_t *bad, int32_t device, void *stream);

/* One batched verification round (decoding/verification.py:18-48 verify_prefix
 * over the rows models/transformers.py:181-201 selects from).  Sequence s owns
 * rows [s*rows_per_seq, (s+1)*rows_per_seq); row s*rows_per_seq + i is the
 * target's prediction after proposals[s, :i].  proposals is [seqs,
 * rows_per_seq - 1], lengths[s] proposals are live.  Outputs: per row the
 * masked argmax, count, status and policy budget; per sequence the accepted
 * prefix length, the correction / bonus / fallback token, its kind (0
 * correction, 1 bonus, 2 fallback) and a status that is nonzero only when a
 * row the reference would have consumed failed.  row_counts and row_budget
 * may be NULL (then policy may be NULL); `workspace` may be NULL.  Mask table (no
 * reference counterpart): with `mask_rows` non-NULL, `masks` is a table of
 * `mask_table_rows` mask rows resident on the device (e.g. one per grammar state)
 * and row r uses table row mask_rows[r] (int32, device); an index outside the
 * table fails that row with BMS_STATUS_BAD_MASK_ROW. */
BMS_API int bms_verify_batch(const void *logits, int32_t dtype, const int32_t *masks, int64_t seqs,
                     int64_t rows_per_seq, int64_t vocab, const int64_t *proposals,
                     const int32_t *lengths, const bms_policy *policy, int64_t *row_tokens,
                     int64_t *row_counts, int32_t *row_status, int32_t *row_budget,
                     int32_t *accept_len, int64_t *token, int32_t *kind, int32_t *seq_status,
                     const int32_t *mask_rows, int64_t mask_table_rows, void *workspace,
                     int64_t workspace_bytes, int32_t device, void *stream);

/* ---- vocabulary shards ----------------------------------------------------------------
 * A row's vocabulary split across ranks (GPUs), each holding logits [rows, vocab_shard] of its
 * slice and the full mask rows.  Each rank computes one 32-byte partial per row; the partials of
 * all ranks, gathered in rank order (e.g. an NCCL all-gather), are merged on every rank.  The
 * merge uses the same arithmetic as the single-GPU kernel's cluster merge, so a single-GPU run
 * whose cluster ranks cover the same slices gives identical results. No reference counterpart:
 * the reference ran one row on one device (docs/design.md:10-11). */
typedef struct bms_partial {
    uint32_t a, b, c, d; /* argmax: ordered max bits, ~first global index, count, flags;
                            sampler: max bits, count, flags, 0 */
    double s;            /* sampler: shard mass relative to its max */
    double reserved;
} bms_partial;

/* Bytes of one row's sampler granule record for a shard of `vocab_shard` tokens (-1 if invalid). */
BMS_API int64_t bms_shard_granule_bytes(int32_t dtype, int64_t vocab_shard);

/* Partials of this rank's shard: tokens [token_offset, token_offset + vocab_shard) of every row
 * (token_offset a multiple of 32).  `masks` are the full rows ([rows, mask_words] int32).
 * temperature 0: argmax partials (granules may be NULL); else sampler partials plus one granule
 * record per row at `granules + row * granule_stride` (stride >= bms_shard_granule_bytes, multiple
 * of 16). */
BMS_API int bms_shard_partials(const void *logits, int32_t dtype, const int32_t *masks, int64_t mask_words,
                               int64_t rows, int64_t vocab_shard, int64_t token_offset, double temperature,
                               bms_partial *partials, void *granules, int64_t granule_stride, int32_t device,
                               void *stream);

/* bms_shard_partials with a mask table: row r's mask is row mask_rows[r] of `masks`
 * ([mask_table_rows, mask_words] int32; mask_rows int32 on the device), so rows that share mask
 * rows need no gathered copy -- the draft rows of bms_speculative_accept: draft row s * K + i takes
 * mask row s * (K + 1) + i.  An index outside [0, mask_table_rows) fails its row with
 * BMS_STATUS_BAD_MASK_ROW.  mask_rows NULL is bms_shard_partials. */
BMS_API int bms_shard_partials_indexed(const void *logits, int32_t dtype, const int32_t *masks, int64_t mask_words,
                                       const int32_t *mask_rows, int64_t mask_table_rows, int64_t rows,
                                       int64_t vocab_shard, int64_t token_offset, double temperature,
                                       bms_partial *partials, void *granules, int64_t granule_stride,
                                       int32_t device, void *stream);

/* Merge `shards` ranks' partials ([shards, rows] in rank order) on rank `shard`.  temperature 0:
 * final argmax tokens, counts and status of every row (identical on every rank).  Sampler: status
 * and counts of every row; `tokens[row]` is the sampled token if it lies in this rank's shard and
 * -1 otherwise (a max-reduction over ranks gives the token).  The sampler walk re-reads this rank's
 * shard (`logits`, `masks`, `granules` as given to bms_shard_partials); uniforms are [rows]. */
BMS_API int bms_shard_merge(const bms_partial *partials, int32_t shards, int32_t shard, int64_t rows,
                            double temperature, const double *uniforms, const void *logits, int32_t dtype,
                            const int32_t *masks, int64_t mask_words, int64_t vocab_shard, int64_t token_offset,
                            const void *granules, int64_t granule_stride, int64_t *tokens, int64_t *counts,
                            int32_t *status, int32_t device, void *stream);

/* Stochastic speculative acceptance (speculative sampling; no counterpart in the reference, whose
 * correctness contract is greedy, docs/design.md:5-11).  Sequence s has lengths[s] = L <= K drafts
 * proposals[s, i] ([seqs, K] int64, K = rows_per_seq - 1) that were drawn from the draft model's
 * masked softmax q_i at `temperature` (draft logits row s * K + i); target logits row
 * s * rows_per_seq + i gives p_i; both use mask row s * rows_per_seq + i.  The partials are
 * bms_shard_partials outputs (whole rows, token_offset 0, the same temperature) of the target rows
 * and of the draft rows (bms_shard_partials_indexed for the draft rows' mask rows).  Both NULL: the
 * kernel computes the normalisers of the positions it consumes itself, position by position up to
 * the first rejection (rows and mask rows must then be 16-byte aligned, rows a multiple of 16 bytes,
 * mask rows a multiple of 4 words; else BMS_ERROR_UNSUPPORTED).  Draft i is accepted iff accept_uniforms[s, i] * q_i(d_i) < p_i(d_i); at the
 * first rejection j the token is drawn by inverse CDF with resample_uniforms[s] from
 * max(0, p_j - q_j) normalised (from p_j if that rounds to zero mass), after L acceptances from p_L:
 * every emitted token is distributed as the target's masked softmax.  Outputs per sequence: accepted
 * length, token (-1 on error), kind (0 replacement, 1 bonus, 2 fallback for L = 0) and status
 * (BMS_STATUS_* of the first consumed row that cannot be sampled; 6 for L outside [0, K]).  Uniforms
 * are float64 in [0, 1).  temperature must be positive (temperature 0 is bms_verify_batch). */
BMS_API int bms_speculative_accept(const void *target_logits, const void *draft_logits, int32_t dtype,
                                   const int32_t *masks, int64_t seqs, int64_t rows_per_seq, int64_t vocab,
                                   const int64_t *proposals, const int32_t *lengths,
                                   const bms_partial *target_partials, const bms_partial *draft_partials,
                                   double temperature, const double *accept_uniforms, const double *resample_uniforms,
                                   int32_t *accept_len, int64_t *token, int32_t *kind, int32_t *status,
                                   int32_t device, void *stream);

/* ---- Peer-memory exchange of argmax shard partials (no reference counterpart: it replaces the
 * NCCL all-gather between bms_shard_partials and bms_shard_merge with stores over NVLink).
 * Each rank of a group of `ranks` (<= 8, one GPU each) creates one exchange area in its device
 * memory and exports it; every rank opens the peers' areas.  `areas` below is a host array of
 * `ranks` device pointers in rank order: this rank's own area at [rank], the peers' mapped areas
 * elsewhere.  Step `epoch` starts at 1 and grows by one per step on every rank.  A step is one
 * bms_shard_partials_exchange and one bms_shard_merge_exchange per rank on the same stream; the
 * selection kernel stores each row's partial into every area while it streams, the merge waits
 * (bounded, about one second) until every rank's partials of the step arrived.  A wait that gives
 * up reports status 7 (BMS_STATUS_TIMEOUT) for the affected rows.  Every rank passes the same
 * `rows` in a step: each partial carries its step's epoch, and a row whose partial from some rank
 * has another epoch (that rank's step had fewer rows) also reports status 7.  Callers must check
 * the statuses for 7; the ranks' results are then undefined for those rows. */
typedef struct bms_ipc_handle {
    unsigned char bytes[64]; /* cudaIpcMemHandle_t */
} bms_ipc_handle;

/* Bytes of one exchange area for `ranks` ranks and batches of at most `rows_cap` rows (-1 if invalid). */
BMS_API int64_t bms_exchange_bytes(int32_t ranks, int64_t rows_cap);

/* Allocate this rank's exchange area (zeroed) on `device` and export it. */
BMS_API int bms_exchange_create(int32_t device, int32_t ranks, int64_t rows_cap, void **area,
                                bms_ipc_handle *handle);

/* Map a peer's exported area into this process (peer access enabled on demand). */
BMS_API int bms_exchange_open(int32_t device, const bms_ipc_handle *handle, void **area);

/* Unmap a peer's area / free this rank's own area. */
BMS_API int bms_exchange_close(int32_t device, void *area);
BMS_API int bms_exchange_destroy(int32_t device, void *area);

/* bms_shard_partials at temperature 0 with every row's partial also stored into each rank's area. */
BMS_API int bms_shard_partials_exchange(const void *logits, int32_t dtype, const int32_t *masks, int64_t mask_words,
                                        int64_t rows, int64_t vocab_shard, int64_t token_offset,
                                        void *const *areas, int32_t ranks, int32_t rank, int64_t rows_cap,
                                        uint32_t epoch, int32_t device, void *stream);

/* bms_shard_merge at temperature 0 over the step's partials in this rank's area. */
BMS_API int bms_shard_merge_exchange(void *const *areas, int32_t ranks, int32_t rank, int64_t rows_cap,
                                     uint32_t epoch, int64_t rows, int64_t *tokens, int64_t *counts,
                                     int32_t *status, int32_t device, void *stream);

/* Test hook: force the cluster size (1, 2, 4, 8 or 16) and the number of
 * clusters of the selection kernels' fixed schedule; 0 restores the automatic
 * choice.  With cluster 0 and a workspace, `clusters` caps the number of CTAs of
 * the dynamic schedule.  Any override turns the flat sampler schedule off.
 * Process-wide; not for concurrent use with other calls. */
BMS_API int bms_set_launch_override(int32_t cluster, int32_t clusters);

#ifdef __cplusplus
}
#endif

#endif /* BMS_B200_H */
