/*
 * speckv.h - C ABI of the B200 (sm_100a) static-KV-cache / tree-verify library.
 *
 * Every entry point takes plain device pointers, element counts / strides and
 * a cudaStream_t passed as `void*` (NULL = legacy default stream). Nothing here
 * allocates device memory: buffers (pools, index lists, masks, outputs, the
 * optional remap scratch) are owned by the caller. Every call is asynchronous
 * on `stream` and returns a status code; the message for a non-zero status is
 * available from speckv_last_error() on the calling thread.
 *
 * Pool layout (one K pool and one V pool per layer, as the reference keeps):
 *   pool[batch_capacity][heads][capacity][dim], row = dim * elem_bytes bytes,
 *   contiguous. A "row" below is one (sequence, head, position) vector.
 *
 * Layer-batched calls take host arrays of `layers` device pointers (K pools and
 * V pools); all layers of one call share geometry. At most SPECKV_MAX_LAYERS
 * layers per call.
 *
 * Index inputs (int64) that address cache rows are bounds-checked on the
 * device: an out-of-range entry is skipped and recorded in a device-side error
 * word that speckv_device_error() reads back and clears. Kernels never trap.
 *
 * Kernels launch on the CURRENT device: an operand that is device memory of
 * another GPU, or plain host memory, is refused with SPECKV_EINVAL before any
 * launch (checked with the driver's pointer attributes). A prepared plan
 * launches only while the device it was prepared on is current.
 */
#ifndef SPECKV_H
#define SPECKV_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SPECKV_OK 0
#define SPECKV_EINVAL 1      /* bad argument (host-side check) */
#define SPECKV_ECUDA 2       /* a CUDA runtime call failed */
#define SPECKV_ENOSUPPORT 3  /* shape outside what this build handles */

#define SPECKV_MAX_LAYERS 64

/* Device error word kinds (upper 16 bits of the word; lower 48 = offending value). */
#define SPECKV_DERR_REMAP_INDEX 1
#define SPECKV_DERR_COMPACT_INDEX 2
#define SPECKV_DERR_MOVE_INDEX 3
#define SPECKV_DERR_TREE_INDEX 4
#define SPECKV_DERR_OWNER_INDEX 5
#define SPECKV_DERR_TIMEOUT 6  /* a bounded wait inside a kernel expired; value = wait site */
#define SPECKV_DERR_PACKET 7   /* scheduling packet inconsistent with the commit; value = its width */
#define SPECKV_DERR_SEEN_INDEX 8 /* draft expansion: seen position outside [0, columns) */
#define SPECKV_DERR_HISTORY_INDEX 9 /* history append: owner row or source position out of range */
#define SPECKV_DERR_ROW_TABLE 10    /* row table entry outside the pools' rows; value = the entry */

#define SPECKV_HISTORY_MAX_FIELDS 4

/* dtype codes for masks / attention operands */
#define SPECKV_F32 0
#define SPECKV_BF16 1
#define SPECKV_F16 2

/* ---- library state -------------------------------------------------------- */

/* ABI version (major*100 + minor). */
int speckv_version(void);

/* Message of the last non-zero status returned on this thread. */
const char* speckv_last_error(void);

/* Copy the device error word of the current device to *word (0 = none) and
 * clear it. Synchronises `stream`. */
int speckv_device_error(uint64_t* word, void* stream);

/* ---- Row tables ------------------------------------------------------------
 * speckv_append_rows, speckv_compact_suffix, speckv_commit_round (and their
 * prepared forms) and speckv_tree_attention_bits take an optional row table:
 * row_table[b] (int64, device) is the pool row holding sequence b, for b < batch;
 * pool_rows (kv_batch for the attention) is the pools' row count, which every
 * entry must stay below (an entry outside it sets device error
 * SPECKV_DERR_ROW_TABLE and that sequence is skipped). NULL keeps sequence b in
 * pool row b (pool_rows may then be 0). With a table, releasing and admitting
 * sequences is an update of the table instead of a move of their histories
 * (the reference's swap_remove moves whole rows, helper/opd_static_cache.py:157-174);
 * the reference has no such table. */

/* ---- KV rows: append / grow --------------------------------------------- */

/* Append `rows` new positions for every (sequence, head) of `layers` layers:
 *   pool[b][h][length + t][:] = src[b][h][t][:]   for b < batch, h < heads, t < rows
 * Sources are strided views (B, H, rows, dim) with unit stride on dim and the
 * given element strides on (b, h, t); K and V sources may differ in stride.
 * Replaces StaticAppendLayer.update's two copies
 * (helper/opd_static_cache.py:106-107) and, with length = 0 and the old pool as
 * source, the history copy of StaticAppendLayer._grow (:88-90). */
int speckv_append_rows(void* const* key_pools, void* const* value_pools,
                       const void* const* key_srcs, const void* const* value_srcs,
                       int32_t layers, int64_t batch, int64_t heads, int64_t rows,
                       int64_t dim, int64_t capacity, int64_t length,
                       const int64_t* key_src_strides, const int64_t* value_src_strides,
                       int32_t elem_bytes, const int64_t* row_table, int64_t pool_rows, void* stream);

/* ---- KV rows: accepted-suffix compaction ------------------------------- */

/* For every layer, K and V, sequence b < batch and head h < heads:
 *   tmp[j]                 = pool[b][h][chosen[b][extension + j]]   j < width - extension
 *   pool[b][h][past + extension + j] = tmp[j]
 * (all reads of one (b, h) happen before its writes, as the reference's
 * gather-into-scratch then copy). `length` is the visible length the chosen
 * positions must lie below. Replaces compact_suffix_inplace
 * (helper/opd_scheduling.py:35-58) and its per-layer loop
 * (helper/opd_generate.py:637-641) with one launch. */
int speckv_compact_suffix(void* const* key_pools, void* const* value_pools, int32_t layers,
                          int64_t batch, int64_t heads, int64_t dim, int64_t capacity,
                          int64_t length, const int64_t* chosen, int64_t chosen_stride_b,
                          int64_t chosen_stride_w, int64_t past, int64_t extension,
                          int64_t width, int32_t elem_bytes, const int64_t* row_table, int64_t pool_rows,
                          void* stream);

/* ---- KV rows: device-scheduled commit of a verify round ----------------- */

/* speckv_compact_suffix of every layer followed by speckv_position_update, in
 * one launch, with width and extension read from the scheduling packet on the
 * device instead of passed by the host:
 *   width     = max_b packet[b][0]                      (longest accepted path)
 *   extension = min over b with packet[b][1] == 0 of packet[b][2]
 *               (= width when every sequence finished)
 * so the commit can be enqueued right after speckv_pad_schedule, before the
 * host reads the packet back. `chosen` / `newly_padded` / `positions` are the
 * full (batch, max_width) padded-schedule outputs; columns >= width are not
 * read. layers == 0 skips the compaction, positions == NULL skips the position
 * update. A packet whose width exceeds max_width or length - past sets device
 * error SPECKV_DERR_PACKET and moves nothing. Replaces the host round trip
 * between schedule (helper/opd_scheduling.py:5-32) and the commit at
 * helper/opd_generate.py:632-650 (compaction loop, crop, position update). */
int speckv_commit_round(void* const* key_pools, void* const* value_pools, int32_t layers,
                        int64_t batch, int64_t heads, int64_t dim, int64_t capacity, int64_t length,
                        int32_t elem_bytes, const int64_t* chosen, int64_t chosen_stride_b,
                        int64_t chosen_stride_w, int64_t past, const int64_t* packet,
                        int64_t packet_stride, int64_t max_width, uint8_t* pad_rows,
                        int64_t pad_rows_stride, int64_t pad_rows_count, const int64_t* owners,
                        uint8_t* pad_live, int64_t pad_live_stride, const uint8_t* newly_padded,
                        int64_t np_stride_b, int64_t* positions, int64_t positions_stride_b,
                        int64_t* past_positions, const int64_t* row_table, int64_t pool_rows, void* stream);

/* ---- Draft-model attention masks ---------------------------------------- */

/* Causal additive mask (batch, 1, query, columns), contiguous: entry (b, r, c) is 0
 * when c <= past + r and pad[b][c] is false (pad may be NULL; element strides
 * pad_stride_b, pad_stride_c), else the dtype's lowest finite value (dtype
 * SPECKV_F32 / BF16 / F16). Replaces AttentionWorkspace.causal's CUDA branch
 * (helper/opd_attention.py:31-43) and its kernel
 * (helper/opd_attention_kernels.py:7-22). */
int speckv_causal_mask(void* mask, int32_t dtype, int64_t batch, int64_t query, int64_t past,
                       int64_t columns, const uint8_t* pad, int64_t pad_stride_b, int64_t pad_stride_c,
                       uint32_t* bits, int64_t row_words, int32_t* first_col, void* stream);

/* Draft expansion mask (batch, 1, query, columns), contiguous: entry (b, r, c) is 0
 * when (c < init_length or c == seen[b][r]) and pad[b][c] is false, else the dtype's
 * lowest value; seen is int64 with element strides (seen_stride_b, seen_stride_r).
 * One launch for the zero / [init:] fill / scatter / padding fill sequence of
 * helper/opd_generate.py:143-161 (bool padding form). A seen position outside
 * [0, columns) sets device error SPECKV_DERR_SEEN_INDEX and that row sees only
 * its first init_length columns. */
int speckv_expansion_mask(void* mask, int32_t dtype, int64_t batch, int64_t query, int64_t columns,
                          int64_t init_length, const int64_t* seen, int64_t seen_stride_b,
                          int64_t seen_stride_r, const uint8_t* pad, int64_t pad_stride_b,
                          int64_t pad_stride_c, uint32_t* bits, int64_t row_words, int32_t* first_col,
                          void* stream);

/* Both mask entries optionally (bits non-NULL) also write the mask's visibility in
 * the form speckv_tree_attention_bits reads: bits[b * query + r][w] bit i = entry
 * (b, r, 32 w + i) is 0; row_words >= 4 * ceil(columns / 128), words past the last
 * column 0; first_col[b] = the first column any row of sequence b sees
 * (0x7f7f7f7f when none). The draft attention then skips the dense mask read. */

/* ---- Rollout history ---------------------------------------------------- */

/* Appends positions to up to SPECKV_HISTORY_MAX_FIELDS history pools in one launch:
 *   pool_f[owners[i]][starts[f] + w] = src_f[src_rows ? src_rows[i] : i][index_f ? index_f[i][w] : w]
 * for i < n, w < widths[f]; with gathered[f] non-NULL the same elements also go
 * to a contiguous (n, widths[f], row_bytes[f]) buffer, and with pools[f] NULL
 * only there. Strides: pool_strides / src_strides are (row, position) pairs in
 * BYTES per field; index_strides (row, position) pairs in elements; a position
 * holds row_bytes[f] bytes (any element type). src_positions[f] bounds the
 * source position; starts[f] + widths[f] must not exceed capacities[f]. An owner
 * outside [0, pool_rows) or a source position outside [0, src_positions[f]) sets
 * device error SPECKV_DERR_HISTORY_INDEX and that element is skipped.
 * Replaces ContiguousRolloutHistory.append's per-field index_copy_
 * (helper/opd_history.py:24-42), the initial repeated copy (:12-22) and the grow
 * copy (:34-38); with an index it fuses the accepted-feature gather
 * (helper/opd_generate.py:567-571) with the append of :572-579. */
int speckv_history_append(int32_t fields, void* const* pools, const int64_t* pool_strides,
                          const void* const* srcs, const int64_t* src_strides,
                          const int64_t* const* indices, const int64_t* index_strides,
                          void* const* gathered, const int64_t* row_bytes,
                          const int64_t* src_positions, const int64_t* starts, const int64_t* widths,
                          const int64_t* capacities, const int64_t* owners, const int64_t* src_rows,
                          int64_t n, int64_t pool_rows, void* stream);

/* Packs the used prefix of every pool row into dst (contiguous, row_bytes per
 * position): dst[offsets[r] + p] = pool[r][p] for p < offsets[r + 1] - offsets[r],
 * r < rows; offsets is a device array of rows + 1 int64 values, max_length the
 * longest row (grid sizing only). Pool strides in bytes. Replaces the
 * repeat_interleave + index_select gather of ContiguousRolloutHistory.finalize
 * (helper/opd_history.py:52-67). */
int speckv_history_pack(void* dst, const void* pool, int64_t pool_row_stride, int64_t pool_pos_stride,
                        int64_t row_bytes, const int64_t* offsets, int64_t rows, int64_t max_length,
                        void* stream);

/* speckv_append_rows fused with the accepted-suffix compaction of the previous
 * verify round, in one launch: for every (layer, K/V, sequence b, head h)
 *   pool[b][h][past + j][:] = pool[b][h][chosen[b][j]][:]   for extension <= j < width
 *   pool[b][h][length + t][:] = src[b][h][t][:]             for t < rows
 * with every row of a (layer, K/V, sequence, head) read before any is written and
 * the new rows written last (where the two destinations overlap, the new rows
 * win). The compaction of a round only has to land before the next attention
 * reads the cache, so a verify loop can move it into the next round's append
 * (the round's own commit then updates positions only: speckv_commit_round with
 * no layers) and run it at the append's bandwidth. chosen positions outside
 * [0, capacity) set SPECKV_DERR_COMPACT_INDEX and are skipped. No row tables.
 * Returns SPECKV_ENOSUPPORT when (width - extension) * row vectors exceeds 256
 * or rows * row vectors exceeds 4096 (16-byte vectors): use
 * speckv_compact_suffix, then speckv_append_rows. Replaces, for one round, the
 * per-layer compact_suffix_inplace calls of helper/opd_generate.py:632-643
 * together with the next round's StaticAppendLayer.update copies
 * (helper/opd_static_cache.py:106-107). */
int speckv_append_commit_rows(void* const* key_pools, void* const* value_pools,
                              const void* const* key_srcs, const void* const* value_srcs,
                              int32_t layers, int64_t batch, int64_t heads, int64_t rows, int64_t dim,
                              int64_t capacity, int64_t length, const int64_t* key_src_strides,
                              const int64_t* value_src_strides, int32_t elem_bytes, const int64_t* chosen,
                              int64_t chosen_stride_b, int64_t chosen_stride_w, int64_t past, int64_t extension,
                              int64_t width, void* stream);

/* ---- Prepared launches -------------------------------------------------- */

/* speckv_append_rows / speckv_commit_round / speckv_append_commit_rows split in
 * two: *_prepare validates and
 * packs the same arguments (without the stream) into *plan and launches nothing;
 * speckv_plan_launch enqueues the prepared kernel on `stream`, whose host cost
 * is then one kernel launch, so a caller can do the preparation while the GPU
 * still runs the previous kernel. A plan keeps device pointers and sizes only
 * (the caller keeps the buffers alive and unchanged in shape); it can be
 * launched any number of times and is freed by speckv_plan_release. On error
 * *plan is NULL. Same results as the one-call entries. */
int speckv_append_commit_rows_prepare(void* const* key_pools, void* const* value_pools,
                                      const void* const* key_srcs, const void* const* value_srcs,
                                      int32_t layers, int64_t batch, int64_t heads, int64_t rows, int64_t dim,
                                      int64_t capacity, int64_t length, const int64_t* key_src_strides,
                                      const int64_t* value_src_strides, int32_t elem_bytes, const int64_t* chosen,
                                      int64_t chosen_stride_b, int64_t chosen_stride_w, int64_t past,
                                      int64_t extension, int64_t width, void** plan);
int speckv_append_rows_prepare(void* const* key_pools, void* const* value_pools,
                               const void* const* key_srcs, const void* const* value_srcs,
                               int32_t layers, int64_t batch, int64_t heads, int64_t rows,
                               int64_t dim, int64_t capacity, int64_t length,
                               const int64_t* key_src_strides, const int64_t* value_src_strides,
                               int32_t elem_bytes, const int64_t* row_table, int64_t pool_rows,
                               void** plan);
int speckv_commit_round_prepare(void* const* key_pools, void* const* value_pools, int32_t layers,
                                int64_t batch, int64_t heads, int64_t dim, int64_t capacity,
                                int64_t length, int32_t elem_bytes, const int64_t* chosen,
                                int64_t chosen_stride_b, int64_t chosen_stride_w, int64_t past,
                                const int64_t* packet, int64_t packet_stride, int64_t max_width,
                                uint8_t* pad_rows, int64_t pad_rows_stride, int64_t pad_rows_count,
                                const int64_t* owners, uint8_t* pad_live, int64_t pad_live_stride,
                                const uint8_t* newly_padded, int64_t np_stride_b, int64_t* positions,
                                int64_t positions_stride_b, int64_t* past_positions,
                                const int64_t* row_table, int64_t pool_rows, void** plan);
int speckv_plan_launch(const void* plan, void* stream);
void speckv_plan_release(void* plan);

/* ---- KV rows: batch remap (repeat / select) ---------------------------- */

/* Row remap over the live prefix [0, length) of every layer:
 *   pool'[i][h][t][:] = pool[indices[i]][h][t][:]   i < new_batch
 * with arbitrary permutations and duplicates (all reads before writes).
 * indices[i] must lie in [0, batch_capacity). `scratch` (scratch_bytes) is only
 * used when new_batch rows of one position do not fit on chip; it then needs
 * 2 * new_batch * heads * length * dim * elem_bytes bytes. Replaces
 * remap_rows (helper/opd_kv_kernels.py:34-40) called per layer from
 * StaticAppendLayer.batch_select_indices (helper/opd_static_cache.py:118-149). */
int speckv_remap_rows(void* const* key_pools, void* const* value_pools, int32_t layers,
                      const int64_t* indices, int64_t new_batch, int64_t batch_capacity,
                      int64_t heads, int64_t dim, int64_t capacity, int64_t length,
                      void* scratch, int64_t scratch_bytes, int32_t elem_bytes, void* stream);

/* Scratch bytes speckv_remap_rows needs for this geometry (0 when the remap
 * runs in a single on-chip pass). Host-only, no CUDA call. */
int64_t speckv_remap_scratch_bytes(int64_t new_batch, int64_t heads, int64_t dim, int64_t length,
                                   int32_t elem_bytes);

/* speckv_remap_rows for callers that cannot allocate device memory: a host
 * that has handed all device memory to its own pooling allocator up front (a
 * raw cudaMalloc would fail there), a latency-critical loop where cudaMalloc /
 * cudaFree would synchronise the device, or a foreign-language binding with no
 * access to the owning framework's allocator. It takes no scratch argument and
 * calls no allocator: the gather-then-scatter runs through a fixed
 * SPECKV_REMAP_STATIC_SCRATCH_BYTES array compiled into the library, which
 * every GPU that loads it holds until the process exits.
 * - Limit: 2 * new_batch * heads * dim * elem_bytes (K and V of one position of
 *   every output row) must fit in the array, else SPECKV_EINVAL; longer
 *   prefixes are processed in position chunks.
 * - The first call on each device looks the array's device address up
 *   (cudaGetSymbolAddress, with that device current); make that first call
 *   before any stream capture.
 * - All calls on a device share the one array and leave their data in it.
 *   Nothing in it needs to start at zero (every byte read was written by the
 *   same call), but calls that overlap on the GPU (other streams, other host
 *   threads) race on it: serialise them.
 * No counterpart in the reference: its remap always allocates its scratch
 * (helper/opd_static_cache.py:128-132). */
#define SPECKV_REMAP_STATIC_SCRATCH_BYTES (64ull << 20)
int speckv_remap_rows_static(void* const* key_pools, void* const* value_pools, int32_t layers,
                             const int64_t* indices, int64_t new_batch, int64_t batch_capacity,
                             int64_t heads, int64_t dim, int64_t capacity, int64_t length,
                             int32_t elem_bytes, void* stream);

/* ---- KV rows: release of finished rows (swap-remove) ------------------- */

/* pool[destinations[j]][h][t][:] = pool[sources[j]][h][t][:] for t < length,
 * j < count; sources and destinations disjoint. Replaces move_tail_rows
 * (helper/opd_kv_kernels.py:56-58) called per layer from
 * StaticAppendLayer.swap_remove (helper/opd_static_cache.py:157-174). */
int speckv_move_rows(void* const* key_pools, void* const* value_pools, int32_t layers,
                     const int64_t* sources, const int64_t* destinations, int64_t count,
                     int64_t batch_capacity, int64_t heads, int64_t dim, int64_t capacity,
                     int64_t length, int32_t elem_bytes, void* stream);

/* ---- tree kernels (helper/tree_kernels.py plugin) ----------------------- */

/* Re-index the confidence-selected draft nodes into a parent-closed packed
 * tree with the root at row 0 (helper/tree_verification.py:200-227):
 *   parents[b][0] = -1, tokens[b][0] = -1, contexts[b][0] = 0,
 *   parents[b][j+1] = packed row of full_parents[b][chosen[b][j]] (root = 0),
 *   tokens[b][j+1] = all_tokens[b][chosen[b][j]], contexts[b][j+1] = full_contexts[b][chosen[b][j]].
 * full_* are contiguous (batch, full_count), chosen contiguous (batch,
 * packed_count); outputs (batch, packed_count + 1) with row stride
 * out_stride_b. A node whose parent is not an earlier packed row is recorded
 * in the device error word (the reference's torch._assert_async). */
int speckv_pack_tree(const int64_t* full_parents, const int64_t* full_contexts, const int64_t* all_tokens,
                     const int64_t* chosen, int64_t batch, int64_t full_count, int64_t packed_count,
                     int64_t* out_parents, int64_t* out_tokens, int64_t* out_contexts,
                     int64_t out_stride_b, void* stream);

/* Greedy acceptance walk (helper/tree_kernels.py:68-95,
 * helper/tree_verification.py:286-322). parents/tokens/contexts/samples are
 * contiguous (batch, rows) int64; outputs (batch, width) with the given
 * strides; lengths (batch,). */
int speckv_trace_path(const int64_t* parents, const int64_t* tokens, const int64_t* contexts,
                      const int64_t* samples, int64_t batch, int64_t rows, int64_t eos,
                      int64_t* out_tokens, int64_t* out_indices, int64_t* out_contexts,
                      int64_t out_stride_b, int64_t out_stride_w, int64_t width,
                      int64_t* lengths, void* stream);

/* Gap-first padded commit layout (helper/tree_verification.py:237-268,
 * helper/tree_kernels.py:97-137). Inputs (batch, capacity) int64 with strides;
 * outputs tokens/indices (int64) and mask (bool bytes) (batch, width) with
 * out strides; last (batch,) with stride last_stride. */
int speckv_pad_verified_path(const int64_t* tokens, int64_t tok_stride_b, int64_t tok_stride_w,
                             const int64_t* indices, int64_t idx_stride_b, int64_t idx_stride_w,
                             const int64_t* lengths, int64_t batch, int64_t capacity,
                             int64_t width, int64_t past, int64_t eos,
                             int64_t* out_tokens, int64_t* out_indices, uint8_t* out_mask,
                             int64_t out_stride_b, int64_t out_stride_w,
                             int64_t* last, int64_t last_stride, void* stream);

/* Padded schedule + host packet (helper/tree_kernels.py:7-41): as above with
 * width = max(lengths) computed on the device, plus
 *   packet[b] = [length, last token == eos, extension, pad ids (capacity)..., snapshot?]
 * `snapshot` may be NULL (then column capacity + 3 is not written). */
int speckv_pad_schedule(const int64_t* tokens, int64_t tok_stride_b, int64_t tok_stride_w,
                        const int64_t* indices, int64_t idx_stride_b, int64_t idx_stride_w,
                        const int64_t* lengths, int64_t batch, int64_t capacity,
                        int64_t past, int64_t eos,
                        int64_t* out_tokens, int64_t* out_indices, uint8_t* out_mask,
                        int64_t out_stride_b, int64_t out_stride_w,
                        int64_t* last, int64_t last_stride,
                        int64_t* packet, int64_t packet_stride_b, int64_t packet_stride_w,
                        const int64_t* snapshot, void* stream);

/* Additive tree mask (batch, 1, rows, past + rows) (helper/tree_kernels.py:139-155,
 * helper/tree_verification.py:19-42): 0 where column <= past or column is
 * past + an ancestor of the row within `steps` parent hops (row itself
 * included), the dtype's lowest finite value elsewhere. If `pad` is non-NULL,
 * columns with pad[b * pad_stride_b + c] != 0 are forced to the lowest value
 * (the masked_fill_ at helper/opd_generate.py:483-484). */
int speckv_tree_mask(const int64_t* parents, int64_t batch, int64_t rows, int64_t past,
                     int64_t steps, void* mask, int32_t dtype, const uint8_t* pad,
                     int64_t pad_stride_b, void* stream);

/* Position / padding update after a commit (helper/opd_generate.py:556-558,
 * 644-650):
 *   pad_rows[owners[b]][past + j] = newly_padded[b][j]          (if pad_rows)
 *   pad_live[b][past + j]         = newly_padded[b][j]          (if pad_live)
 *   positions[b][j] = past_positions[b] + #{k <= j : !newly_padded[b][k]}
 *   past_positions[b] = positions[b][width - 1]
 * newly_padded is (batch, width) bool bytes with row stride np_stride_b. */
int speckv_position_update(uint8_t* pad_rows, int64_t pad_rows_stride, int64_t pad_rows_count,
                           const int64_t* owners, uint8_t* pad_live, int64_t pad_live_stride,
                           const uint8_t* newly_padded, int64_t np_stride_b, int64_t batch,
                           int64_t past, int64_t width, int64_t* positions,
                           int64_t positions_stride_b, int64_t* past_positions, void* stream);

/* Acceptance counters of one verify round, from the schedule packet's rows
 * [length, last token == eos, ...] (row stride packet_stride_b int64):
 *   counts[0] = sum over rows of max(length - 1, 0)   (accepted draft tokens)
 *   counts[1] = proposed_per_row * batch              (proposed draft tokens)
 *   counts[2] = sum of lengths, counts[3] = batch      (accepted-length sum / rows)
 *   counts[4] = rows whose last token is eos
 * (written, not accumulated; counts is a device array of 5 int64). The
 * increments helper/opd_generate.py:551-555 adds on the host after each
 * verification, computed on the device so that a sequence-sharded job can
 * all_reduce them without a host round trip. */
int speckv_acceptance_counts(const int64_t* packet, int64_t packet_stride_b, int64_t batch,
                             int64_t proposed_per_row, int64_t* counts, void* stream);

/* ---- tree-verify attention -------------------------------------------- */

/* GQA attention of `rows` tree queries over kv_len cached positions with an
 * additive mask, without materialising repeated K/V.
 * Head dim 128 in bf16 / fp16 runs on the tcgen05 tensor-core kernels only: a
 * view of that shape with a base or stride that is not 16-byte aligned is
 * refused with SPECKV_ENOSUPPORT (no silent slower path). Other head dims and
 * fp32 run on a CUDA-core kernel. speckv_attention_launches counts both.
 *   out[b][r][hq][:] = softmax_c(q[b][hq][r] . k[b][hq / g][c] * scale + mask[b][0][r][c]) v[b][hq/g][c]
 * g = q_heads / kv_heads. q/k/v element strides are given as (b, h, t) with unit
 * stride on dim; mask is (batch, 1, rows, kv_len) contiguous in `mask_dtype`
 * or NULL; out is contiguous (batch, rows, q_heads, dim) in `dtype`.
 * Replaces repeat_kv + F.scaled_dot_product_attention in transformers'
 * sdpa_attention_forward (integrations/sdpa_attention.py:56-104) as called from
 * Qwen2Attention.forward (models/qwen2/modeling_qwen2.py:206-240). */
int speckv_tree_attention(const void* q, const int64_t* q_strides,
                          const void* k, const int64_t* k_strides,
                          const void* v, const int64_t* v_strides,
                          const void* mask, int32_t mask_dtype,
                          void* out, int64_t batch, int64_t q_heads, int64_t kv_heads,
                          int64_t rows, int64_t kv_len, int64_t dim, float scale,
                          int32_t dtype, void* stream);

/* Bit-packed visibility of the tree mask for the tensor-core attention:
 *   bits[b][r][w] bit i = 1 iff column 32 w + i is visible to tree row r
 * with the same rule as speckv_tree_mask (columns >= past + rows are 0), and
 * first_col[b] = the first column any row of sequence b sees (tiles before it
 * are skipped). row_words must be >= 4 * ceil((past + rows) / 128). */
int speckv_tree_mask_bits(const int64_t* parents, int64_t batch, int64_t rows, int64_t past, int64_t steps,
                          const uint8_t* pad, int64_t pad_stride_b, uint32_t* bits, int64_t row_words,
                          int32_t* first_col, void* stream);

/* Visibility bits of a dense additive mask (batch, 1, rows, columns) with element
 * strides mask_strides = (b, r, c): bit set iff the entry is 0; entries equal to
 * the dtype's lowest finite value or -inf are masked; any other value sets
 * *nonbinary = 1 (device int32) and the bits must not be used. first_col[b] =
 * the first column any row of sequence b sees (0x7f7f7f7f when none). bits,
 * row_words and first_col as for speckv_tree_mask_bits. Lets the drop-in
 * attention convert transformers' per-forward 4-D mask (built once, read by every
 * layer, integrations/sdpa_attention.py:40-104) once into the form
 * speckv_tree_attention_bits reads. */
int speckv_mask_bits(const void* mask, int32_t dtype, int64_t batch, int64_t rows, int64_t columns,
                     const int64_t* mask_strides, uint32_t* bits, int64_t row_words, int32_t* first_col,
                     int32_t* nonbinary, void* stream);

/* speckv_tree_attention with visibility taken from speckv_tree_mask_bits output
 * instead of a dense mask (masked scores contribute exactly 0). first_col may
 * be NULL. */
int speckv_tree_attention_bits(const void* q, const int64_t* q_strides,
                               const void* k, const int64_t* k_strides,
                               const void* v, const int64_t* v_strides,
                               const uint32_t* bits, int64_t row_words, const int32_t* first_col,
                               void* out, int64_t batch, int64_t q_heads, int64_t kv_heads,
                               int64_t rows, int64_t kv_len, int64_t dim, float scale,
                               int32_t dtype, const int64_t* row_table, int64_t kv_batch, void* stream);

/* The round's tree-row append fused into the verify attention of one layer: the
 * same pools and output as speckv_append_rows(k_new / v_new into the pools at
 * position past) followed by speckv_tree_attention_bits over kv_len = past + rows,
 * in one launch. Replaces, per decoder layer, the two copy_ calls of
 * StaticAppendLayer.update (helper/opd_static_cache.py:106-107) together with the
 * attention that reads the cache right after them (transformers
 * integrations/sdpa_attention.py:40-104, called from helper/opd_generate.py:490).
 * k_pool / v_pool: (batch, kv_heads, capacity, dim) strided pools holding `past`
 * cached positions, past + rows <= capacity; k_new / v_new: (batch, kv_heads, rows,
 * dim) strided views (the projection output). The cached positions are attended in
 * 128-key tiles (the last one cut at past) and the new rows as one more tile read
 * straight from k_new / v_new, which the kernel stores into the pools once loaded.
 * Head dim 128, bf16 / fp16, rows <= 128, 16-byte aligned bases and strides; no row
 * table. bits / row_words / first_col as for speckv_tree_attention_bits over the
 * past + rows columns. The attention sums over a different key-tile split than
 * speckv_tree_attention_bits, so outputs agree to rounding, not bit for bit; the
 * pools are bit-exact. */
int speckv_tree_attention_bits_append(const void* q, const int64_t* q_strides,
                                      void* k_pool, const int64_t* k_pool_strides,
                                      void* v_pool, const int64_t* v_pool_strides,
                                      int64_t past, int64_t capacity,
                                      const void* k_new, const int64_t* k_new_strides,
                                      const void* v_new, const int64_t* v_new_strides,
                                      const uint32_t* bits, int64_t row_words, const int32_t* first_col,
                                      void* out, int64_t batch, int64_t q_heads, int64_t kv_heads,
                                      int64_t rows, int64_t dim, float scale, int32_t dtype, void* stream);

/* Launches issued since the library was loaded by speckv_tree_attention /
 * speckv_tree_attention_bits calls, per kernel family: *tensor_core the tcgen05
 * kernels, *cuda_core the CUDA-core kernel (other head dims, fp32). Replays of a
 * captured CUDA graph are not calls and are not counted. No reference
 * counterpart (the reference dispatches inside torch's SDPA). */
int speckv_attention_launches(int64_t* tensor_core, int64_t* cuda_core);

/* Upper bound on the persistent grid of speckv_tree_attention_bits for this process
 * (0, the default: one CTA per SM). A job that runs a collective beside the attention
 * (the sequence-sharded verify loop's counter all_reduce on a side stream) sets it to the
 * SM count minus the collective's CTAs, so that no attention CTA waits for an SM the
 * collective holds while it waits for the other ranks. No reference counterpart. */
int speckv_attention_set_ctas(int32_t ctas);

/* Key-range chunks in speckv_tree_attention_bits for this process (on = 1; 0, the default,
 * turns them off). With chunks on, a launch in which some sequence has more key tiles than a
 * CTA's average share of the launch (sum over sequences of key tiles x items per sequence,
 * over the grid) splits that sequence's work items into key-range chunks of about that share,
 * run by different CTAs; each chunk stores its unnormalised output rows with their running
 * max and sum in the library's partial buffers, and the CTA that finishes a row tile's last
 * chunk merges them (a softmax merge in fp32) and writes the output. For batches of ragged,
 * long sequences (a few sequences far longer than the rest), whose longest items otherwise
 * set the launch's duration. Launches with a row table run without chunks. Up to 4 launches
 * with chunks may run at the same time on one device (on different streams); make the first
 * launch with chunks on each device before any stream capture. No reference counterpart. */
int speckv_attention_set_chunks(int32_t on);

/* Test hook of the tensor-core attention kernels on the current device
 * (synchronous): every bounded wait inside them gives up after wait_limit_ns
 * (0 = the default of 2 s) and records SPECKV_DERR_TIMEOUT with the wait site;
 * withhold_q_arrival = 1 makes CTA 0 of the visibility-bits kernel withhold the
 * arrival of its first Q tile, so that the MMA warp's wait for it runs out with
 * no copy or MMA in flight and the kernel unwinds. Lets a test check the
 * timeout path without a GPU fault; keep both 0 otherwise. No reference
 * counterpart (the reference's kernels have no bounded waits). */
int speckv_attention_test_hooks(int64_t wait_limit_ns, int32_t withhold_q_arrival);

#ifdef __cplusplus
}
#endif

#endif /* SPECKV_H */
