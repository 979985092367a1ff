/*
 * silkern_b200 -- C ABI of the B200 (sm_100a) sparse-index localization converter.
 *
 * The converter turns one selection batch of global logical token positions
 * (batch, width) int32 into the rank-local physical KV slots that one decode
 * context-parallel (DCP) rank owns, compacted to the front of each row in the
 * selector's order, plus an exact valid count per row.
 *
 * Per element t of row r (request q = req_ids[r], table row = block_table[q]):
 *   owner = (t / interleave) % dcp_size                       (t >= 0 only)
 *   local = (t / (dcp_size * interleave)) * interleave + t % interleave
 *   lb, off = local / block_size, local % block_size
 *   valid  = t >= 0 && owner == dcp_rank && lb < table_width
 *   phys   = block_table[q][lb] * block_size + off            (int32 wrap)
 * With compaction (compact_valid_to_front && dcp_size > 1) the valid values
 * fill out[r][0:count] in input order and the rest of the row is -1; without
 * it every column keeps its own value (phys, or -1 when invalid).
 *
 * Conventions shared by every entry point:
 *   - every buffer is caller-owned int32 device memory, contiguous, on the
 *     device that is current on the calling thread; nothing is allocated and
 *     nothing is synchronised, so calls may be captured in a CUDA graph;
 *   - `stream` is a cudaStream_t (NULL = legacy default stream);
 *   - launches use programmatic dependent launch: each kernel waits on the
 *     previous grid in the stream before it reads any input;
 *   - `status` may be NULL; otherwise a row whose request id is outside
 *     [0, table_rows) is emitted as all -1 with count 0 and the kernel stores
 *     SILKERN_STATUS_BAD_REQUEST into *status, and a cluster whose count
 *     exchange ran out of its wait bound ORs in SILKERN_STATUS_EXCHANGE_TIMEOUT
 *     (the kernel never clears *status);
 *   - return value: 0 on success, a positive SILKERN_E* code when an argument
 *     is rejected before launch (nothing is enqueued), or -(cudaError_t) when
 *     the launch itself fails.
 */
#ifndef SILKERN_B200_H_
#define SILKERN_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SILKERN_ABI_VERSION 1

#define SILKERN_OK 0
#define SILKERN_E_NULL 1         /* a required pointer is NULL */
#define SILKERN_E_SHAPE 2        /* batch/width/table dimensions out of range */
#define SILKERN_E_DCP 3          /* invalid dcp_size / dcp_rank / interleave */
#define SILKERN_E_BLOCK_SIZE 4   /* block_size < 1 or not divisible by interleave */
#define SILKERN_E_TILE 5         /* unsupported tile_size */
#define SILKERN_E_ALIAS 6        /* an output overlaps an input or another output */
#define SILKERN_E_GEOMETRY 7     /* explicit launch geometry rejected */
#define SILKERN_E_SCRATCH 8      /* batch x tiles exceeds SILKERN_NOALLOC_MAX_TILES */

#define SILKERN_STATUS_BAD_REQUEST 1
/* Status bit of the converter entry points (OR-ed into *status): a row split
 * over a thread-block cluster whose CTAs did not complete their count
 * exchange within the kernel's wait bound. The CTAs that gave up store
 * nothing for that row (out, counts and tiles keep their previous contents).
 * It does not occur in a working cluster launch. */
#define SILKERN_STATUS_EXCHANGE_TIMEOUT 4
/* Status bit of the fused top-k entry point (OR-ed into *status). */
#define SILKERN_STATUS_BAD_LENGTH 2 /* a seq_len outside [0, logits_width]; clamped */

/* Widest selection row either entry point accepts. */
#define SILKERN_MAX_ROW_WIDTH 16384
/* Hierarchical tile sizes accepted by the workspace geometry. */
#define SILKERN_MIN_TILE_SIZE 64
#define SILKERN_MAX_TILE_SIZE 1024

/*
 * Row-wise stable localization: one launch; each row is scanned by one CTA
 * or by a group of threads inside one (or, for long rows with few requests,
 * by a thread-block cluster that exchanges per-CTA counts through distributed
 * shared memory).
 * Replaces silkern/kernels.py:318-434 (localize_rowwise and _rowwise_kernel,
 * kernels.py:51-125). block_table is (table_rows, table_width); tokens and
 * out are (batch, width); req_ids and counts are (batch,).
 */
int silkern_localize_rowwise_v1(const int32_t* req_ids, const int32_t* block_table,
                                int64_t table_rows, int64_t table_width,
                                const int32_t* tokens, int32_t* out, int32_t* counts,
                                int64_t batch, int64_t width, int32_t block_size,
                                int32_t dcp_size, int32_t dcp_rank, int32_t dcp_interleave,
                                int32_t compact_valid_to_front, int32_t* status,
                                void* stream);

/*
 * Hierarchical stable localization for wide rows: each row is split into
 * tiles of tile_size columns; the CTAs of one row form a thread-block cluster,
 * compose their tile-prefix offsets deterministically (no atomics) and
 * publish them into the caller-owned workspace: tile_counts[r][k] is the
 * number of valid elements in tile k and tile_offsets[r][k] the exclusive
 * prefix of those counts, both (batch, ceil(width / tile_size)).
 * mapped_ws and local_positions_ws, (batch, width), are accepted for
 * interface compatibility and are neither read nor written (may be NULL).
 * Replaces silkern/kernels.py:436-633 (localize_hierarchical and the
 * _map_tiles / _tile_prefix / _fill_output / _scatter_tiles kernels,
 * kernels.py:127-315).
 */
int silkern_localize_hierarchical_v1(const int32_t* req_ids, const int32_t* block_table,
                                     int64_t table_rows, int64_t table_width,
                                     const int32_t* tokens, int32_t* out, int32_t* counts,
                                     int32_t* mapped_ws, int32_t* local_positions_ws,
                                     int32_t* tile_counts_ws, int32_t* tile_offsets_ws,
                                     int64_t batch, int64_t width, int32_t block_size,
                                     int32_t dcp_size, int32_t dcp_rank, int32_t dcp_interleave,
                                     int32_t compact_valid_to_front, int32_t tile_size,
                                     int32_t* status, void* stream);

/*
 * Exact caller-owned workspace shapes for the hierarchical entry point, as
 * four (rows, cols) pairs in the order mapped, local_positions, tile_counts,
 * tile_offsets. Host only; touches no device. Replaces
 * silkern/workspace.py:22-53 (workspace_shapes).
 */
int silkern_workspace_shapes_v1(int64_t batch, int64_t width, int32_t tile_size,
                                int64_t out_shapes[8]);

/*
 * Row-wise or hierarchical localization with an explicit launch geometry, for
 * conformance sweeps and tuning: cluster_size CTAs per row (1, 2, 4 or 8),
 * stage_table = 1 stages the request's block-table row in shared memory
 * (table_width <= 4096), 0 gathers it from global memory, -1 lets the
 * library decide; prefetch_table likewise for the L2 bulk prefetch of the
 * whole table; chunks_per_thread (1, 2, 4 or 8; 0 = library choice) makes
 * each thread map a run of 4 x chunks_per_thread consecutive columns.
 * tile_size = 0 selects row-wise semantics (no workspace).
 * Same semantics and outputs as the entry points above. No counterpart in the
 * reference (its launch geometry is fixed inside each launcher).
 */
int silkern_localize_explicit_v1(const int32_t* req_ids, const int32_t* block_table,
                                 int64_t table_rows, int64_t table_width,
                                 const int32_t* tokens, int32_t* out, int32_t* counts,
                                 int32_t* tile_counts_ws, int32_t* tile_offsets_ws,
                                 int64_t batch, int64_t width, int32_t block_size,
                                 int32_t dcp_size, int32_t dcp_rank, int32_t dcp_interleave,
                                 int32_t compact_valid_to_front, int32_t tile_size,
                                 int32_t cluster_size, int32_t stage_table,
                                 int32_t prefetch_table, int32_t chunks_per_thread,
                                 int32_t* status, void* stream);

/*
 * Hierarchical localization for callers that cannot allocate device memory:
 * the same computation and outputs (out, counts) as
 * silkern_localize_hierarchical_v1, but without workspace arguments. Its
 * tile workspace (tile counts and tile offsets) lives in a fixed array inside
 * this library, SILKERN_NOALLOC_MAX_TILES entries for each, 256 KiB in total,
 * which every GPU that loads the library holds until the process exits.
 * Callers whose memory is planned outside their control use it: plugin hosts
 * and serving runtimes whose enqueue path forbids cudaMalloc, or code run
 * while another framework records a CUDA graph, where a new allocation would
 * break the recording or stall it.
 *   - batch * ceil(width / tile_size) above SILKERN_NOALLOC_MAX_TILES is
 *     rejected with SILKERN_E_SCRATCH before anything is launched;
 *   - the first call on a device looks up the array's device address with
 *     that device current, so make that first call before any stream capture;
 *   - every call shares the one array and leaves its tile decomposition there
 *     (nothing in it has to start at zero: each call writes every entry it
 *     uses before reading any), so calls that overlap on the GPU, from two
 *     streams or two threads, race on it and must be serialised.
 * Nothing is allocated or freed. No counterpart in the reference (its
 * hierarchical launcher always takes caller-owned workspace).
 */
#define SILKERN_NOALLOC_MAX_TILES 32768
int silkern_localize_hierarchical_noalloc_v1(const int32_t* req_ids, const int32_t* block_table,
                                             int64_t table_rows, int64_t table_width,
                                             const int32_t* tokens, int32_t* out,
                                             int32_t* counts, int64_t batch, int64_t width,
                                             int32_t block_size, int32_t dcp_size,
                                             int32_t dcp_rank, int32_t dcp_interleave,
                                             int32_t compact_valid_to_front, int32_t tile_size,
                                             int32_t* status, void* stream);

/*
 * Device-side equality check used by the CUDA-graph replay gate: adds the
 * number of positions i < n with a[i] != b[i] to *mismatches (one atomic add
 * per CTA). No counterpart in the reference (its replay check copies to the
 * host, silkern/verify.py:362-372).
 */
int silkern_count_mismatches_v1(const int32_t* a, const int32_t* b, int64_t n,
                                int32_t* mismatches, void* stream);

/*
 * silkern_count_mismatches_v1 per segment, for the decode-step replay gate:
 * a and b hold `segments` consecutive segments of segment_elems int32 each
 * (one per layer of a step), and counters[s] (int32, segments entries) is
 * increased by the number of positions of segment s where a and b differ.
 * One launch; segments <= 65535. No counterpart in the reference.
 */
int silkern_count_segment_mismatches_v1(const int32_t* a, const int32_t* b, int64_t segments,
                                        int64_t segment_elems, int32_t* counters, void* stream);

/*
 * Measurement reference, not the product: dst[0..n) = src[0..n) (int32) with
 * the converter's data movement and launch mode and none of its work. CTAs of
 * `threads` threads (a multiple of 32, at most 1024) each copy a contiguous
 * chunk of threads * run elements, each thread a run of `run` (8 or 16)
 * elements with 256-bit accesses where aligned; programmatic dependent launch,
 * with a bulk L2 prefetch of the chunk issued before the wait on the previous
 * grid. ctas_per_sm in 1..8 reserves shared memory so that at most that many
 * of these CTAs share an SM (the converter's residency control); 0 reserves
 * none. The time of back-to-back calls over the converter's tokens and output
 * is the floor a converter call of the same size runs against. src and dst
 * must not overlap (SILKERN_E_ALIAS). No counterpart in the reference.
 */
int silkern_copy_floor_v1(const int32_t* src, int32_t* dst, int64_t n, int32_t run, int32_t threads,
                          int32_t ctas_per_sm, void* stream);

/*
 * Comparison baseline, not the product: the atomic-reservation converter of
 * the reference's bench/atomic_baseline.py:40-111 and :313-385 (itself a
 * restatement of the upstream vLLM converter). Same set and counts as the
 * entry points above, but each 128-column tile reserves its output segment
 * with an atomicAdd on scratch[row] (int32, (batch,)), so the order of the
 * segments varies from run to run. Three stream operations: reset, reserve
 * and scatter, counts <- scratch.
 */
int silkern_atomic_baseline_v1(const int32_t* req_ids, const int32_t* block_table,
                               int64_t table_rows, int64_t table_width, const int32_t* tokens,
                               int32_t* out, int32_t* counts, int32_t* scratch, int64_t batch,
                               int64_t width, int32_t block_size, int32_t dcp_size,
                               int32_t dcp_rank, int32_t dcp_interleave, void* stream);

/*
 * Fused indexer top-k + localization: selection and conversion in one launch,
 * without the (batch, top_k) selection round trip through HBM. This is the
 * "fuse the converter into the indexer's top-k epilogue" step beyond the
 * reference's converter boundary; its localization half is the contract above
 * (silkern/contract.py:67-158), applied to the selected positions.
 *
 * logits is float32 (batch, logits_width) with row stride logits_stride
 * (elements, >= logits_width); row r scores the positions [0, L) with
 * L = seq_lens[r] (values outside [0, logits_width] are clamped and flagged
 * with SILKERN_STATUS_BAD_LENGTH); columns at and beyond L are never read.
 * Selection: every position when L <= top_k; otherwise the top_k positions
 * with the largest keys, where key(x) orders the float bit patterns totally
 * (-NaN < -inf < ... < -0 < +0 < ... < +inf < +NaN), ties going to the lower
 * position. The selected positions, in ascending order and padded with -1 to
 * top_k, form the selection row that is localized into out (batch, top_k)
 * and counts (batch,), exactly as silkern_localize_rowwise_v1 would localize
 * it. positions (batch, top_k) may be NULL; otherwise it receives that
 * selection row. 1 <= top_k <= SILKERN_MAX_ROW_WIDTH; logits_width <=
 * SILKERN_TOPK_MAX_WIDTH. One CTA per row: a sampled estimate of the
 * threshold, one streaming pass over the row that keeps candidate bit masks,
 * an exact radix select over the candidates in shared memory (or over the
 * whole row when the estimate misses), and the converter's compaction.
 */
#define SILKERN_TOPK_MAX_WIDTH 262144
int silkern_topk_localize_v1(const float* logits, int64_t logits_stride, int64_t logits_width,
                             const int32_t* seq_lens, const int32_t* req_ids,
                             const int32_t* block_table, int64_t table_rows, int64_t table_width,
                             int32_t* positions, int32_t* out, int32_t* counts, int64_t batch,
                             int32_t top_k, int32_t block_size, int32_t dcp_size, int32_t dcp_rank,
                             int32_t dcp_interleave, int32_t compact_valid_to_front,
                             int32_t* status, void* stream);

/*
 * silkern_topk_localize_v1 with explicit internals (tuning and test hook):
 * candidate_capacity entries in the shared-memory candidate list (0 =
 * automatic; top_k .. the shared-memory budget; a capacity of top_k sends
 * almost every row down the whole-row path) and stage_table (-1 automatic,
 * 0 gather the block table from global memory, 1 stage the request's row in
 * shared memory, which needs table_width <= 4096). SILKERN_E_GEOMETRY when
 * either is out of range.
 */
int silkern_topk_localize_explicit_v1(const float* logits, int64_t logits_stride,
                                      int64_t logits_width, const int32_t* seq_lens,
                                      const int32_t* req_ids, const int32_t* block_table,
                                      int64_t table_rows, int64_t table_width, int32_t* positions,
                                      int32_t* out, int32_t* counts, int64_t batch, int32_t top_k,
                                      int32_t block_size, int32_t dcp_size, int32_t dcp_rank,
                                      int32_t dcp_interleave, int32_t compact_valid_to_front,
                                      int32_t candidate_capacity, int32_t stage_table,
                                      int32_t* status, void* stream);

/*
 * silkern_topk_localize_explicit_v1 with the CTA shape pinned as well:
 * cta_threads 0 (automatic: 1024 threads, one CTA per SM, when batch is at
 * most the device's SM count, else 512 threads, two per SM), 512 or 1024.
 * SILKERN_E_GEOMETRY for any other value.
 */
int silkern_topk_localize_explicit_v2(const float* logits, int64_t logits_stride,
                                      int64_t logits_width, const int32_t* seq_lens,
                                      const int32_t* req_ids, const int32_t* block_table,
                                      int64_t table_rows, int64_t table_width, int32_t* positions,
                                      int32_t* out, int32_t* counts, int64_t batch, int32_t top_k,
                                      int32_t block_size, int32_t dcp_size, int32_t dcp_rank,
                                      int32_t dcp_interleave, int32_t compact_valid_to_front,
                                      int32_t candidate_capacity, int32_t stage_table,
                                      int32_t cta_threads, int32_t* status, void* stream);

/* Static text for a return code (positive SILKERN_E*, 0, or -cudaError_t). */
const char* silkern_status_string_v1(int code);

/* SILKERN_ABI_VERSION of the loaded library. */
int silkern_abi_version_v1(void);

/*
 * Host check of the invariant-divisor division the kernels use: returns the
 * number of n in [n_begin, n_begin + n_count) (all < 2^31) for which the fast
 * quotient differs from n / divisor. Test hook; touches no device.
 */
int64_t silkern_fastdiv_selftest_v1(uint32_t divisor, uint32_t n_begin, uint32_t n_count);

#ifdef __cplusplus
}
#endif

#endif /* SILKERN_B200_H_ */
