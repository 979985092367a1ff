/*
 * CPU oracle for the localization converter -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference's normative loop,
 * silkern/contract.py:67-158 (localize_reference), used by the tests and by
 * the bench's CPU baseline to check and time the CUDA path. Nothing in the
 * product links or calls it.
 *
 * Arithmetic: tokens are int32 and every intermediate is computed in int64
 * exactly as Python integers would be (contract.py:138-147). The physical
 * slot table_row[lb] * block_size + offset is stored as int32, wrapping mod
 * 2^32 like the int32 lanes of the reference's Triton kernel
 * (silkern/kernels.py:101); the Python oracle agrees whenever it fits.
 *
 * Return: 0, or ORACLE_E_REQUEST when a request id is outside the table
 * (contract.py:129-130 raises there), or ORACLE_E_ARGS for a configuration
 * contract.py:50-122 rejects.
 */
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>

#define ORACLE_OK 0
#define ORACLE_E_ARGS 1
#define ORACLE_E_REQUEST 2

typedef struct {
  const int32_t* req_ids;
  const int32_t* table;
  int64_t table_rows;
  int64_t table_width;
  const int32_t* tokens;
  int32_t* out;
  int32_t* counts;
  int64_t width;
  int64_t block_size;
  int64_t dcp_size;
  int64_t dcp_rank;
  int64_t interleave;
  int compact;
  int64_t row_begin;
  int64_t row_end;
  int status;
} oracle_job;

/* Python floor division and modulo for a >= 0, b > 0 (contract.py uses //, %). */
static inline int64_t fdiv(int64_t a, int64_t b) { return a / b; }

static void run_rows(oracle_job* job) {
  const int64_t group = job->dcp_size * job->interleave;
  for (int64_t row = job->row_begin; row < job->row_end; ++row) {
    const int64_t request = job->req_ids[row];
    if (request < 0 || request >= job->table_rows) { /* contract.py:129-130 */
      job->status = ORACLE_E_REQUEST;
      return;
    }
    const int32_t* entries = job->table + request * job->table_width;
    const int32_t* src = job->tokens + row * job->width;
    int32_t* dst = job->out + row * job->width;
    int64_t kept = 0;
    for (int64_t col = 0; col < job->width; ++col) {
      const int64_t token = src[col];
      int64_t value = -1;
      int valid = 0;
      if (token >= 0) { /* contract.py:138 */
        const int64_t owner = fdiv(token, job->interleave) % job->dcp_size; /* :139 */
        if (owner == job->dcp_rank) {
          const int64_t local =
              fdiv(token, group) * job->interleave + token % job->interleave; /* :141-143 */
          const int64_t logical_block = fdiv(local, job->block_size);       /* :144 */
          const int64_t offset = local % job->block_size;
          if (logical_block < job->table_width) { /* :145 */
            value = (int64_t)entries[logical_block] * job->block_size + offset; /* :146-147 */
            valid = 1;
          }
        }
      }
      const int32_t stored = (int32_t)(uint32_t)(uint64_t)value;
      if (job->compact) {
        if (valid) dst[kept] = stored; /* :150-151, :155 */
      } else {
        dst[col] = stored; /* :149, :157 */
      }
      kept += valid;
    }
    if (job->compact) {
      for (int64_t col = kept; col < job->width; ++col) dst[col] = -1; /* :155 */
    }
    job->counts[row] = (int32_t)kept; /* :153 */
  }
}

static void* worker(void* arg) {
  run_rows((oracle_job*)arg);
  return NULL;
}

/* contract.py:50-122: the configuration checks that do not depend on list shapes. */
static int check_args(int64_t batch, int64_t width, int64_t table_rows, int64_t table_width,
                      int64_t block_size, int64_t dcp_size, int64_t dcp_rank, int64_t interleave) {
  if (dcp_size < 1 || dcp_rank < 0 || dcp_rank >= dcp_size || interleave < 1) return ORACLE_E_ARGS;
  if (block_size < 1 || block_size % interleave != 0) return ORACLE_E_ARGS;
  if (batch < 1 || width < 1 || table_rows < 1 || table_width < 1) return ORACLE_E_ARGS;
  return ORACLE_OK;
}

int oracle_localize(const int32_t* req_ids, const int32_t* table, int64_t table_rows,
                    int64_t table_width, const int32_t* tokens, int32_t* out, int32_t* counts,
                    int64_t batch, int64_t width, int64_t block_size, int64_t dcp_size,
                    int64_t dcp_rank, int64_t interleave, int compact_valid_to_front,
                    int threads) {
  const int rc = check_args(batch, width, table_rows, table_width, block_size, dcp_size, dcp_rank,
                            interleave);
  if (rc != ORACLE_OK) return rc;
  if (threads < 1) threads = 1;
  if (threads > batch) threads = (int)batch;
  oracle_job* jobs = (oracle_job*)calloc((size_t)threads, sizeof(oracle_job));
  pthread_t* handles = (pthread_t*)calloc((size_t)threads, sizeof(pthread_t));
  if (!jobs || !handles) {
    free(jobs);
    free(handles);
    return ORACLE_E_ARGS;
  }
  const int compact = compact_valid_to_front && dcp_size > 1; /* contract.py:126 */
  for (int t = 0; t < threads; ++t) {
    oracle_job* job = &jobs[t];
    job->req_ids = req_ids;
    job->table = table;
    job->table_rows = table_rows;
    job->table_width = table_width;
    job->tokens = tokens;
    job->out = out;
    job->counts = counts;
    job->width = width;
    job->block_size = block_size;
    job->dcp_size = dcp_size;
    job->dcp_rank = dcp_rank;
    job->interleave = interleave;
    job->compact = compact;
    job->row_begin = batch * t / threads;
    job->row_end = batch * (t + 1) / threads;
    job->status = ORACLE_OK;
  }
  int started = 0;
  for (int t = 1; t < threads; ++t) {
    if (pthread_create(&handles[t], NULL, worker, &jobs[t]) != 0) break;
    started = t;
  }
  run_rows(&jobs[0]);
  for (int t = 1; t <= started; ++t) pthread_join(handles[t], NULL);
  for (int t = started + 1; t < threads; ++t) run_rows(&jobs[t]);
  int status = ORACLE_OK;
  for (int t = 0; t < threads; ++t) {
    if (jobs[t].status != ORACLE_OK) status = jobs[t].status;
  }
  free(jobs);
  free(handles);
  return status;
}

/* Tile decomposition published by the hierarchical path (the reference's
 * _map_tiles_kernel writes tile_counts, silkern/kernels.py:203-208, and
 * _tile_prefix_kernel the exclusive prefix, :240-247): per row and tile of
 * tile_size columns, the number of valid elements and their row prefix. */
int oracle_tiles(const int32_t* req_ids, const int32_t* table, int64_t table_rows,
                 int64_t table_width, const int32_t* tokens, int32_t* tile_counts,
                 int32_t* tile_offsets, int64_t batch, int64_t width, int64_t block_size,
                 int64_t dcp_size, int64_t dcp_rank, int64_t interleave, int64_t tile_size) {
  const int rc = check_args(batch, width, table_rows, table_width, block_size, dcp_size, dcp_rank,
                            interleave);
  if (rc != ORACLE_OK || tile_size < 1) return ORACLE_E_ARGS;
  const int64_t tiles = (width + tile_size - 1) / tile_size;
  const int64_t group = dcp_size * interleave;
  for (int64_t row = 0; row < batch; ++row) {
    const int64_t request = req_ids[row];
    if (request < 0 || request >= table_rows) return ORACLE_E_REQUEST;
    const int32_t* src = tokens + row * width;
    int64_t prefix = 0;
    for (int64_t tile = 0; tile < tiles; ++tile) {
      int64_t count = 0;
      const int64_t end = (tile + 1) * tile_size < width ? (tile + 1) * tile_size : width;
      for (int64_t col = tile * tile_size; col < end; ++col) {
        const int64_t token = src[col];
        if (token < 0 || fdiv(token, interleave) % dcp_size != dcp_rank) continue;
        const int64_t local = fdiv(token, group) * interleave + token % interleave;
        if (fdiv(local, block_size) < table_width) ++count;
      }
      tile_counts[row * tiles + tile] = (int32_t)count;
      tile_offsets[row * tiles + tile] = (int32_t)prefix;
      prefix += count;
    }
  }
  return ORACLE_OK;
}
