/*
 * A plain C program that uses the converter through its C ABI only: no torch,
 * no Python. It allocates device buffers with the CUDA runtime, calls the
 * row-wise, hierarchical and allocation-free hierarchical entry points on the
 * same seeded batch, and checks each result against the C oracle
 * (oracle/localize_oracle.c, test infrastructure). It then runs the fused
 * top-k + localization entry point on distinct scores, whose selection is
 * computed here by sorting, and localizes that selection with the oracle to
 * check the fused output. Exit status 0 = all equal.
 */
#include <cuda_runtime_api.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "silkern_b200.h"

int oracle_localize(const int32_t* req_ids, const int32_t* table, int64_t table_rows,
                    int64_t table_width, const int32_t* tokens, int32_t* out, int32_t* counts,
                    int64_t batch, int64_t width, int64_t block_size, int64_t dcp_size,
                    int64_t dcp_rank, int64_t interleave, int compact_valid_to_front, int threads);

#define CHECK_CUDA(x)                                                        \
  do {                                                                       \
    cudaError_t e_ = (x);                                                    \
    if (e_ != cudaSuccess) {                                                 \
      fprintf(stderr, "%s: %s\n", #x, cudaGetErrorString(e_));              \
      return 2;                                                              \
    }                                                                        \
  } while (0)

static uint64_t lcg_state = 0x9E3779B97F4A7C15ull;
static uint32_t lcg(void) {
  lcg_state = lcg_state * 6364136223846793005ull + 1442695040888963407ull;
  return (uint32_t)(lcg_state >> 33);
}

/* Scores of the fused check: distinct per row, the top ones spread out. */
static const float* g_scores;
static int by_score_desc(const void* a, const void* b) {
  const float x = g_scores[*(const int32_t*)a], y = g_scores[*(const int32_t*)b];
  return (x < y) - (x > y);
}
static int by_value(const void* a, const void* b) {
  const int32_t x = *(const int32_t*)a, y = *(const int32_t*)b;
  return (x > y) - (x < y);
}

static int compare(const char* what, const int32_t* got, const int32_t* want, size_t n) {
  for (size_t i = 0; i < n; ++i) {
    if (got[i] != want[i]) {
      fprintf(stderr, "%s: mismatch at %zu: %d != %d\n", what, i, got[i], want[i]);
      return 1;
    }
  }
  return 0;
}

int main(void) {
  const int64_t batch = 37, width = 3000, rows = 41, twidth = 90;
  const int32_t block_size = 64, dcp_size = 4, interleave = 1, tile = 256;
  const size_t nt = (size_t)(batch * width);
  int32_t* req = malloc(sizeof(int32_t) * batch);
  int32_t* table = malloc(sizeof(int32_t) * rows * twidth);
  int32_t* tokens = malloc(sizeof(int32_t) * nt);
  int32_t* out = malloc(sizeof(int32_t) * nt);
  int32_t* counts = malloc(sizeof(int32_t) * batch);
  int32_t* want = malloc(sizeof(int32_t) * nt);
  int32_t* want_counts = malloc(sizeof(int32_t) * batch);
  for (int64_t i = 0; i < batch; ++i) req[i] = (int32_t)(lcg() % rows);
  for (int64_t i = 0; i < rows * twidth; ++i) table[i] = (int32_t)(lcg() % 100000) - 3;
  for (size_t i = 0; i < nt; ++i) tokens[i] = (int32_t)(lcg() % (block_size * twidth * dcp_size + 500)) - 5;

  int32_t *d_req, *d_table, *d_tokens, *d_out, *d_counts, *d_tc, *d_to;
  const int64_t tiles = (width + tile - 1) / tile;
  CHECK_CUDA(cudaMalloc((void**)&d_req, sizeof(int32_t) * batch));
  CHECK_CUDA(cudaMalloc((void**)&d_table, sizeof(int32_t) * rows * twidth));
  CHECK_CUDA(cudaMalloc((void**)&d_tokens, sizeof(int32_t) * nt));
  CHECK_CUDA(cudaMalloc((void**)&d_out, sizeof(int32_t) * nt));
  CHECK_CUDA(cudaMalloc((void**)&d_counts, sizeof(int32_t) * batch));
  CHECK_CUDA(cudaMalloc((void**)&d_tc, sizeof(int32_t) * batch * tiles));
  CHECK_CUDA(cudaMalloc((void**)&d_to, sizeof(int32_t) * batch * tiles));
  CHECK_CUDA(cudaMemcpy(d_req, req, sizeof(int32_t) * batch, cudaMemcpyHostToDevice));
  CHECK_CUDA(cudaMemcpy(d_table, table, sizeof(int32_t) * rows * twidth, cudaMemcpyHostToDevice));
  CHECK_CUDA(cudaMemcpy(d_tokens, tokens, sizeof(int32_t) * nt, cudaMemcpyHostToDevice));
  cudaStream_t stream;
  CHECK_CUDA(cudaStreamCreate(&stream));

  int failures = 0;
  for (int32_t rank = 0; rank < dcp_size; ++rank) {
    if (oracle_localize(req, table, rows, twidth, tokens, want, want_counts, batch, width, block_size,
                        dcp_size, rank, interleave, 1, 4) != 0) {
      fprintf(stderr, "oracle rejected the case\n");
      return 3;
    }
    for (int arm = 0; arm < 3; ++arm) {
      CHECK_CUDA(cudaMemsetAsync(d_out, 0x5A, sizeof(int32_t) * nt, stream));
      int rc;
      if (arm == 0) {
        rc = silkern_localize_rowwise_v1(d_req, d_table, rows, twidth, d_tokens, d_out, d_counts, batch,
                                         width, block_size, dcp_size, rank, interleave, 1, NULL, stream);
      } else if (arm == 1) {
        rc = silkern_localize_hierarchical_v1(d_req, d_table, rows, twidth, d_tokens, d_out, d_counts, NULL,
                                              NULL, d_tc, d_to, batch, width, block_size, dcp_size, rank,
                                              interleave, 1, tile, NULL, stream);
      } else {
        rc = silkern_localize_hierarchical_noalloc_v1(d_req, d_table, rows, twidth, d_tokens, d_out,
                                                      d_counts, batch, width, block_size, dcp_size, rank,
                                                      interleave, 1, tile, NULL, stream);
      }
      if (rc != SILKERN_OK) {
        fprintf(stderr, "arm %d rank %d: %s\n", arm, rank, silkern_status_string_v1(rc));
        return 4;
      }
      CHECK_CUDA(cudaMemcpyAsync(out, d_out, sizeof(int32_t) * nt, cudaMemcpyDeviceToHost, stream));
      CHECK_CUDA(cudaMemcpyAsync(counts, d_counts, sizeof(int32_t) * batch, cudaMemcpyDeviceToHost, stream));
      CHECK_CUDA(cudaStreamSynchronize(stream));
      failures += compare("out", out, want, nt) + compare("counts", counts, want_counts, (size_t)batch);
    }
  }
  if (silkern_localize_rowwise_v1(d_req, d_table, rows, twidth, d_tokens, d_tokens, d_counts, batch, width,
                                  block_size, dcp_size, 0, interleave, 1, NULL, stream) != SILKERN_E_ALIAS) {
    fprintf(stderr, "aliased output was not rejected\n");
    ++failures;
  }

  /* fused top-k + localization: scores (batch, lw), row lengths, top k */
  {
    const int64_t lw = 9000;
    const int32_t k = 700;
    float* scores = malloc(sizeof(float) * batch * lw);
    int32_t* lens = malloc(sizeof(int32_t) * batch);
    int32_t* sel = malloc(sizeof(int32_t) * batch * k);
    int32_t* order = malloc(sizeof(int32_t) * lw);
    int32_t* fout = malloc(sizeof(int32_t) * batch * k);
    int32_t* fwant = malloc(sizeof(int32_t) * batch * k);
    for (int64_t r = 0; r < batch; ++r) {
      lens[r] = (int32_t)(lcg() % (lw + 1));
      for (int64_t c = 0; c < lw; ++c) scores[r * lw + c] = (float)((c * 7919 + r * 31) % lw) - 4000.0f;
      g_scores = scores + r * lw;
      for (int32_t c = 0; c < lens[r]; ++c) order[c] = c;
      const int32_t n = lens[r] < k ? lens[r] : k;
      if (lens[r] > k) qsort(order, (size_t)lens[r], sizeof(int32_t), by_score_desc);
      qsort(order, (size_t)n, sizeof(int32_t), by_value); /* the selection row: ascending positions */
      for (int32_t j = 0; j < k; ++j) sel[r * k + j] = j < n ? order[j] : -1;
    }
    float* d_scores;
    int32_t *d_lens, *d_fout, *d_fcounts;
    CHECK_CUDA(cudaMalloc((void**)&d_scores, sizeof(float) * batch * lw));
    CHECK_CUDA(cudaMalloc((void**)&d_lens, sizeof(int32_t) * batch));
    CHECK_CUDA(cudaMalloc((void**)&d_fout, sizeof(int32_t) * batch * k));
    CHECK_CUDA(cudaMalloc((void**)&d_fcounts, sizeof(int32_t) * batch));
    CHECK_CUDA(cudaMemcpy(d_scores, scores, sizeof(float) * batch * lw, cudaMemcpyHostToDevice));
    CHECK_CUDA(cudaMemcpy(d_lens, lens, sizeof(int32_t) * batch, cudaMemcpyHostToDevice));
    const int32_t rank = 1;
    if (oracle_localize(req, table, rows, twidth, sel, fwant, want_counts, batch, k, block_size, dcp_size, rank,
                        interleave, 1, 4) != 0) {
      fprintf(stderr, "oracle rejected the fused case\n");
      return 3;
    }
    const int rc = silkern_topk_localize_v1(d_scores, lw, lw, d_lens, d_req, d_table, rows, twidth, NULL, d_fout,
                                            d_fcounts, batch, k, block_size, dcp_size, rank, interleave, 1, NULL,
                                            stream);
    if (rc != SILKERN_OK) {
      fprintf(stderr, "fused: %s\n", silkern_status_string_v1(rc));
      return 4;
    }
    CHECK_CUDA(cudaMemcpyAsync(fout, d_fout, sizeof(int32_t) * batch * k, cudaMemcpyDeviceToHost, stream));
    CHECK_CUDA(cudaMemcpyAsync(counts, d_fcounts, sizeof(int32_t) * batch, cudaMemcpyDeviceToHost, stream));
    CHECK_CUDA(cudaStreamSynchronize(stream));
    failures += compare("fused out", fout, fwant, (size_t)(batch * k)) +
                compare("fused counts", counts, want_counts, (size_t)batch);
    if (silkern_topk_localize_v1(NULL, lw, lw, d_lens, d_req, d_table, rows, twidth, NULL, d_fout, d_fcounts,
                                 batch, k, block_size, dcp_size, rank, interleave, 1, NULL, stream) != SILKERN_E_NULL) {
      fprintf(stderr, "NULL logits were not rejected\n");
      ++failures;
    }
  }
  printf("%s (abi %d)\n", failures ? "FAILED" : "ok", silkern_abi_version_v1());
  return failures ? 1 : 0;
}
