// Atomic-reservation converter: the comparison baseline, not the product.
//
// Restates the algorithm of the reference's bench/atomic_baseline.py:40-111,
// which in turn restates the upstream vLLM converter: per tile of 128
// columns, a tile-local scan, then one atomicAdd on a per-row counter reserves
// the tile's output segment, then the tile's survivors are scattered into it.
// The set of survivors and the count are exact; the order of the tiles'
// segments in the row is whatever order the atomics landed in, which varies
// from run to run. It exists to be timed beside the stable kernel and to show
// that instability.
#include <cuda_runtime.h>

#include <cstdint>

#include "fastdiv.cuh"
#include "silkern_b200.h"

namespace silkern {
namespace {

constexpr int kTile = 128;  // BLOCK_N of the reference baseline

struct AtomicParams {
  const int32_t* req_ids;
  const int32_t* table;
  const int32_t* tokens;
  int32_t* out;
  int32_t* scratch;
  int64_t table_rows;
  uint32_t table_width;
  int32_t width;
  int32_t tiles;
  uint32_t dcp_rank, dcp_size, interleave, block_size;
  FastDiv div_il, div_dcp, div_bs;
};

// out <- -1, scratch <- 0 (bench/atomic_baseline.py:40-44).
__global__ void atomic_reset_kernel(int32_t* out, int64_t elements, int32_t* scratch, int64_t batch) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < elements; i += stride) {
    out[i] = -1;
  }
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < batch; i += stride) {
    scratch[i] = 0;
  }
}

// One CTA per (row, tile): map, tile-local scan, reserve, scatter
// (bench/atomic_baseline.py:46-111).
__global__ void __launch_bounds__(kTile) atomic_reserve_kernel(const __grid_constant__ AtomicParams p) {
  __shared__ int s_warp[kTile / 32];
  __shared__ int s_base;
  const int64_t row = blockIdx.x / static_cast<uint32_t>(p.tiles);
  const int tile = static_cast<int>(blockIdx.x - row * p.tiles);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int col = tile * kTile + tid;
  const int32_t t = col < p.width ? p.tokens[row * p.width + col] : -1;
  const int32_t req = p.req_ids[row];
  const bool req_ok = req >= 0 && static_cast<int64_t>(req) < p.table_rows;
  bool valid = false;
  int32_t phys = -1;
  if (t >= 0 && req_ok) {
    const uint32_t u = static_cast<uint32_t>(t);
    const uint32_t q1 = fastdiv(u, p.div_il);
    const uint32_t q2 = fastdiv(q1, p.div_dcp);
    const uint32_t local = q2 * p.interleave + (u - q1 * p.interleave);
    const uint32_t lb = fastdiv(local, p.div_bs);
    if (q1 - q2 * p.dcp_size == p.dcp_rank && lb < p.table_width) {
      const int32_t blk = p.table[static_cast<int64_t>(req) * p.table_width + lb];
      phys = static_cast<int32_t>(static_cast<uint32_t>(blk) * p.block_size + (local - lb * p.block_size));
      valid = true;
    }
  }
  const uint32_t ballot = __ballot_sync(0xffffffffu, valid);
  const int in_warp = __popc(ballot & ((1u << lane) - 1u));
  if (lane == 0) s_warp[warp] = __popc(ballot);
  __syncthreads();
  int before = 0, total = 0;
  for (int w = 0; w < kTile / 32; ++w) {
    before += w < warp ? s_warp[w] : 0;
    total += s_warp[w];
  }
  if (tid == 0) s_base = total ? atomicAdd(p.scratch + row, total) : 0;  // the reservation
  __syncthreads();
  if (valid) p.out[row * p.width + s_base + before + in_warp] = phys;
}

}  // namespace
}  // namespace silkern

extern "C" int silkern_atomic_baseline_v1(const int32_t* req_ids, const int32_t* block_table,
                                          int64_t table_rows, int64_t table_width,
                                          const int32_t* tokens, int32_t* out, int32_t* counts,
                                          int32_t* scratch, int64_t batch, int64_t width,
                                          int32_t block_size, int32_t dcp_size, int32_t dcp_rank,
                                          int32_t dcp_interleave, void* stream) {
  using namespace silkern;
  if (!req_ids || !block_table || !tokens || !out || !counts || !scratch) return SILKERN_E_NULL;
  if (batch < 1 || width < 1 || width > SILKERN_MAX_ROW_WIDTH || table_rows < 1 || table_width < 1 ||
      table_width > INT32_MAX || batch > (int64_t{1} << 20)) {
    return SILKERN_E_SHAPE;
  }
  if (dcp_size < 1 || dcp_rank < 0 || dcp_rank >= dcp_size || dcp_interleave < 1) return SILKERN_E_DCP;
  if (block_size < 1 || block_size % dcp_interleave != 0) return SILKERN_E_BLOCK_SIZE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  AtomicParams p{};
  p.req_ids = req_ids;
  p.table = block_table;
  p.tokens = tokens;
  p.out = out;
  p.scratch = scratch;
  p.table_rows = table_rows;
  p.table_width = static_cast<uint32_t>(table_width);
  p.width = static_cast<int32_t>(width);
  p.tiles = static_cast<int32_t>((width + kTile - 1) / kTile);
  p.dcp_rank = static_cast<uint32_t>(dcp_rank);
  p.dcp_size = static_cast<uint32_t>(dcp_size);
  p.interleave = static_cast<uint32_t>(dcp_interleave);
  p.block_size = static_cast<uint32_t>(block_size);
  p.div_il = make_fastdiv(p.interleave);
  p.div_dcp = make_fastdiv(p.dcp_size);
  p.div_bs = make_fastdiv(p.block_size);
  const int64_t elements = batch * width;
  int64_t reset_blocks = (elements + 255) / 256;
  if (reset_blocks > 4096) reset_blocks = 4096;
  atomic_reset_kernel<<<static_cast<unsigned>(reset_blocks), 256, 0, s>>>(out, elements, scratch, batch);
  atomic_reserve_kernel<<<static_cast<unsigned>(batch * p.tiles), kTile, 0, s>>>(p);
  // counts.copy_(scratch) (bench/atomic_baseline.py:186)
  cudaError_t err = cudaMemcpyAsync(counts, scratch, sizeof(int32_t) * batch, cudaMemcpyDeviceToDevice, s);
  if (err == cudaSuccess) err = cudaGetLastError();
  if (err != cudaSuccess) {
    (void)cudaGetLastError();
    return -static_cast<int>(err);
  }
  return SILKERN_OK;
}
