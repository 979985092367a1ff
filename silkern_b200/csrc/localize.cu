// Sparse-index localization for decode context parallelism on B200 (sm_100a).
//
// One kernel family serves both public entry points. A row of `width`
// selected token positions is split into `cluster` contiguous column slices;
// each slice is one CTA, and the CTAs of one row form a thread-block cluster
// (cluster == 1 for the common row-wise case, where several rows can share a
// CTA as independent row groups). Each thread owns a run of G consecutive
// columns of its slice (G = 4, 8, 16 or 32). Per CTA:
//
//   0. before waiting on the previous grid (programmatic dependent launch),
//      ask L2 for this slice's tokens, the row's request id and this CTA's
//      share of the block table. A prefetch only fills L2, which is the
//      device's point of coherence, so it never returns stale data: loads
//      issued after the wait see every write of the previous grid. Call
//      N + 1 therefore reads DRAM while call N is still running;
//   1. read the request id, the thread's run of tokens (one 256-bit load per
//      eight columns when the run is 32-byte aligned) and, when the table is
//      staged (an explicit option; the default gathers from L2), the
//      request's block-table row into shared memory in the same wave
//      (speculating that row r belongs to request r, repaired when not);
//   2. apply ownership and deinterleave: with interleave 1 and powers of two,
//      one rotate and one unsigned compare decide ownership, sign and table
//      bounds together; otherwise shifts or invariant-divisor multiplies;
//   3. stable compaction: each thread counts its valid elements, ballots over
//      the count's bits give each thread its exclusive prefix in the warp,
//      warp totals go through shared memory and one redux.sync gives each
//      warp its base; across a cluster, each CTA stores its total into every
//      CTA's shared memory (DSMEM, st.async) and each CTA waits, with a bound,
//      on its own transaction barrier for all of them. No atomics, so the
//      order is the selector's order on every run;
//   4. paged translation: each valid element reads its block from the staged
//      table row (or, unstaged, from the L2 gather issued in step 2);
//   5. a row that is one CTA's is staged in shared memory at its final
//      positions and written run by run, each thread storing its own
//      columns (survivors, then -1 past the count) with 256-bit stores;
//      across a cluster, each CTA stores its survivors after its row offset
//      and fills the -1 tail of its own slice. Every output element is
//      written exactly once.
//
// Semantics follow silkern/contract.py:67-158 (localize_reference) and the
// int32 lanes of silkern/kernels.py:51-125 (_rowwise_kernel).
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <mutex>

#include "fastdiv.cuh"
#include "ptx.cuh"
#include "silkern_b200.h"

namespace silkern {

constexpr int kMaxThreads = 512;      // threads per CTA (row groups, or one cluster slice)
constexpr int kMaxCluster = 8;
// Polls of a CTA's count-exchange barrier before it gives up (each poll may
// suspend the thread for a while); the exchange completes within a few
// microseconds, so only a broken cluster ever reaches the bound.
constexpr uint32_t kExchangePolls = 1u << 16;
constexpr int kTableStageMax = 4096;  // block-table entries staged in shared memory
constexpr int kSmemMax = 200 * 1024;      // dynamic shared memory per CTA, any launch
constexpr uint32_t kFull = 0xffffffffu;
constexpr int kModeGeneral = 0;  // invariant-divisor multiplies
constexpr int kModePow2 = 1;     // interleave, dcp_size, block_size powers of two
constexpr int kModePow2Il1 = 2;  // ... and interleave 1: rotate + one compare

struct Params {
  const int32_t* req_ids;
  const int32_t* table;
  const int32_t* tokens;
  int32_t* out;
  int32_t* counts;
  int32_t* tile_counts;   // hierarchical workspace, or nullptr
  int32_t* tile_offsets;  // hierarchical workspace, or nullptr
  int32_t* status;        // optional error word
  int64_t table_rows;
  uint64_t table_bytes;   // bytes of the block table covered by the L2 prefetch
  uint32_t table_chunk;   // per-CTA share of that prefetch (multiple of 16), 0 = off
  uint32_t table_width;
  uint32_t local_limit;   // interleave-1 mode: a valid element's local position is below this
  int32_t width;
  int32_t slice;          // columns per CTA
  int32_t cluster;        // CTAs per row
  int32_t tile_shift;     // log2(tile_size) when publishing tiles, else -1
  int32_t tiles_per_row;
  int32_t smem_group;     // ints of dynamic shared memory per row group
  int32_t smem_out;       // offset of the staged output in a group's region
  int32_t smem_wt;        // offset of the warp totals
  int32_t smem_tile;      // offset of the tile offsets
  int32_t row_threads;    // threads per row group (a power of two without a cluster)
  int32_t row_threads_shift;
  int32_t rows_base;      // rows per CTA: rows_base, plus one for the first rows_extra CTAs
  int32_t rows_extra;
  uint32_t dcp_rank;
  uint32_t dcp_size;
  uint32_t interleave;
  uint32_t block_size;
  // general path
  FastDiv div_il, div_dcp, div_bs;
  // all-powers-of-two paths
  uint32_t il_shift, dcp_shift, group_shift, bs_shift;
  uint32_t il_mask, dcp_mask, bs_mask;
};

// v[0..G) = src[0..n) and -1 past n (n may be <= 0): 256-bit loads when the
// run is whole and 32-byte aligned, 128-bit when 16-byte aligned, else scalar.
template <int G>
__device__ __forceinline__ void load_run(const int32_t* src, int n, int32_t (&v)[G]) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(src);
  if (n >= G && (G % 8 == 0) && (a & 31u) == 0) {
#pragma unroll
    for (int i = 0; i < G / 8; ++i) {
      int32_t q[8];
      ld_nc_v8(src + 8 * i, q);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[8 * i + j] = q[j];
    }
  } else if (n >= G && (a & 15u) == 0) {
#pragma unroll
    for (int i = 0; i < G / 4; ++i) {
      const int4 q = __ldg(reinterpret_cast<const int4*>(src) + i);
      v[4 * i + 0] = q.x;
      v[4 * i + 1] = q.y;
      v[4 * i + 2] = q.z;
      v[4 * i + 3] = q.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < G; ++j) v[j] = j < n ? __ldg(src + j) : -1;
  }
}

// dst[0..min(n, G)) = w[0..): the widest aligned stores the run allows.
template <int G>
__device__ __forceinline__ void store_run(int32_t* dst, int n, const int32_t (&w)[G]) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(dst);
  if (n >= G && (G % 8 == 0) && (a & 31u) == 0) {
#pragma unroll
    for (int i = 0; i < G / 8; ++i) {
      int32_t q[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) q[j] = w[8 * i + j];
      st_v8(dst + 8 * i, q);
    }
  } else if (n >= G && (a & 15u) == 0) {
#pragma unroll
    for (int i = 0; i < G / 4; ++i) {
      reinterpret_cast<int4*>(dst)[i] = make_int4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
    }
  } else {
#pragma unroll
    for (int j = 0; j < G; ++j) {
      if (j < n) dst[j] = w[j];
    }
  }
}

// Exclusive prefix of c over the lanes of the warp, from one ballot per bit
// of c (c < 2^BITS).
template <int BITS>
__device__ __forceinline__ int warp_exclusive(uint32_t c) {
  const uint32_t lt = lanemask_lt();
  int e = 0;
#pragma unroll
  for (int b = 0; b < BITS; ++b) e += __popc(__ballot_sync(kFull, (c >> b) & 1u) & lt) << b;
  return e;
}

__host__ __device__ constexpr int count_bits(int g) { return g < 2 ? 1 : 1 + count_bits(g >> 1); }

// G columns per thread; CLUSTER: rows split over a cluster; MODE: general
// arithmetic, all powers of two, or all powers of two with interleave 1;
// COMPACT: valid values go to the front of the row; STAGE: the request's
// block-table row is staged in shared memory and read only for valid
// elements, instead of gathered from L2 for every element.
//
// Without a cluster a CTA holds p.rows_base or p.rows_base + 1 consecutive
// rows, one group of p.row_threads threads per row (each group with its own
// shared-memory region): one row, except narrow rows of large batches, which
// share a CTA of at least 128 threads. Up to four rows per SM the host's
// shared-memory reservation bounds how many CTAs share an SM, so under
// programmatic dependent launch the next call's CTAs spread over the SMs
// instead of piling onto the ones this call left room on.
template <int G, bool CLUSTER, int MODE, bool COMPACT, bool STAGE>
__global__ void __launch_bounds__(kMaxThreads, (CLUSTER || G > 16) ? 1 : 2)
    localize_kernel(const __grid_constant__ Params p) {
  // per row group: [staged table row][staged output][warp totals][tile offsets]
  extern __shared__ __align__(16) int32_t smem[];
  __shared__ int32_t s_cta_total[kMaxCluster];
  __shared__ __align__(8) uint64_t s_xbar;  // the cluster's count exchange

  int nthreads, tid, group;
  int64_t row;
  int crank;
  bool active;
  if constexpr (CLUSTER) {
    nthreads = blockDim.x;
    tid = threadIdx.x;
    group = 0;
    row = cluster_id_x();
    crank = static_cast<int>(cluster_ctarank());
    active = true;
    if (threadIdx.x == 0) {
      // Completes when this thread has arrived and 4 bytes (one CTA total)
      // have landed from every CTA of the cluster, this one included.
      mbar_init_cluster(&s_xbar, 1);
      mbar_arrive_expect_tx(&s_xbar, 4u * static_cast<uint32_t>(p.cluster));
    }
    cluster_arrive_relaxed();  // phase 0: this CTA is resident, its barrier initialised
  } else {
    nthreads = p.row_threads;
    group = static_cast<int>(threadIdx.x >> p.row_threads_shift);
    tid = static_cast<int>(threadIdx.x) & (nthreads - 1);
    const int extra = static_cast<int>(blockIdx.x) < p.rows_extra ? 1 : 0;
    const int64_t first = static_cast<int64_t>(blockIdx.x) * p.rows_base +
                          min(static_cast<int>(blockIdx.x), p.rows_extra);
    active = group < p.rows_base + extra;
    row = first + (active ? group : 0);
    crank = 0;
  }
  const int nwarps = nthreads >> 5;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  int32_t* gsmem = smem + group * p.smem_group;
  int32_t* s_tbl = gsmem;
  int32_t* s_wt = gsmem + p.smem_wt;
  int32_t* s_tile = gsmem + p.smem_tile;
  pdl_launch_dependents();

  const int c0 = crank * p.slice;
  const int len = active ? min(p.slice, p.width - c0) : 0;
  const int32_t* tok = p.tokens + row * p.width + c0;

  if (tid == 0 && active) {
    prefetch_l2_line(p.req_ids + row);
    const uintptr_t lo = (reinterpret_cast<uintptr_t>(tok) + 15u) & ~uintptr_t{15};
    const uintptr_t hi = reinterpret_cast<uintptr_t>(tok + len) & ~uintptr_t{15};
    if (hi > lo) prefetch_l2_bulk(reinterpret_cast<const void*>(lo), static_cast<uint32_t>(hi - lo));
    if (p.table_chunk != 0 && group == 0) {
      const uint64_t begin = static_cast<uint64_t>(blockIdx.x) * p.table_chunk;
      if (begin < p.table_bytes) {
        const uint64_t end = begin + p.table_chunk < p.table_bytes ? begin + p.table_chunk : p.table_bytes;
        prefetch_l2_bulk(reinterpret_cast<const char*>(p.table) + begin, static_cast<uint32_t>(end - begin));
      }
    }
  }

  pdl_wait();  // everything below may read what the previous grid wrote

  const int32_t req = __ldg(p.req_ids + row);
  const int col = tid * G;  // this thread's first column inside the slice
  int32_t v[G];
  load_run<G>(tok + col, len - col, v);
  const uint32_t tw = p.table_width;
  // Staged table: speculate that row r belongs to request r (one selection
  // row per request, in order) and load that table row in the same wave as
  // the tokens; it is repaired below once the request id is known.
  const int64_t spec = row < p.table_rows ? row : 0;
  int32_t t0 = 0;
  if constexpr (STAGE) {
    if (static_cast<uint32_t>(tid) < tw) t0 = __ldg(p.table + spec * tw + tid);
  }

  const bool req_ok = req >= 0 && static_cast<int64_t>(req) < p.table_rows;
  if (!req_ok && p.status != nullptr && tid == 0 && active) {
    *reinterpret_cast<volatile int32_t*>(p.status) = SILKERN_STATUS_BAD_REQUEST;
  }
  const int32_t* trow = p.table + static_cast<int64_t>(req_ok ? req : 0) * tw;
  // A row whose request id is outside the table keeps no element.
  const uint32_t twidth = req_ok ? tw : 0u;
  const uint32_t limit = req_ok ? p.local_limit : 0u;

  // Map every element: bit j of `bits` marks a valid one, and v[j] becomes
  // its local position. Unstaged, its block-table entry is requested here as
  // well (an invalid element reads entry 0 of the row, branch-free, and never
  // uses it) into blk[j], so the gather's round trip overlaps the scan.
  uint32_t bits = 0;
  int32_t blk[STAGE ? 1 : G];
#pragma unroll
  for (int j = 0; j < G; ++j) {
    const uint32_t u = static_cast<uint32_t>(v[j]);
    uint32_t lb, local;
    bool ok;
    if constexpr (MODE == kModePow2Il1) {
      // x = t - rank is a multiple of dcp_size exactly when this rank owns
      // t, and then rotating x right by log2(dcp_size) gives t's local
      // position. Otherwise (t not owned, t < rank, or t negative) the
      // rotation leaves a result of at least 2^(31 - log2(dcp_size)), which
      // the host keeps local_limit at or below; so one compare tests
      // ownership, sign and lb < table_width together.
      const uint32_t x = u - p.dcp_rank;
      local = __funnelshift_r(x, x, p.dcp_shift);
      lb = local >> p.bs_shift;
      ok = local < limit;
    } else if constexpr (MODE == kModePow2) {
      local = ((u >> p.group_shift) << p.il_shift) | (u & p.il_mask);
      lb = local >> p.bs_shift;
      ok = static_cast<int32_t>(u) >= 0 && ((u >> p.il_shift) & p.dcp_mask) == p.dcp_rank && lb < twidth;
    } else {
      const uint32_t q1 = fastdiv(u, p.div_il);   // t / interleave
      const uint32_t q2 = fastdiv(q1, p.div_dcp);  // t / (dcp_size * interleave)
      local = q2 * p.interleave + (u - q1 * p.interleave);
      lb = fastdiv(local, p.div_bs);
      ok = static_cast<int32_t>(u) >= 0 && q1 - q2 * p.dcp_size == p.dcp_rank && lb < twidth;
    }
    if constexpr (!STAGE) blk[j] = __ldg(trow + (ok ? lb : 0u));
    v[j] = static_cast<int32_t>(local);
    bits |= ok ? (1u << j) : 0u;
  }

  // Exclusive prefix of this thread's first element inside the CTA.
  const uint32_t c = __popc(bits);
  const int excl = warp_exclusive<count_bits(G)>(c);
  if constexpr (STAGE) {
    // Repair a wrong speculation (the same decision for the whole row group:
    // each thread overwrites exactly the entries it loaded), then publish
    // the staged row; the barrier below makes it visible to the group.
    if (req_ok && req != spec && static_cast<uint32_t>(tid) < tw) t0 = __ldg(trow + tid);
    if (static_cast<uint32_t>(tid) < tw) s_tbl[tid] = t0;
    for (uint32_t e = static_cast<uint32_t>(tid + nthreads); e < tw; e += static_cast<uint32_t>(nthreads)) {
      s_tbl[e] = __ldg(trow + e);
    }
  }
  if (lane == 31) s_wt[warp] = excl + static_cast<int>(c);
  __syncthreads();
  const int x = lane < nwarps ? s_wt[lane] : 0;
  const int pos = __reduce_add_sync(kFull, lane < warp ? x : 0) + excl;
  const int cta_total = __reduce_add_sync(kFull, x);

  // Hierarchical: the CTA-local exclusive position of each tile's first
  // column is that tile's offset (before the row offset). Tiles are
  // multiples of 64 columns and G divides 64, so every tile starts at some
  // thread's first column.
  const bool tiles = p.tile_shift >= 0;
  if (tiles && col < len && (col & ((1 << p.tile_shift) - 1)) == 0) s_tile[col >> p.tile_shift] = pos;

  int row_off = 0;
  int row_total = cta_total;
  if constexpr (CLUSTER) {
    const int cs = p.cluster;
    // The last CTA barrier of a cluster CTA: after the exchange below a
    // thread may leave on its own.
    if (tiles) __syncthreads();  // s_tile is complete
    cluster_wait_acquire();  // phase 0 complete: every CTA runs, every barrier is initialised
    // Push this CTA's total into every CTA's s_cta_total[crank]. The store
    // completes a transaction on the receiver's barrier, so no release fence
    // or second cluster barrier is needed. No CTA exits before all totals
    // have reached it, and no CTA writes another's shared memory after that.
    if (tid < cs) st_async_cluster(&s_cta_total[crank], &s_xbar, static_cast<uint32_t>(tid), cta_total);
    if (!mbar_wait_cluster(&s_xbar, 0, kExchangePolls)) {
      // Only a broken cluster gets here: store nothing for the row.
      if (p.status != nullptr) atomicOr(p.status, SILKERN_STATUS_EXCHANGE_TIMEOUT);
      return;
    }
    row_total = 0;
    for (int r = 0; r < cs; ++r) {
      const int w = s_cta_total[r];
      row_off += r < crank ? w : 0;
      row_total += w;
    }
  }

  // Paged translation: physical = table[lb] * block_size + (local mod
  // block_size), one multiply-add that wraps like the reference's int32
  // lanes; invalid elements become -1 (never stored when compacting).
#pragma unroll
  for (int j = 0; j < G; ++j) {
    const uint32_t local = static_cast<uint32_t>(v[j]);
    uint32_t lb, off;
    if constexpr (MODE == kModeGeneral) {
      lb = fastdiv(local, p.div_bs);
      off = local - lb * p.block_size;
    } else {
      lb = local >> p.bs_shift;
      off = local & p.bs_mask;
    }
    int32_t b;
    if constexpr (STAGE) {
      b = 0;
      if ((bits >> j) & 1u) b = s_tbl[lb];
    } else {
      b = blk[j];
    }
    const int32_t phys = static_cast<int32_t>(static_cast<uint32_t>(b) * p.block_size + off);
    // A compacting call never stores an invalid element: no select needed.
    v[j] = (COMPACT || ((bits >> j) & 1u)) ? phys : -1;
  }

  int32_t* orow = p.out + row * p.width;
  if constexpr (COMPACT && !CLUSTER) {
    // Stage each survivor at its position in the row; then each thread
    // writes its own columns, survivors below the count and -1 from it on.
    int32_t* s_out = gsmem + p.smem_out;
    int k = pos;
#pragma unroll
    for (int j = 0; j < G; ++j) {
      if ((bits >> j) & 1u) s_out[k] = v[j];
      k += static_cast<int>((bits >> j) & 1u);
    }
    __syncthreads();  // s_out and s_tile are complete
    if (col < len) {
      int32_t w[G];
      if (col + G <= cta_total) {
#pragma unroll
        for (int i = 0; i < G / 4; ++i) {
          const int4 q = reinterpret_cast<const int4*>(s_out + col)[i];
          w[4 * i + 0] = q.x;
          w[4 * i + 1] = q.y;
          w[4 * i + 2] = q.z;
          w[4 * i + 3] = q.w;
        }
      } else if (col >= cta_total) {
#pragma unroll
        for (int j = 0; j < G; ++j) w[j] = -1;
      } else {
#pragma unroll
        for (int j = 0; j < G; ++j) w[j] = col + j < cta_total ? s_out[col + j] : -1;
      }
      store_run<G>(orow + col, len - col, w);
    }
  } else if constexpr (COMPACT) {
    // Across a cluster each survivor goes straight to its final position
    // after the CTA's row offset; then the -1 tail within the CTA's own slice.
    int32_t* dst = orow + row_off + pos;
    int k = 0;
#pragma unroll
    for (int j = 0; j < G; ++j) {
      if ((bits >> j) & 1u) dst[k] = v[j];
      k += static_cast<int>((bits >> j) & 1u);
    }
    // The -1 tail: each thread writes its own run of columns where it lies
    // past the row's count (positions below the count get survivors, from
    // whichever CTA holds them). One 256-bit store per run instead of a
    // strided fill of the slice: config 4 took 2.80 against 3.00 us per call.
    if (col < len) {
      const int g0 = c0 + col;
      const int n = len - col < G ? len - col : G;
      if (g0 >= row_total) {
        int32_t w[G];
#pragma unroll
        for (int j = 0; j < G; ++j) w[j] = -1;
        store_run<G>(orow + g0, n, w);
      } else if (g0 + n > row_total) {
#pragma unroll
        for (int j = 0; j < G; ++j) {
          if (j < n && g0 + j >= row_total) orow[g0 + j] = -1;
        }
      }
    }
  } else {
    if (tiles && !CLUSTER) __syncthreads();  // s_tile is complete (a cluster CTA's already was)
    if (col < len) store_run<G>(orow + c0 + col, len - col, v);
  }

  if (tiles) {
    // Offsets and counts (differences of offsets) of this CTA's tiles.
    const int ntiles = (len + (1 << p.tile_shift) - 1) >> p.tile_shift;
    const int64_t tbase = row * p.tiles_per_row + (c0 >> p.tile_shift);
    for (int m = tid; m < ntiles; m += nthreads) {
      const int o = s_tile[m];
      const int next = m + 1 < ntiles ? s_tile[m + 1] : cta_total;
      p.tile_offsets[tbase + m] = row_off + o;
      p.tile_counts[tbase + m] = next - o;
    }
  }

  if (crank == 0 && tid == 0 && active) p.counts[row] = row_total;
}

// Tile workspace of the allocation-free hierarchical entry point: tile counts
// in the first SILKERN_NOALLOC_MAX_TILES entries, tile offsets in the rest.
// Loaded with the module on every device that uses the library; shared by all
// calls. Host code must not pass this symbol to a kernel: its device address
// comes from cudaGetSymbolAddress (noalloc_scratch below).
static __device__ __align__(256) int32_t g_noalloc_tiles[2 * SILKERN_NOALLOC_MAX_TILES];

// The converter's data movement without its work: dst = src, each CTA a
// contiguous chunk of blockDim.x * G elements, each thread a run of G, with
// the converter's launch mode (programmatic dependent launch, a bulk L2
// prefetch of the chunk before the wait) and its run loads and stores. The
// time of a call is the floor a converter call of the same bytes moves
// against.
template <int G>
__global__ void __launch_bounds__(1024) copy_floor_kernel(const int32_t* src, int32_t* dst, int64_t n) {
  pdl_launch_dependents();
  const int64_t c0 = static_cast<int64_t>(blockIdx.x) * blockDim.x * G;
  const int64_t left = n - c0;
  const int len = left < static_cast<int64_t>(blockDim.x) * G ? static_cast<int>(left) : blockDim.x * G;
  if (threadIdx.x == 0) {
    const uintptr_t lo = (reinterpret_cast<uintptr_t>(src + c0) + 15u) & ~uintptr_t{15};
    const uintptr_t hi = reinterpret_cast<uintptr_t>(src + c0 + len) & ~uintptr_t{15};
    if (hi > lo) prefetch_l2_bulk(reinterpret_cast<const void*>(lo), static_cast<uint32_t>(hi - lo));
  }
  pdl_wait();
  const int col = static_cast<int>(threadIdx.x) * G;
  if (col < len) {
    int32_t v[G];
    load_run<G>(src + c0 + col, len - col, v);
    store_run<G>(dst + c0 + col, len - col, v);
  }
}

// Adds the number of differing positions to *mismatches.
__global__ void __launch_bounds__(256) count_mismatches_kernel(const int32_t* a, const int32_t* b,
                                                               int64_t n, int32_t* mismatches) {
  __shared__ int s_part[8];
  pdl_launch_dependents();
  pdl_wait();
  int local = 0;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    local += a[i] != b[i] ? 1 : 0;
  }
  local = __reduce_add_sync(kFull, local);
  if ((threadIdx.x & 31) == 0) s_part[threadIdx.x >> 5] = local;
  __syncthreads();
  if (threadIdx.x == 0) {
    int total = 0;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) total += s_part[w];
    if (total != 0) atomicAdd(mismatches, total);
  }
}

// counters[s] += the number of differing positions inside segment s of
// segment_elems elements; blockIdx.y is the segment.
__global__ void __launch_bounds__(256) count_segment_mismatches_kernel(const int32_t* a, const int32_t* b,
                                                                       int64_t segment_elems,
                                                                       int32_t* counters) {
  __shared__ int s_part[8];
  pdl_launch_dependents();
  pdl_wait();
  const int64_t base = static_cast<int64_t>(blockIdx.y) * segment_elems;
  int local = 0;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < segment_elems; i += stride) {
    local += a[base + i] != b[base + i] ? 1 : 0;
  }
  local = __reduce_add_sync(kFull, local);
  if ((threadIdx.x & 31) == 0) s_part[threadIdx.x >> 5] = local;
  __syncthreads();
  if (threadIdx.x == 0) {
    int total = 0;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) total += s_part[w];
    if (total != 0) atomicAdd(counters + blockIdx.y, total);
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

namespace {

using KernelFn = void (*)(Params);

template <int G, bool CLUSTER, int MODE, bool COMPACT>
KernelFn pick_stage(bool stage) {
  return stage ? localize_kernel<G, CLUSTER, MODE, COMPACT, true> : localize_kernel<G, CLUSTER, MODE, COMPACT, false>;
}

template <int G, bool CLUSTER, int MODE>
KernelFn pick_compact(bool compact, bool stage) {
  return compact ? pick_stage<G, CLUSTER, MODE, true>(stage) : pick_stage<G, CLUSTER, MODE, false>(stage);
}

template <int G, bool CLUSTER>
KernelFn pick_mode(int mode, bool compact, bool stage) {
  switch (mode) {
    case kModePow2Il1: return pick_compact<G, CLUSTER, kModePow2Il1>(compact, stage);
    case kModePow2: return pick_compact<G, CLUSTER, kModePow2>(compact, stage);
    default: return pick_compact<G, CLUSTER, kModeGeneral>(compact, stage);
  }
}

template <int G>
KernelFn pick_for_run(bool cluster, int mode, bool compact, bool stage) {
  return cluster ? pick_mode<G, true>(mode, compact, stage) : pick_mode<G, false>(mode, compact, stage);
}

KernelFn pick_kernel(int run, bool cluster, int mode, bool compact, bool stage) {
  switch (run) {
    case 4: return pick_for_run<4>(cluster, mode, compact, stage);
    case 8: return pick_for_run<8>(cluster, mode, compact, stage);
    case 16: return pick_for_run<16>(cluster, mode, compact, stage);
    case 32: return pick_for_run<32>(cluster, mode, compact, stage);
    default: return nullptr;
  }
}

bool is_pow2(uint32_t v) { return v != 0 && (v & (v - 1)) == 0; }

uint32_t log2_exact(uint32_t v) {
  uint32_t s = 0;
  while ((1u << s) < v) ++s;
  return s;
}

int sm_count() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

bool overlaps(const void* a, int64_t a_elems, const void* b, int64_t b_elems) {
  if (a == nullptr || b == nullptr) return false;
  const uintptr_t a0 = reinterpret_cast<uintptr_t>(a), b0 = reinterpret_cast<uintptr_t>(b);
  const uintptr_t a1 = a0 + static_cast<uintptr_t>(a_elems) * 4u;
  const uintptr_t b1 = b0 + static_cast<uintptr_t>(b_elems) * 4u;
  return a0 < b1 && b0 < a1;
}

struct Request {
  const int32_t* req_ids;
  const int32_t* table;
  int64_t table_rows, table_width;
  const int32_t* tokens;
  int32_t* out;
  int32_t* counts;
  int32_t* tile_counts;
  int32_t* tile_offsets;
  int64_t batch, width;
  int32_t block_size, dcp_size, dcp_rank, interleave, compact_flag;
  int32_t tile_size;  // 0 = row-wise semantics
  int32_t* status;
  cudaStream_t stream;
};

// Argument checks shared by every entry point, before anything is launched.
// need_tile_buffers = false skips only the check that the tile workspace
// pointers are set (the allocation-free entry point supplies its own).
int validate(const Request& r, bool need_tile_buffers = true) {
  if (!r.req_ids || !r.table || !r.tokens || !r.out || !r.counts) return SILKERN_E_NULL;
  if (r.batch < 1 || r.width < 1 || r.width > SILKERN_MAX_ROW_WIDTH || r.table_rows < 1 ||
      r.table_width < 1 || r.table_width > INT32_MAX || r.batch > (int64_t{1} << 27)) {
    return SILKERN_E_SHAPE;
  }
  if (r.dcp_size < 1 || r.dcp_rank < 0 || r.dcp_rank >= r.dcp_size || r.interleave < 1) return SILKERN_E_DCP;
  if (r.block_size < 1 || r.block_size % r.interleave != 0) return SILKERN_E_BLOCK_SIZE;
  if (r.tile_size != 0) {
    if (r.tile_size < SILKERN_MIN_TILE_SIZE || r.tile_size > SILKERN_MAX_TILE_SIZE ||
        !is_pow2(static_cast<uint32_t>(r.tile_size))) {
      return SILKERN_E_TILE;
    }
    if (need_tile_buffers && (!r.tile_counts || !r.tile_offsets)) return SILKERN_E_NULL;
  }
  const int64_t bw = r.batch * r.width;
  const int64_t tiles = r.tile_size ? r.batch * ((r.width + r.tile_size - 1) / r.tile_size) : 0;
  struct Range {
    const void* p;
    int64_t n;
  };
  const Range inputs[3] = {{r.req_ids, r.batch}, {r.table, r.table_rows * r.table_width}, {r.tokens, bw}};
  const Range outputs[4] = {{r.out, bw}, {r.counts, r.batch}, {r.tile_counts, tiles}, {r.tile_offsets, tiles}};
  for (const Range& o : outputs) {
    for (const Range& in : inputs) {
      if (overlaps(o.p, o.n, in.p, in.n)) return SILKERN_E_ALIAS;
    }
  }
  for (int a = 0; a < 4; ++a) {
    for (int b = a + 1; b < 4; ++b) {
      if (overlaps(outputs[a].p, outputs[a].n, outputs[b].p, outputs[b].n)) return SILKERN_E_ALIAS;
    }
  }
  return SILKERN_OK;
}

struct Geometry {
  int cluster;
  int slice;
  int threads;  // per row group (per CTA with a cluster)
  int run;      // columns per thread
  bool stage;
  bool prefetch;
  int rows_per_cta;   // row groups per CTA (1 with a cluster)
  int64_t row_ctas;   // CTAs over the batch (times `cluster` for the grid)
  // dynamic shared memory per row group, in ints: [table stage][staged
  // output][warp totals][tile offsets], every part 16-byte aligned
  int smem_out, smem_wt, smem_tile, smem_group;
};

uint32_t next_pow2(uint32_t v) {
  uint32_t p = 1;
  while (p < v) p <<= 1;
  return p;
}

// Shared memory per SM and reserved per CTA, for occupancy shaping.
void smem_limits(int* per_sm, int* reserved) {
  static int cache_sm[64] = {0}, cache_res[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    (void)cudaGetLastError();
    *per_sm = 233472;
    *reserved = 1024;
    return;
  }
  if (cache_sm[dev] == 0) {
    int a = 0, b = 0;
    if (cudaDeviceGetAttribute(&a, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev) != cudaSuccess || a <= 0) {
      a = 233472;
    }
    if (cudaDeviceGetAttribute(&b, cudaDevAttrReservedSharedMemoryPerBlock, dev) != cudaSuccess || b < 0) b = 1024;
    (void)cudaGetLastError();
    cache_res[dev] = b;
    cache_sm[dev] = a;
  }
  *per_sm = cache_sm[dev];
  *reserved = cache_res[dev];
}

// Columns per thread and threads for `slice` columns: the shortest run from
// `first` columns up (8, or 16 for batches of several waves) that covers the
// slice with at most kMaxThreads threads, unless run_req pins it (4, 8, 16
// or 32). Threads are a whole number of warps; a row group (no cluster) is a
// power of two of them.
bool fit_slice(int slice, int run_req, int first, bool cluster, int* run, int* threads) {
  int g = run_req;
  if (g == 0) {
    g = first;
    while (g < 32 && (slice + g - 1) / g > kMaxThreads) g *= 2;
  }
  int t = (slice + g - 1) / g;
  t = (t + 31) / 32 * 32;
  if (!cluster) t = static_cast<int>(next_pow2(static_cast<uint32_t>(t)));
  if (t > kMaxThreads) return false;
  *run = g;
  *threads = t;
  return true;
}

void layout_smem(const Request& r, bool compact, Geometry* g) {
  const int ntiles_cta = r.tile_size ? (g->slice + r.tile_size - 1) / r.tile_size : 0;
  const int stage_ints = g->stage ? static_cast<int>((r.table_width + 3) / 4 * 4) : 0;
  g->smem_out = stage_ints;
  g->smem_wt = g->smem_out + ((compact && g->cluster == 1) ? (g->slice + 3) / 4 * 4 : 0);
  g->smem_tile = g->smem_wt + 32;
  g->smem_group = (g->smem_tile + ntiles_cta + 3) / 4 * 4;
}

int choose_geometry(const Request& r, bool compact, int cluster_req, int stage_req, int prefetch_req,
                    int run_req, Geometry* g) {
  const int width = static_cast<int>(r.width);
  int cs;
  int slice;
  if (r.tile_size != 0) {
    // Hierarchical: a CTA covers a whole number of tiles; the cluster is the
    // largest power of two (up to 8) that keeps batch x cluster within about
    // one CTA per SM, and (unless the row is shorter) a CTA covers at least
    // 1024 columns.
    const int tiles = (width + r.tile_size - 1) / r.tile_size;
    int per_cta;
    if (cluster_req > 0) {
      per_cta = (tiles + cluster_req - 1) / cluster_req;
    } else {
      const int sms = sm_count();
      int cs_target = 1;
      while (cs_target < kMaxCluster && r.batch * cs_target * 2 <= sms) cs_target *= 2;
      per_cta = (tiles + cs_target - 1) / cs_target;
      const int min_tiles = (1024 + r.tile_size - 1) / r.tile_size;
      if (per_cta < min_tiles) per_cta = min_tiles;
      if (per_cta > tiles) per_cta = tiles;
    }
    slice = per_cta * r.tile_size;
    cs = (tiles + per_cta - 1) / per_cta;
  } else {
    if (cluster_req > 0) {
      cs = cluster_req;
    } else {
      // Row-wise: rows up to 8192 columns stay on one CTA (row groups keep
      // the SMs balanced and a cluster exchange costs more than it saves);
      // longer rows are split over a cluster when there are few of them.
      const int sms = sm_count();
      cs = 1;
      while (width > 8192 && cs < kMaxCluster && r.batch * cs * 2 <= sms && width / (2 * cs) >= 2048) {
        cs *= 2;
      }
    }
    // Slices start on 64-column boundaries, so every run keeps the row's
    // alignment.
    slice = (width + cs - 1) / cs;
    slice = (slice + 63) / 64 * 64;
    cs = (width + slice - 1) / slice;
  }
  if (cluster_req > 0 && cs != cluster_req) return SILKERN_E_GEOMETRY;
  if (cs < 1 || cs > kMaxCluster) return SILKERN_E_GEOMETRY;
  // Short runs (more warps, shorter per-thread chains) measured faster while
  // one call's rows fit the GPU in a few waves (600 rows of 2048: 4.64
  // against 5.33 us per call with 16-column runs); from about six rows per
  // SM the work is issue-bound and 16-column runs, which amortise each
  // thread's fixed instructions over twice the columns, measured faster
  // (1024 rows: 5.50 against 6.04; 16384 rows: 66.7 against 69.9).
  const int first_run = (cs == 1 && r.batch >= int64_t{6} * sm_count()) ? 16 : 8;
  if (!fit_slice(slice, run_req, first_run, cs > 1, &g->run, &g->threads)) return SILKERN_E_GEOMETRY;
  g->cluster = cs;
  g->slice = slice;
  g->rows_per_cta = 1;
  g->row_ctas = r.batch;
  if (cs == 1) {
    // Row groups: one row per CTA. Up to four rows per SM on average the
    // shared-memory reservation below keeps as many CTAs per SM as the batch
    // needs, no more: 256 rows of 2048 measured 2.16 us per call against
    // 2.24-2.41 with two-row CTAs on 148 SMs, 400 rows 2.74 against 3.12.
    // Larger batches run in waves of small CTAs that retire independently:
    // 16384 rows of 2048 measured 54.9 us per call (0.75 of the copy peak)
    // against 66.8 with four-row CTAs. Only narrow rows share a CTA there, so
    // that a CTA keeps at least 128 threads.
    const int64_t max_rows = r.batch <= int64_t{4} * sm_count() || g->threads >= 128
                                 ? 1
                                 : (128 / g->threads < kMaxThreads / g->threads ? 128 / g->threads
                                                                                 : kMaxThreads / g->threads);
    int64_t ctas = r.batch < sm_count() ? r.batch : sm_count();
    int64_t rows = (r.batch + ctas - 1) / ctas;
    if (rows > max_rows) {
      rows = max_rows;
      ctas = (r.batch + rows - 1) / rows;
    }
    g->rows_per_cta = static_cast<int>(rows);
    g->row_ctas = ctas;
  }
  // Table stage only on request (rows up to kTableStageMax entries): the L2
  // gather measured faster by default, on one CTA (config 3: 2.24 against
  // 2.39 us per call; its latency hides behind the other warps' issue while
  // the stage adds instructions) and across a cluster at one CTA per SM
  // (config 4: 3.38 against 3.45).
  if (stage_req == 1 && r.table_width > kTableStageMax) return SILKERN_E_GEOMETRY;
  g->stage = stage_req == 1;
  layout_smem(r, compact, g);
  if (static_cast<int64_t>(g->smem_group) * 4 * g->rows_per_cta > kSmemMax) return SILKERN_E_GEOMETRY;
  const int64_t table_bytes = r.table_rows * r.table_width * 4;
  const bool aligned = (reinterpret_cast<uintptr_t>(r.table) & 15u) == 0;
  const bool possible = aligned && table_bytes >= 16 && table_bytes <= (int64_t{1} << 32);
  g->prefetch = prefetch_req >= 0 ? (prefetch_req == 1 && possible)
                                   : (possible && table_bytes <= 2 * r.batch * r.width * 4);
  if (g->row_ctas * cs > INT32_MAX) return SILKERN_E_SHAPE;
  return SILKERN_OK;
}

// Dynamic shared memory above 48 KB must be enabled per kernel and device.
// The largest size granted so far is remembered per kernel and device, so a
// steady stream of calls makes the driver call once.
int allow_large_smem(KernelFn fn, size_t bytes) {
  struct Grant {
    KernelFn fn;
    int device;
    size_t bytes;
  };
  static std::mutex mutex;
  static Grant grants[256];
  static int n_grants = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    const cudaError_t err = cudaGetLastError();
    return -static_cast<int>(err == cudaSuccess ? cudaErrorInvalidDevice : err);
  }
  std::lock_guard<std::mutex> lock(mutex);
  Grant* slot = nullptr;
  for (int i = 0; i < n_grants; ++i) {
    if (grants[i].fn == fn && grants[i].device == dev) slot = &grants[i];
  }
  if (slot != nullptr && slot->bytes >= bytes) return SILKERN_OK;
  const cudaError_t err =
      cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
  if (err != cudaSuccess) {
    (void)cudaGetLastError();
    return -static_cast<int>(err);
  }
  if (slot == nullptr && n_grants < 256) slot = &grants[n_grants++];
  if (slot != nullptr) *slot = Grant{fn, dev, bytes};
  return SILKERN_OK;
}

int launch(const Request& r, int cluster_req, int stage_req, int prefetch_req, int run_req) {
  int rc = validate(r);
  if (rc != SILKERN_OK) return rc;
  const bool compact = r.compact_flag != 0 && r.dcp_size > 1;
  Geometry g;
  rc = choose_geometry(r, compact, cluster_req, stage_req, prefetch_req, run_req, &g);
  if (rc != SILKERN_OK) return rc;

  Params p{};
  p.req_ids = r.req_ids;
  p.table = r.table;
  p.tokens = r.tokens;
  p.out = r.out;
  p.counts = r.counts;
  p.tile_counts = r.tile_counts;
  p.tile_offsets = r.tile_offsets;
  p.status = r.status;
  p.table_rows = r.table_rows;
  p.table_width = static_cast<uint32_t>(r.table_width);
  p.width = static_cast<int32_t>(r.width);
  p.slice = g.slice;
  p.cluster = g.cluster;
  p.tile_shift = r.tile_size ? static_cast<int32_t>(log2_exact(static_cast<uint32_t>(r.tile_size))) : -1;
  p.tiles_per_row = r.tile_size ? static_cast<int32_t>((r.width + r.tile_size - 1) / r.tile_size) : 0;
  const int64_t grid = g.row_ctas * g.cluster;
  p.row_threads = g.threads;
  p.row_threads_shift = static_cast<int32_t>(log2_exact(static_cast<uint32_t>(g.threads)));
  p.rows_base = static_cast<int32_t>(r.batch / g.row_ctas);
  p.rows_extra = static_cast<int32_t>(r.batch % g.row_ctas);
  if (g.prefetch) {
    const uint64_t bytes = static_cast<uint64_t>(r.table_rows * r.table_width * 4) & ~uint64_t{15};
    uint64_t chunk = (bytes + static_cast<uint64_t>(grid) - 1) / static_cast<uint64_t>(grid);
    chunk = (chunk + 15u) & ~uint64_t{15};
    if (chunk < 256) chunk = 256;
    p.table_bytes = bytes;
    p.table_chunk = static_cast<uint32_t>(chunk);
  }
  p.dcp_rank = static_cast<uint32_t>(r.dcp_rank);
  p.dcp_size = static_cast<uint32_t>(r.dcp_size);
  p.interleave = static_cast<uint32_t>(r.interleave);
  p.block_size = static_cast<uint32_t>(r.block_size);
  p.div_il = make_fastdiv(p.interleave);
  p.div_dcp = make_fastdiv(p.dcp_size);
  p.div_bs = make_fastdiv(p.block_size);
  const bool pow2 = is_pow2(p.interleave) && is_pow2(p.dcp_size) && is_pow2(p.block_size) &&
                    log2_exact(p.interleave) + log2_exact(p.dcp_size) <= 31;
  int mode = kModeGeneral;
  if (pow2) {
    p.il_shift = log2_exact(p.interleave);
    p.dcp_shift = log2_exact(p.dcp_size);
    p.group_shift = p.il_shift + p.dcp_shift;
    p.bs_shift = log2_exact(p.block_size);
    p.il_mask = p.interleave - 1;
    p.dcp_mask = p.dcp_size - 1;
    p.bs_mask = p.block_size - 1;
    mode = kModePow2;
    if (p.interleave == 1) {
      // A valid element's local position is below table_width * block_size
      // (lb < table_width) and, since t < 2^31, below 2^(31 - log2(dcp_size));
      // every element this rank does not own, or that is negative, rotates
      // to at least 2^(31 - log2(dcp_size)).
      const uint64_t by_table = static_cast<uint64_t>(r.table_width) << p.bs_shift;
      const uint64_t by_sign = uint64_t{1} << (31 - p.dcp_shift);
      p.local_limit = static_cast<uint32_t>(by_table < by_sign ? by_table : by_sign);
      mode = kModePow2Il1;
    }
  }

  KernelFn fn = pick_kernel(g.run, g.cluster > 1, mode, compact, g.stage);
  if (fn == nullptr) return SILKERN_E_GEOMETRY;
  p.smem_out = g.smem_out;
  p.smem_wt = g.smem_wt;
  p.smem_tile = g.smem_tile;
  p.smem_group = g.smem_group;
  size_t smem = sizeof(int32_t) * static_cast<size_t>(p.smem_group) * static_cast<size_t>(g.rows_per_cta);
  if (g.cluster > 1) {
    // One cluster CTA per SM. With two, the next call's clusters (launched
    // early by programmatic dependent launch) share the SMs of the running
    // call; one per SM measured 4.05 -> 3.45 us per call at 32 rows x 16384
    // columns over four-CTA clusters.
    int per_sm = 0, reserved = 0;
    smem_limits(&per_sm, &reserved);
    const size_t one_per_sm = static_cast<size_t>(per_sm / 2 - reserved + 16);
    if (smem < one_per_sm) smem = one_per_sm;
  }
  if (g.cluster == 1 && grid <= int64_t{4} * sm_count()) {
    // Residency under programmatic dependent launch: the next call's CTAs
    // become resident wherever this call leaves room. When the batch leaves
    // SMs free, one CTA per SM measured faster: the next call lands on SMs
    // of its own (64 x 2048: 2.19 -> 1.80 us per call; 128 x 2048: 2.29 ->
    // 1.87). When a call fills the SMs, as many per SM as the call needs
    // (two for up to two CTAs per SM, and so on), so the next call's CTAs
    // spread over the SMs instead of piling onto the ones this call left
    // room on.
    int per_sm = 0, reserved = 0;
    smem_limits(&per_sm, &reserved);
    const int per_sm_ctas = grid < sm_count() ? 1 : static_cast<int>((grid + sm_count() - 1) / sm_count());
    const size_t reserve = static_cast<size_t>(per_sm / (per_sm_ctas + 1) - reserved + 16);
    if (smem < reserve) smem = reserve;
  }
  if (smem > 48 * 1024) {
    rc = allow_large_smem(fn, smem);
    if (rc != SILKERN_OK) return rc;
  }

  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
  cfg.blockDim = dim3(static_cast<unsigned>(g.threads * g.rows_per_cta), 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = r.stream;
  cudaLaunchAttribute attrs[2];
  int nattr = 0;
  attrs[nattr].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[nattr].val.programmaticStreamSerializationAllowed = 1;
  ++nattr;
  if (g.cluster > 1) {
    attrs[nattr].id = cudaLaunchAttributeClusterDimension;
    attrs[nattr].val.clusterDim.x = static_cast<unsigned>(g.cluster);
    attrs[nattr].val.clusterDim.y = 1;
    attrs[nattr].val.clusterDim.z = 1;
    ++nattr;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = nattr;
  const cudaError_t err = cudaLaunchKernelEx(&cfg, fn, p);
  if (err != cudaSuccess) {
    (void)cudaGetLastError();
    return -static_cast<int>(err);
  }
  return SILKERN_OK;
}

}  // namespace
}  // namespace silkern

using silkern::Request;

extern "C" int silkern_localize_rowwise_v1(const int32_t* req_ids, const int32_t* block_table,
                                           int64_t table_rows, int64_t table_width,
                                           const int32_t* tokens, int32_t* out, int32_t* counts,
                                           int64_t batch, int64_t width, int32_t block_size,
                                           int32_t dcp_size, int32_t dcp_rank,
                                           int32_t dcp_interleave, int32_t compact_valid_to_front,
                                           int32_t* status, void* stream) {
  const Request r{req_ids, block_table, table_rows, table_width, tokens, out, counts, nullptr, nullptr,
                  batch, width, block_size, dcp_size, dcp_rank, dcp_interleave,
                  compact_valid_to_front, 0, status, static_cast<cudaStream_t>(stream)};
  return silkern::launch(r, 0, -1, -1, 0);
}

extern "C" int silkern_localize_hierarchical_v1(
    const int32_t* req_ids, const int32_t* block_table, int64_t table_rows, int64_t table_width,
    const int32_t* tokens, int32_t* out, int32_t* counts, int32_t* mapped_ws,
    int32_t* local_positions_ws, int32_t* tile_counts_ws, int32_t* tile_offsets_ws, int64_t batch,
    int64_t width, int32_t block_size, int32_t dcp_size, int32_t dcp_rank, int32_t dcp_interleave,
    int32_t compact_valid_to_front, int32_t tile_size, int32_t* status, void* stream) {
  (void)mapped_ws;
  (void)local_positions_ws;
  if (tile_size == 0) return SILKERN_E_TILE;
  const Request r{req_ids, block_table, table_rows, table_width, tokens, out, counts,
                  tile_counts_ws, tile_offsets_ws, batch, width, block_size, dcp_size, dcp_rank,
                  dcp_interleave, compact_valid_to_front, tile_size, status,
                  static_cast<cudaStream_t>(stream)};
  return silkern::launch(r, 0, -1, -1, 0);
}

extern "C" int silkern_localize_explicit_v1(
    const int32_t* req_ids, const int32_t* block_table, int64_t table_rows, int64_t table_width,
    const int32_t* tokens, int32_t* out, int32_t* counts, int32_t* tile_counts_ws,
    int32_t* tile_offsets_ws, int64_t batch, int64_t width, int32_t block_size, int32_t dcp_size,
    int32_t dcp_rank, int32_t dcp_interleave, int32_t compact_valid_to_front, int32_t tile_size,
    int32_t cluster_size, int32_t stage_table, int32_t prefetch_table, int32_t chunks_per_thread,
    int32_t* status, void* stream) {
  if (cluster_size < 1 || cluster_size > silkern::kMaxCluster) return SILKERN_E_GEOMETRY;
  if (stage_table < -1 || stage_table > 1 || prefetch_table < -1 || prefetch_table > 1) {
    return SILKERN_E_GEOMETRY;
  }
  if (chunks_per_thread != 0 && chunks_per_thread != 1 && chunks_per_thread != 2 &&
      chunks_per_thread != 4 && chunks_per_thread != 8) {
    return SILKERN_E_GEOMETRY;
  }
  const Request r{req_ids, block_table, table_rows, table_width, tokens, out, counts,
                  tile_counts_ws, tile_offsets_ws, batch, width, block_size, dcp_size, dcp_rank,
                  dcp_interleave, compact_valid_to_front, tile_size, status,
                  static_cast<cudaStream_t>(stream)};
  return silkern::launch(r, cluster_size, stage_table, prefetch_table, 4 * chunks_per_thread);
}

namespace silkern {
namespace {

// The driver's cuCtxGetCurrent and cuCtxGetId, reached through the runtime
// so the library needs no link-time dependency on libcuda. A context's id is
// unique for the life of the process, even when a reset frees the context
// and a new one takes its place (and perhaps its handle).
using CtxGetCurrentFn = int (*)(void**);
using CtxGetIdFn = int (*)(void*, unsigned long long*);

bool current_context_id(unsigned long long* id) {
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult found = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &fn, 12000, cudaEnableDefault, &found) ==
            cudaSuccess &&
        found == cudaDriverEntryPointSuccess) {
      get_current = reinterpret_cast<CtxGetCurrentFn>(fn);
    }
    fn = nullptr;
    found = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetId", &fn, 12000, cudaEnableDefault, &found) ==
            cudaSuccess &&
        found == cudaDriverEntryPointSuccess) {
      get_id = reinterpret_cast<CtxGetIdFn>(fn);
    }
    (void)cudaGetLastError();
  });
  if (get_current == nullptr || get_id == nullptr) return false;
  void* ctx = nullptr;
  if (get_current(&ctx) != 0 || ctx == nullptr) return false;
  return get_id(ctx, id) == 0;
}

// Device address of g_noalloc_tiles in the current device's context. It is
// looked up with cudaGetSymbolAddress the first time a device (with that
// device current) calls, and again whenever the device's context has changed
// since (a cudaDeviceReset, for one), so a cached address never outlives its
// context. Without the driver's context ids it is looked up on every call.
int noalloc_scratch(int32_t** out) {
  struct Slot {
    int32_t* ptr;
    unsigned long long ctx_id;
  };
  static std::mutex mu;
  static Slot cache[64] = {};
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) {
    (void)cudaGetLastError();
    return -static_cast<int>(err);
  }
  if (dev < 0 || dev >= 64) return SILKERN_E_SCRATCH;
  std::lock_guard<std::mutex> lock(mu);
  unsigned long long id = 0;
  if (cache[dev].ptr != nullptr && current_context_id(&id) && id == cache[dev].ctx_id) {
    *out = cache[dev].ptr;
    return SILKERN_OK;
  }
  void* ptr = nullptr;
  err = cudaGetSymbolAddress(&ptr, g_noalloc_tiles);  // makes the device's context current if needed
  if (err != cudaSuccess || ptr == nullptr) {
    (void)cudaGetLastError();
    return err != cudaSuccess ? -static_cast<int>(err) : SILKERN_E_SCRATCH;
  }
  cache[dev] = current_context_id(&id) ? Slot{static_cast<int32_t*>(ptr), id} : Slot{nullptr, 0};
  *out = static_cast<int32_t*>(ptr);
  return SILKERN_OK;
}

}  // namespace
}  // namespace silkern

extern "C" int silkern_localize_hierarchical_noalloc_v1(
    const int32_t* req_ids, const int32_t* block_table, int64_t table_rows, int64_t table_width,
    const int32_t* tokens, int32_t* out, int32_t* counts, int64_t batch, int64_t width,
    int32_t block_size, int32_t dcp_size, int32_t dcp_rank, int32_t dcp_interleave,
    int32_t compact_valid_to_front, int32_t tile_size, int32_t* status, void* stream) {
  if (tile_size == 0) return SILKERN_E_TILE;
  Request r{req_ids, block_table, table_rows, table_width, tokens, out, counts, nullptr, nullptr,
            batch, width, block_size, dcp_size, dcp_rank, dcp_interleave, compact_valid_to_front,
            tile_size, status, static_cast<cudaStream_t>(stream)};
  // The same checks, in the same order, as the workspace entry point; the
  // static array's limit comes after them.
  int rc = silkern::validate(r, /*need_tile_buffers=*/false);
  if (rc != SILKERN_OK) return rc;
  if (batch * ((width + tile_size - 1) / tile_size) > SILKERN_NOALLOC_MAX_TILES) return SILKERN_E_SCRATCH;
  int32_t* scratch = nullptr;
  rc = silkern::noalloc_scratch(&scratch);
  if (rc != SILKERN_OK) return rc;
  r.tile_counts = scratch;
  r.tile_offsets = scratch + SILKERN_NOALLOC_MAX_TILES;
  return silkern::launch(r, 0, -1, -1, 0);
}

extern "C" int silkern_workspace_shapes_v1(int64_t batch, int64_t width, int32_t tile_size,
                                           int64_t out_shapes[8]) {
  if (out_shapes == nullptr) return SILKERN_E_NULL;
  if (batch < 1 || width < 1 || width > SILKERN_MAX_ROW_WIDTH) return SILKERN_E_SHAPE;
  if (tile_size < SILKERN_MIN_TILE_SIZE || tile_size > SILKERN_MAX_TILE_SIZE ||
      !silkern::is_pow2(static_cast<uint32_t>(tile_size))) {
    return SILKERN_E_TILE;
  }
  const int64_t tiles = (width + tile_size - 1) / tile_size;
  const int64_t shapes[8] = {batch, width, batch, width, batch, tiles, batch, tiles};
  for (int i = 0; i < 8; ++i) out_shapes[i] = shapes[i];
  return SILKERN_OK;
}

extern "C" int silkern_count_mismatches_v1(const int32_t* a, const int32_t* b, int64_t n,
                                           int32_t* mismatches, void* stream) {
  if (!a || !b || !mismatches) return SILKERN_E_NULL;
  if (n < 0) return SILKERN_E_SHAPE;
  if (n == 0) return SILKERN_OK;
  int64_t blocks = (n + 255) / 256;
  const int64_t cap = static_cast<int64_t>(silkern::sm_count()) * 8;
  if (blocks > cap) blocks = cap;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(blocks), 1, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  const cudaError_t err = cudaLaunchKernelEx(&cfg, silkern::count_mismatches_kernel, a, b, n, mismatches);
  if (err != cudaSuccess) {
    (void)cudaGetLastError();
    return -static_cast<int>(err);
  }
  return SILKERN_OK;
}

extern "C" int silkern_copy_floor_v1(const int32_t* src, int32_t* dst, int64_t n, int32_t run,
                                     int32_t threads, int32_t ctas_per_sm, void* stream) {
  if (!src || !dst) return SILKERN_E_NULL;
  if (n < 0) return SILKERN_E_SHAPE;
  if ((run != 8 && run != 16) || threads < 32 || threads > 1024 || threads % 32 != 0 || ctas_per_sm < 0 ||
      ctas_per_sm > 8) {
    return SILKERN_E_GEOMETRY;
  }
  if (silkern::overlaps(src, n, dst, n)) return SILKERN_E_ALIAS;
  if (n == 0) return SILKERN_OK;
  const int64_t per_cta = static_cast<int64_t>(threads) * run;
  const int64_t blocks = (n + per_cta - 1) / per_cta;
  if (blocks > INT32_MAX) return SILKERN_E_SHAPE;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(blocks), 1, 1);
  cfg.blockDim = dim3(static_cast<unsigned>(threads), 1, 1);
  cfg.stream = static_cast<cudaStream_t>(stream);
  void (*fn)(const int32_t*, int32_t*, int64_t) =
      run == 8 ? silkern::copy_floor_kernel<8> : silkern::copy_floor_kernel<16>;
  if (ctas_per_sm > 0) {
    // The converter's residency control: a shared-memory reservation that
    // lets at most ctas_per_sm of these CTAs share an SM, so the next call's
    // CTAs (launched early under programmatic dependent launch) spread out.
    int per_sm = 0, reserved = 0;
    silkern::smem_limits(&per_sm, &reserved);
    cfg.dynamicSmemBytes = static_cast<size_t>(per_sm / (ctas_per_sm + 1) - reserved + 16);
    if (cfg.dynamicSmemBytes > 48 * 1024) {
      const cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 static_cast<int>(cfg.dynamicSmemBytes));
      if (e != cudaSuccess) {
        (void)cudaGetLastError();
        return -static_cast<int>(e);
      }
    }
  }
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  const cudaError_t err = cudaLaunchKernelEx(&cfg, fn, src, dst, n);
  if (err != cudaSuccess) {
    (void)cudaGetLastError();
    return -static_cast<int>(err);
  }
  return SILKERN_OK;
}

extern "C" int silkern_count_segment_mismatches_v1(const int32_t* a, const int32_t* b, int64_t segments,
                                                   int64_t segment_elems, int32_t* counters,
                                                   void* stream) {
  if (!a || !b || !counters) return SILKERN_E_NULL;
  if (segments < 0 || segments > 65535 || segment_elems < 0) return SILKERN_E_SHAPE;
  if (segments == 0 || segment_elems == 0) return SILKERN_OK;
  int64_t blocks = (segment_elems + 255) / 256;
  const int64_t cap = (static_cast<int64_t>(silkern::sm_count()) * 8 + segments - 1) / segments;
  if (blocks > cap) blocks = cap;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(blocks), static_cast<unsigned>(segments), 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  const cudaError_t err = cudaLaunchKernelEx(&cfg, silkern::count_segment_mismatches_kernel, a, b,
                                             segment_elems, counters);
  if (err != cudaSuccess) {
    (void)cudaGetLastError();
    return -static_cast<int>(err);
  }
  return SILKERN_OK;
}

extern "C" const char* silkern_status_string_v1(int code) {
  switch (code) {
    case SILKERN_OK: return "ok";
    case SILKERN_E_NULL: return "a required buffer pointer is NULL";
    case SILKERN_E_SHAPE: return "batch, width or block-table dimensions are out of range";
    case SILKERN_E_DCP: return "invalid dcp configuration";
    case SILKERN_E_BLOCK_SIZE: return "block_size must be a positive integer divisible by dcp_interleave";
    case SILKERN_E_TILE: return "unsupported tile_size";
    case SILKERN_E_ALIAS: return "an output buffer overlaps an input or another output";
    case SILKERN_E_GEOMETRY: return "explicit launch geometry rejected";
    case SILKERN_E_SCRATCH:
      return "batch x tiles exceeds the allocation-free entry point's static workspace";
    default: break;
  }
  if (code < 0) return cudaGetErrorString(static_cast<cudaError_t>(-code));
  return "unknown status";
}

extern "C" int silkern_abi_version_v1(void) { return SILKERN_ABI_VERSION; }

extern "C" int64_t silkern_fastdiv_selftest_v1(uint32_t divisor, uint32_t n_begin, uint32_t n_count) {
  if (divisor == 0 || divisor > (1u << 31)) return -1;
  const silkern::FastDiv d = silkern::make_fastdiv(divisor);
  int64_t bad = 0;
  for (uint64_t k = 0; k < n_count; ++k) {
    const uint64_t n64 = static_cast<uint64_t>(n_begin) + k;
    if (n64 >= (uint64_t{1} << 31)) break;
    const uint32_t n = static_cast<uint32_t>(n64);
    if (silkern::fastdiv(n, d) != n / divisor) ++bad;
  }
  return bad;
}
