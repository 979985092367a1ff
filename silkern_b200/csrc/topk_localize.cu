// Fused indexer top-k + localization on B200 (sm_100a).
//
// A sparse decode step scores every context position of a request (the
// indexer's logits), keeps the top_k of them, and the converter then turns
// those global positions into this DCP rank's physical KV slots. Run as two
// kernels, the (batch, top_k) selection goes to HBM and comes back and the
// second kernel pays a dependent-launch handoff. Here both are one kernel,
// one CTA per row, every row of the batch resident at once (1024-thread CTAs,
// one per SM, when the batch fits the SMs; 512-thread CTAs, two per SM,
// otherwise):
//
//   0. as soon as the row's length is known, bulk L2 prefetches
//      (cp.async.bulk.prefetch.L2) start the whole row streaming from HBM;
//   1. estimate: a histogram of the top 11 bits of the order key over every
//      16th float4 of the row picks a floor bin that should leave ~1.5 x
//      top_k scores at or above it (rows too short for the sample to reach a
//      floor list every column);
//   2. stream: the row is read once (128-bit loads, several 128-column blocks
//      in flight per warp) and only a bit mask of the candidates (scores at or
//      above the floor) is kept, per 128-column block;
//   3. gather: every thread owns a run of whole blocks; one CTA scan over
//      the threads' candidate counts gives each its offset in the list, and it
//      writes its candidates' positions from the masks; then all threads load
//      the keys (L2 hits, eight in flight per lane), feeding the first radix
//      histogram;
//   4. select: the three-pass radix select (11, 11 and 10 key bits) over the
//      list finds the exact threshold key and how many keys equal to it are
//      taken (the lowest positions); it ends at the first pass whose
//      threshold bin is taken whole;
//   5. emit: the selected positions, in ascending order, are the selection
//      row; the converter's contract (silkern/contract.py:67-158: ownership,
//      deinterleave, paged translation, stable compaction, counts) is applied
//      to it. Warps take contiguous runs of the list, lanes consecutive
//      entries; ranks come from ballots and one exchange of the warps' totals,
//      and the request's block-table row is staged in shared memory.
//
// When the estimate misses (fewer than top_k scores above the floor) or the
// candidates overflow the list (heavy ties), the CTA finds the threshold by
// radix passes over the whole row (served from L2) instead and lists exactly
// the selected positions; the output is the same.
//
// Order key: the float's bit pattern with every bit flipped when the sign is
// set and only the sign bit flipped otherwise, compared as unsigned. This is
// the float order extended to a total order on bit patterns (-0 < +0, NaNs
// outside the infinities), so the selection is deterministic for every input.
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <mutex>

#include "fastdiv.cuh"
#include "ptx.cuh"
#include "silkern_b200.h"

namespace silkern {
namespace {

constexpr int kBlockCols = 128;  // one float4 per lane of a warp
constexpr int kBins = 2048;      // 11-bit radix digit
constexpr int kSampleEvery = 16;      // one float4 of every 16 feeds the estimate
constexpr int64_t kPrefetchBytes = 16384;  // per bulk L2 prefetch
constexpr int kStreamUnroll = 8;      // 128-column blocks in flight per warp
constexpr int kTableStageMax = 4096;  // block-table entries staged in shared memory
constexpr int64_t kTopkSmemBudget = 200 * 1024;  // dynamic shared memory per CTA
// The write pass packs a CTA's selected and valid counts into one int, 16
// bits each; a candidate list of 8-byte entries within the budget stays
// below 2^16 entries.
static_assert(kTopkSmemBudget / 8 < 65536, "candidate counts must fit 16 bits");
constexpr int kMaxBlocks = SILKERN_TOPK_MAX_WIDTH / kBlockCols;
constexpr uint32_t kAll = 0xffffffffu;
// CTA shapes (threads T): 512 threads, two CTAs per SM, when the batch needs
// more than one CTA per SM; 1024 threads, one per SM, when every row has an
// SM of its own. Per thread: kBins / T histogram bins, kMaxBlocks / T blocks.
constexpr int kSmallCta = 512;
constexpr int kLargeCta = 1024;
static_assert(kBins / kLargeCta == 2 && kBins / kSmallCta == 4, "per-thread shares of the histogram bins");
static_assert(kMaxBlocks % kLargeCta == 0, "per-thread shares of the blocks");

struct TopkParams {
  const float* logits;
  const int32_t* seq_lens;
  const int32_t* req_ids;
  const int32_t* table;
  int32_t* positions;  // optional selection rows
  int32_t* out;
  int32_t* counts;
  int32_t* status;
  int64_t stride;  // logits row stride (elements)
  int64_t table_rows;
  uint32_t table_width;
  int32_t width;  // logits columns
  int32_t k;
  int32_t cap;    // candidate list capacity (entries)
  int32_t vec;    // rows 16-byte aligned: 128-bit loads
  int32_t stage;  // block-table row staged in shared memory
  int32_t compact;
  uint32_t dcp_rank, dcp_size, interleave;
  int32_t block_size;
  FastDiv div_il, div_dcp, div_bs;
  int32_t pow2;  // interleave, dcp_size and block_size all powers of two: shifts below
  // Start the row streaming into L2 before waiting on the previous grid
  // (batches of at least half an SM count per SM; below that the rows'
  // phases, not their bytes, set a call's time).
  int32_t early_prefetch;
  uint32_t il_shift, dcp_shift, bs_shift;
  // dynamic shared memory layout (byte offsets, 16-byte aligned)
  int32_t off_boff, off_key, off_pos, off_table;
};

__device__ __forceinline__ uint32_t order_key(float v) {
  const uint32_t bits = __float_as_uint(v);
  return bits ^ (static_cast<uint32_t>(static_cast<int32_t>(bits) >> 31) | 0x80000000u);
}

// The float t such that !(x < t) holds for every x whose key is at least
// `key` (and, harmlessly, for a few more: -0 when t is +0, and every NaN). A
// key in a NaN range gives a NaN t, which admits everything.
__device__ __forceinline__ float key_floor(uint32_t key) {
  return __uint_as_float((key & 0x80000000u) ? (key ^ 0x80000000u) : ~key);
}

// Ownership and the logical block of position u (u >= 0): true when this
// rank owns u and the block is inside the request's table row
// (silkern/contract.py:132-149).
__device__ __forceinline__ bool owned(const TopkParams& p, uint32_t u, uint32_t twidth, uint32_t* lb,
                                      uint32_t* local) {
  if (p.pow2) {
    const uint32_t q1 = u >> p.il_shift;
    const uint32_t q2 = q1 >> p.dcp_shift;
    *local = (q2 << p.il_shift) | (u & (p.interleave - 1u));
    *lb = *local >> p.bs_shift;
    return (q1 & (p.dcp_size - 1u)) == p.dcp_rank && *lb < twidth;
  }
  const uint32_t q1 = fastdiv(u, p.div_il);   // u / interleave
  const uint32_t q2 = fastdiv(q1, p.div_dcp);  // u / (dcp_size * interleave)
  *local = q2 * p.interleave + (u - q1 * p.interleave);
  *lb = fastdiv(*local, p.div_bs);
  return q1 - q2 * p.dcp_size == p.dcp_rank && *lb < twidth;
}

// Exclusive prefix of v over the CTA (T threads) in thread order; *total gets
// the sum. Contains two barriers; every thread of the CTA must call it.
template <int T>
__device__ __forceinline__ int cta_scan(int v, int lane, int warp, int* s_scan, int* total) {
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(kAll, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) s_scan[warp] = x;
  __syncthreads();
  const int w = lane < T / 32 ? s_scan[lane] : 0;
  int wi = w;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(kAll, wi, o);
    if (lane >= o) wi += y;
  }
  const int base = __shfl_sync(kAll, wi - w, warp);
  *total = __shfl_sync(kAll, wi, 31);
  __syncthreads();  // s_scan may be reused
  return base + x - v;
}

// Zero a histogram; a later barrier orders it before the next fill.
template <int T>
__device__ __forceinline__ void zero_hist(uint32_t* hist, int tid) {
#pragma unroll
  for (int b = 0; b < kBins / T; ++b) hist[b * T + tid] = 0u;
}

// The histogram is complete (the caller's barrier). Returns whether its total
// reaches `want`; if so, the bin where the count of keys at or above it,
// counted from the top, first reaches `want` is published as s_pick = {bin,
// count above it, count in it}. Ends with a barrier. (s_pick is written only
// after the first barrier here, when every thread has read the last pick.)
template <int T>
__device__ __forceinline__ bool pick_bin(const uint32_t* hist, uint32_t want, int tid, int lane, int warp,
                                         int* s_scan, uint32_t* s_pick) {
  constexpr int kPer = kBins / T;  // this thread's bins: kPer * tid ..
  uint32_t h[kPer];
  if constexpr (kPer == 4) {
    const uint4 hv = *reinterpret_cast<const uint4*>(hist + kPer * tid);
    h[0] = hv.x;
    h[1] = hv.y;
    h[2] = hv.z;
    h[3] = hv.w;
  } else {
    const uint2 hv = *reinterpret_cast<const uint2*>(hist + kPer * tid);
    h[0] = hv.x;
    h[1] = hv.y;
  }
  uint32_t mine = 0u;
#pragma unroll
  for (int b = 0; b < kPer; ++b) mine += h[b];
  // count in the bins of higher threads: suffix over lanes, then warps
  uint32_t suffix = mine;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t t = __shfl_down_sync(kAll, suffix, o);
    if (lane + o < 32) suffix += t;
  }
  if (lane == 0) s_scan[warp] = static_cast<int>(suffix);
  __syncthreads();
  const uint32_t wt = lane < T / 32 ? static_cast<uint32_t>(s_scan[lane]) : 0u;
  const uint32_t above = suffix - mine + __reduce_add_sync(kAll, lane > warp ? wt : 0u);
  const uint32_t all = __reduce_add_sync(kAll, wt);
  if (above < want && want <= above + mine) {
    uint32_t a = above;
#pragma unroll
    for (int b = kPer - 1; b >= 0; --b) {
      if (a + h[b] >= want) {
        s_pick[0] = static_cast<uint32_t>(kPer * tid + b);
        s_pick[1] = a;
        s_pick[2] = h[b];
        break;
      }
      a += h[b];
    }
  }
  __syncthreads();
  return all >= want;
}

// Scores of 128-column block b of the row (this lane's four columns); columns
// at or past `len` read as 0 and must be masked by the caller.
__device__ __forceinline__ float4 load_block(const float* row, int b, int lane, int len, bool vec) {
  const int col = b * kBlockCols + 4 * lane;
  if (vec && col + 4 <= len) return __ldg(reinterpret_cast<const float4*>(row + col));
  float4 v;
  v.x = col + 0 < len ? __ldg(row + col + 0) : 0.0f;
  v.y = col + 1 < len ? __ldg(row + col + 1) : 0.0f;
  v.z = col + 2 < len ? __ldg(row + col + 2) : 0.0f;
  v.w = col + 3 < len ? __ldg(row + col + 3) : 0.0f;
  return v;
}

// Rank of (lane, j) among the set bits of a block's four masks in position
// order (lane-major, then j).
__device__ __forceinline__ int rank_in_block(const uint32_t m[4], uint32_t lt, int lane, int j) {
  int r = __popc(m[0] & lt) + __popc(m[1] & lt) + __popc(m[2] & lt) + __popc(m[3] & lt);
  for (int i = 0; i < j; ++i) r += (m[i] >> lane) & 1u;
  return r;
}

// s_boff[b] = list offset of block b (masks in s_mask, in block order), over
// `nb` blocks, kMaxBlocks / T per thread; *total gets the number of set bits.
template <int T>
__device__ __forceinline__ void block_offsets(const uint4* s_mask, int32_t* s_boff, int nb, int tid, int lane,
                                              int warp, int* s_scan, int* total) {
  constexpr int kPer = kMaxBlocks / T;
  int c[kPer];
  int mine = 0;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int b = kPer * tid + i;
    c[i] = 0;
    if (b < nb) {
      const uint4 m = s_mask[b];
      c[i] = __popc(m.x) + __popc(m.y) + __popc(m.z) + __popc(m.w);
    }
    mine += c[i];
  }
  int run = cta_scan<T>(mine, lane, warp, s_scan, total);
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int b = kPer * tid + i;
    if (b < nb) s_boff[b] = run;
    run += c[i];
  }
  __syncthreads();
}

// Lays the set bits of the blocks' masks (s_mask, `nb` blocks) out in
// position order: thread t owns a contiguous run of whole blocks, one CTA scan
// gives its first list index, and it writes the positions of its own set bits
// (those below `cap`); *total gets the CTA's count. Contains the scan's
// barriers; every thread must call it. The positions are published by the
// caller's next barrier.
template <int T>
__device__ __forceinline__ void list_positions(const uint4* s_mask, int nb, int tid, int lane, int warp,
                                               int* s_scan, int32_t* s_pos, int cap, int* total) {
  const int per = (nb + T - 1) / T;
  const int b_lo = min(nb, tid * per);
  const int b_hi = min(nb, b_lo + per);
  int c = 0;
  for (int b = b_lo; b < b_hi; ++b) {
    const uint4 m = s_mask[b];
    c += __popc(m.x) + __popc(m.y) + __popc(m.z) + __popc(m.w);
  }
  const int first = cta_scan<T>(c, lane, warp, s_scan, total);
  int idx = first;
  for (int b = b_lo; b < b_hi; ++b) {
    const uint4 m = s_mask[b];
    uint32_t any = m.x | m.y | m.z | m.w;
    const int base = b * kBlockCols;
    while (any != 0u) {  // lanes of the block in order; a lane's four columns in order
      const int l = __ffs(any) - 1;
      any &= any - 1u;
      const int col = base + 4 * l;
      if (((m.x >> l) & 1u) && idx < cap) s_pos[idx] = col;
      idx += (m.x >> l) & 1u;
      if (((m.y >> l) & 1u) && idx < cap) s_pos[idx] = col + 1;
      idx += (m.y >> l) & 1u;
      if (((m.z >> l) & 1u) && idx < cap) s_pos[idx] = col + 2;
      idx += (m.z >> l) & 1u;
      if (((m.w >> l) & 1u) && idx < cap) s_pos[idx] = col + 3;
      idx += (m.w >> l) & 1u;
    }
  }
}

template <int T>
__global__ void __launch_bounds__(T, T == kSmallCta ? 2 : 1)
    topk_localize_kernel(const __grid_constant__ TopkParams p) {
  constexpr int kTopkThreads = T;
  constexpr int kTopkWarps = T / 32;
  extern __shared__ __align__(16) unsigned char smem[];
  uint4* s_mask = reinterpret_cast<uint4*>(smem);  // per 128-column block: bit l of word j = column 4l + j
  int32_t* s_boff = reinterpret_cast<int32_t*>(smem + p.off_boff);  // list offset per block
  uint32_t* s_key = reinterpret_cast<uint32_t*>(smem + p.off_key);  // candidate list: order keys
  int32_t* s_pos = reinterpret_cast<int32_t*>(smem + p.off_pos);   // ... and positions, ascending
  int32_t* s_table = reinterpret_cast<int32_t*>(smem + p.off_table);
  __shared__ __align__(16) uint32_t s_hist[2][kBins];  // alternate between radix passes
  __shared__ int s_scan[kTopkWarps];
  __shared__ uint32_t s_pick[3];

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const uint32_t lt = lanemask_lt();
  const int64_t row = blockIdx.x;
  pdl_launch_dependents();
  int hint = -1;
  if (p.early_prefetch) {
    // The row's length as it stands before the previous grid is done, read
    // through L2 only (no copy of a value that grid may still write stays in
    // L1): a hint to start the row streaming into L2 while that grid
    // finishes. Whatever it reads (that grid may be writing it) is clamped to
    // the row and only bounds the prefetch; the length used below is read
    // after the wait. A prefetch only fills L2, the device's point of
    // coherence, so it never makes a later load stale.
    hint = __ldcg(p.seq_lens + row);
    hint = hint < 0 ? 0 : (hint > p.width ? p.width : hint);
    if (hint > p.k && p.vec) {
      const int64_t bytes = static_cast<int64_t>(hint & ~3) * 4;
      const float* base = p.logits + row * p.stride;
      for (int64_t off = static_cast<int64_t>(threadIdx.x) * kPrefetchBytes; off < bytes;
           off += static_cast<int64_t>(T) * kPrefetchBytes) {
        const int64_t m = bytes - off < kPrefetchBytes ? bytes - off : kPrefetchBytes;
        prefetch_l2_bulk(base + off / 4, static_cast<uint32_t>(m));
      }
    }
  }
  // Shared memory only, so it runs while the previous grid finishes: clear
  // both histograms (1 row: 14.90 -> 14.43 us per call; 256 rows 25.37 ->
  // 25.0).
  zero_hist<T>(s_hist[0], tid);
  zero_hist<T>(s_hist[1], tid);
  __syncthreads();
  pdl_wait();  // everything below may read what the previous grid wrote

  int len = __ldg(p.seq_lens + row);
  const bool bad_len = len < 0 || len > p.width;
  len = len < 0 ? 0 : (len > p.width ? p.width : len);
  const int32_t req = __ldg(p.req_ids + row);
  const bool req_ok = req >= 0 && static_cast<int64_t>(req) < p.table_rows;
  if (tid == 0 && p.status != nullptr) {
    if (bad_len) atomicOr(p.status, SILKERN_STATUS_BAD_LENGTH);
    if (!req_ok) atomicOr(p.status, SILKERN_STATUS_BAD_REQUEST);
  }
  const uint32_t twidth = req_ok ? p.table_width : 0u;
  const int32_t* trow = p.table + static_cast<int64_t>(req_ok ? req : 0) * p.table_width;
  if (p.stage && req_ok) {
    for (int e = tid; e < static_cast<int>(p.table_width); e += kTopkThreads) s_table[e] = __ldg(trow + e);
  }
  const int k = p.k;
  const float* lrow = p.logits + row * p.stride;
  const bool vec = p.vec != 0;
  const int nb = (len + kBlockCols - 1) / kBlockCols;  // blocks of the row
  // The estimate's first loads are on the critical path: issue them before
  // anything else reaches the memory system (columns past len count as
  // -NaN: they only lower the estimate).
  const float pad = -__int_as_float(0x7fffffff);
  auto sample = [&](int g) {
    const int col = 4 * g;
    float4 v;
    if (vec && col + 4 <= len) {
      v = __ldg(reinterpret_cast<const float4*>(lrow + col));
    } else {
      v.x = __ldg(lrow + col);
      v.y = col + 1 < len ? __ldg(lrow + col + 1) : pad;
      v.z = col + 2 < len ? __ldg(lrow + col + 2) : pad;
      v.w = col + 3 < len ? __ldg(lrow + col + 3) : pad;
    }
    return v;
  };
  const int g0 = kSampleEvery * tid;
  const int g1 = g0 + kSampleEvery * kTopkThreads;
  // The estimate histogram holds 4 values per sampled float4 (padding
  // included); a row with fewer than `want_sample` of them has no floor to
  // find, and lists every column.
  const uint32_t want_sample = static_cast<uint32_t>(k / kSampleEvery + k / (2 * kSampleEvery) + 16);
  const uint32_t sample_values = 4u * static_cast<uint32_t>((len + 4 * kSampleEvery - 1) / (4 * kSampleEvery));
  const bool sampled = len > k && sample_values >= want_sample;
  float4 first[2];
  if (sampled) {
    if (4 * g0 < len) first[0] = sample(g0);
    if (4 * g1 < len) first[1] = sample(g1);
  }
  if (len > k && vec && len != hint) {
    // Start the whole row streaming into L2 now (unless the early prefetch
    // above already did); the stream pass below then mostly hits L2.
    const int64_t bytes = static_cast<int64_t>(len & ~3) * 4;
    for (int64_t off = static_cast<int64_t>(tid) * kPrefetchBytes; off < bytes;
         off += static_cast<int64_t>(kTopkThreads) * kPrefetchBytes) {
      const int64_t n = bytes - off < kPrefetchBytes ? bytes - off : kPrefetchBytes;
      prefetch_l2_bulk(lrow + off / 4, static_cast<uint32_t>(n));
    }
  }

  // The list: `total` entries in position order holding every selected
  // position. `prefix` is the threshold key: when `need` equals `eq_total`
  // every key at or above it is taken, otherwise every key above it and the
  // `need` lowest-positioned of the `eq_total` keys equal to it.
  // `all_selected` when the list is exactly the selection (short rows, and
  // the whole-row path).
  int total = 0;
  uint32_t prefix = 0;
  int need = 0;
  int eq_total = 0;
  bool all_selected = true;

  if (len > k) {
    // 1. estimate from every 16th float4 (both histograms were cleared
    // before the wait)
    uint32_t lo_bin = 0u;
    if (sampled) {
      auto count = [&](const float4& v) {
        atomicAdd(&s_hist[0][order_key(v.x) >> 21], 1u);
        atomicAdd(&s_hist[0][order_key(v.y) >> 21], 1u);
        atomicAdd(&s_hist[0][order_key(v.z) >> 21], 1u);
        atomicAdd(&s_hist[0][order_key(v.w) >> 21], 1u);
      };
      if (4 * g0 < len) count(first[0]);
      if (4 * g1 < len) count(first[1]);
      for (int g = g1 + kSampleEvery * kTopkThreads; 4 * g < len; g += kSampleEvery * kTopkThreads) {
        count(sample(g));
      }
      __syncthreads();
      lo_bin = pick_bin<T>(s_hist[0], want_sample, tid, lane, warp, s_scan, s_pick) ? s_pick[0] : 0u;
      zero_hist<T>(s_hist[0], tid);  // the first radix pass's (the barriers below order it)
    }
    const float floor_value = key_floor(lo_bin << 21);

    // 2. stream the row once, keeping candidate masks
    for (int b0 = warp; b0 < nb; b0 += kTopkWarps * kStreamUnroll) {
      float4 v[kStreamUnroll];
#pragma unroll
      for (int u = 0; u < kStreamUnroll; ++u) {
        const int b = b0 + u * kTopkWarps;
        if (b < nb) v[u] = load_block(lrow, b, lane, len, vec);
      }
#pragma unroll
      for (int u = 0; u < kStreamUnroll; ++u) {
        const int b = b0 + u * kTopkWarps;
        if (b >= nb) break;
        const int lim = len - (b * kBlockCols + 4 * lane);
        const uint32_t w0 = __ballot_sync(kAll, 0 < lim && !(v[u].x < floor_value));
        const uint32_t w1 = __ballot_sync(kAll, 1 < lim && !(v[u].y < floor_value));
        const uint32_t w2 = __ballot_sync(kAll, 2 < lim && !(v[u].z < floor_value));
        const uint32_t w3 = __ballot_sync(kAll, 3 < lim && !(v[u].w < floor_value));
        if (lane == 0) s_mask[b] = make_uint4(w0, w1, w2, w3);
      }
    }
    __syncthreads();

    // 3. the list in position order: each thread lists the candidates of its
    // own blocks; then all threads load the keys, consecutive entries on
    // consecutive lanes, eight in flight per lane (L2 hits), which feed the
    // first radix histogram. (Per-thread key loads would serialise on dense
    // blocks: a short row, or heavy ties, lists every column.)
    list_positions<T>(s_mask, nb, tid, lane, warp, s_scan, s_pos, p.cap, &total);
    bool whole_row = total > p.cap;
    if (!whole_row) {
      __syncthreads();  // publishes s_pos
      for (int i0 = tid; i0 < total; i0 += 8 * kTopkThreads) {
        uint32_t kk[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int i = i0 + u * kTopkThreads;
          kk[u] = i < total ? order_key(__ldg(lrow + s_pos[i])) : 0u;
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int i = i0 + u * kTopkThreads;
          if (i < total) {
            s_key[i] = kk[u];
            atomicAdd(&s_hist[0][kk[u] >> 21], 1u);
          }
        }
      }
      __syncthreads();

      // 4. exact radix select over the list (first pass counted above). The
      // passes alternate histograms: each pass clears the one the next uses.
      // A pass whose threshold bin is taken whole ends the select; `prefix`
      // then becomes the bin's lowest key.
      need = k;
      int rest = 0;
#pragma unroll 1
      for (int pass = 0; pass < 3; ++pass) {
        const int shift = pass == 0 ? 21 : (pass == 1 ? 10 : 0);
        const int bits = pass == 2 ? 10 : 11;
        uint32_t* hist = s_hist[pass & 1];
        if (pass > 0) {
          if (pass == 1) zero_hist<T>(s_hist[0], tid);
          for (int i = tid; i < total; i += kTopkThreads) {
            const uint32_t key = s_key[i];
            if ((key >> (shift + bits)) == prefix) atomicAdd(&hist[(key >> shift) & (kBins - 1)], 1u);
          }
          __syncthreads();
        }
        const bool found = pick_bin<T>(hist, static_cast<uint32_t>(need), tid, lane, warp, s_scan, s_pick);
        if (pass == 0 && !(found && s_pick[0] >= lo_bin)) {
          whole_row = true;  // fewer than top_k scores above the floor
          break;
        }
        prefix = (prefix << bits) | s_pick[0];
        need -= static_cast<int>(s_pick[1]);
        eq_total = static_cast<int>(s_pick[2]);
        rest = shift;
        if (eq_total == need) break;
      }
      prefix <<= rest;
      all_selected = whole_row;
    }

    if (whole_row) {
      // Threshold from radix passes over the whole row, then list exactly the
      // selected positions: every key above it, and the `need` lowest-
      // positioned keys equal to it.
      prefix = 0;
      need = k;
      int rest = 0;
#pragma unroll 1
      for (int pass = 0; pass < 3; ++pass) {
        const int shift = pass == 0 ? 21 : (pass == 1 ? 10 : 0);
        const int bits = pass == 2 ? 10 : 11;
        zero_hist<T>(s_hist[0], tid);
        __syncthreads();
        for (int b = warp; b < nb; b += kTopkWarps) {
          const float4 v = load_block(lrow, b, lane, len, vec);
          const float vv[4] = {v.x, v.y, v.z, v.w};
          const int col = b * kBlockCols + 4 * lane;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t key = order_key(vv[j]);
            if (col + j < len && ((key >> shift) >> bits) == prefix) {
              atomicAdd(&s_hist[0][(key >> shift) & (kBins - 1)], 1u);
            }
          }
        }
        __syncthreads();
        (void)pick_bin<T>(s_hist[0], static_cast<uint32_t>(need), tid, lane, warp, s_scan, s_pick);
        prefix = (prefix << bits) | s_pick[0];
        need -= static_cast<int>(s_pick[1]);
        eq_total = static_cast<int>(s_pick[2]);
        rest = shift;
        if (eq_total == need) break;  // the threshold bin is taken whole
      }
      prefix <<= rest;  // the lowest key taken when no tie is cut
      const bool tie_cut = eq_total != need;
      if (tie_cut) {
        // masks of the keys equal to the threshold, and their block offsets
        for (int b = warp; b < nb; b += kTopkWarps) {
          const float4 v = load_block(lrow, b, lane, len, vec);
          const int lim = len - (b * kBlockCols + 4 * lane);
          const uint32_t w0 = __ballot_sync(kAll, 0 < lim && order_key(v.x) == prefix);
          const uint32_t w1 = __ballot_sync(kAll, 1 < lim && order_key(v.y) == prefix);
          const uint32_t w2 = __ballot_sync(kAll, 2 < lim && order_key(v.z) == prefix);
          const uint32_t w3 = __ballot_sync(kAll, 3 < lim && order_key(v.w) == prefix);
          if (lane == 0) s_mask[b] = make_uint4(w0, w1, w2, w3);
        }
        __syncthreads();
        int eqs;
        block_offsets<T>(s_mask, s_boff, nb, tid, lane, warp, s_scan, &eqs);
      }
      // selection masks (each warp rewrites only the blocks it read)
      for (int b = warp; b < nb; b += kTopkWarps) {
        const float4 v = load_block(lrow, b, lane, len, vec);
        const float vv[4] = {v.x, v.y, v.z, v.w};
        const int lim = len - (b * kBlockCols + 4 * lane);
        uint32_t eqm[4] = {0u, 0u, 0u, 0u};
        int eq_base = 0;
        if (tie_cut) {
          const uint4 e = s_mask[b];
          eqm[0] = e.x;
          eqm[1] = e.y;
          eqm[2] = e.z;
          eqm[3] = e.w;
          eq_base = s_boff[b];
        }
        uint32_t w[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t key = order_key(vv[j]);
          bool sel = j < lim && key > prefix;
          if (j < lim && key == prefix) sel = !tie_cut || eq_base + rank_in_block(eqm, lt, lane, j) < need;
          w[j] = __ballot_sync(kAll, sel);
        }
        if (lane == 0) s_mask[b] = make_uint4(w[0], w[1], w[2], w[3]);
      }
      __syncthreads();
      list_positions<T>(s_mask, nb, tid, lane, warp, s_scan, s_pos, p.cap, &total);
      total = total < p.cap ? total : p.cap;  // exactly top_k <= cap
    }
  } else {
    total = len;  // every position, listed implicitly: entry i is position i
  }
  __syncthreads();  // the list and the staged table row are complete

  // 5. emit. Warp w owns list entries [w * seg, (w + 1) * seg), seg a
  // multiple of 32, its lanes on consecutive entries; ranks come from
  // ballots and one exchange of the warps' totals.
  const bool implicit = len <= k;
  const bool rank_ties = !all_selected && eq_total != need;
  const int seg = ((total + kTopkWarps - 1) / kTopkWarps + 31) & ~31;
  const int lo = min(total, warp * seg);
  const int hi = min(total, lo + seg);
  int eq_rank = 0;
  if (rank_ties) {  // keys equal to the threshold in the warps before this one
    int c = 0;
    for (int i0 = lo; i0 < hi; i0 += 32) {
      const int i = i0 + lane;
      c += __popc(__ballot_sync(kAll, i < hi && s_key[i] == prefix));
    }
    if (lane == 0) s_scan[warp] = c;
    __syncthreads();
    const int w = lane < kTopkWarps ? s_scan[lane] : 0;
    eq_rank = __reduce_add_sync(kAll, lane < warp ? w : 0);
  }
  // Count pass. Each entry's slots then hold its result: s_pos the position
  // with bit 30 set when selected and bit 29 when valid, s_key (the key is no
  // longer needed) the physical slot.
  constexpr int32_t kSel = 1 << 30, kValid = 1 << 29;
  int nsel = 0, nvalid = 0;  // this warp's
#pragma unroll 2
  for (int i0 = lo; i0 < hi; i0 += 32) {
    // branch-free: every lane reads an entry of the list (lanes past the
    // end re-read the first) and computes its ownership and slot
    const int i = i0 + lane;
    const bool in = i < hi;
    const int ic = in ? i : lo;
    const int32_t pos = implicit ? ic : s_pos[ic];
    bool sel = in;
    if (!all_selected) {
      const uint32_t key = s_key[ic];
      const bool eq = in && key == prefix;
      sel = in && key > prefix;
      if (rank_ties) {
        const uint32_t eqb = __ballot_sync(kAll, eq);
        sel = sel || (eq && eq_rank + __popc(eqb & lt) < need);
        eq_rank += __popc(eqb);
      } else {
        sel = sel || eq;
      }
    }
    uint32_t lb, local;
    const bool own = owned(p, static_cast<uint32_t>(pos), twidth, &lb, &local);
    const bool valid = sel && own;
    const uint32_t lbc = own ? lb : 0u;  // an entry of the row (read, unused, when not owned)
    const int32_t blk = p.stage ? s_table[lbc] : __ldg(trow + lbc);
    const int32_t phys =
        valid ? static_cast<int32_t>((static_cast<uint32_t>(blk) - lb) * static_cast<uint32_t>(p.block_size) + local)
              : -1;
    if (in) {
      s_key[i] = static_cast<uint32_t>(phys);
      s_pos[i] = sel ? (pos | kSel | (valid ? kValid : 0)) : 0;
    }
    nsel += __popc(__ballot_sync(kAll, sel));
    nvalid += __popc(__ballot_sync(kAll, valid));
  }
  // both counts in one exchange: selected in the high half, valid in the low
  __shared__ int s_wsum[kTopkWarps];
  if (lane == 0) s_wsum[warp] = (nsel << 16) | nvalid;
  __syncthreads();
  const int wsum = lane < kTopkWarps ? s_wsum[lane] : 0;
  const int both = __reduce_add_sync(kAll, lane < warp ? wsum : 0);
  const int both_total = __reduce_add_sync(kAll, wsum);
  int js = both >> 16, jv = both & 0xffff;
  const int sel_total = both_total >> 16, valid_total = both_total & 0xffff;
  int32_t* prow = p.positions != nullptr ? p.positions + row * k : nullptr;
  int32_t* orow = p.out + row * k;
#pragma unroll 2
  for (int i0 = lo; i0 < hi; i0 += 32) {
    const int i = i0 + lane;
    const bool in = i < hi;
    const int32_t f = in ? s_pos[i] : 0;
    const int32_t phys = static_cast<int32_t>(s_key[in ? i : lo]);
    const bool sel = (f & kSel) != 0;
    const bool valid = (f & kValid) != 0;
    const uint32_t selb = __ballot_sync(kAll, sel);
    const uint32_t validb = __ballot_sync(kAll, valid);
    const int s = js + __popc(selb & lt);
    const int v = jv + __popc(validb & lt);
    if (prow != nullptr && sel && s < k) prow[s] = f & (kValid - 1);
    if (p.compact) {
      if (valid && v < k) orow[v] = phys;
    } else if (sel && s < k) {
      orow[s] = phys;
    }
    js += __popc(selb);
    jv += __popc(validb);
  }
  const int n_sel = min(sel_total, k);
  if (prow != nullptr) {
    for (int e = n_sel + tid; e < k; e += kTopkThreads) prow[e] = -1;
  }
  for (int e = (p.compact ? min(valid_total, k) : n_sel) + tid; e < k; e += kTopkThreads) orow[e] = -1;
  if (tid == 0) p.counts[row] = valid_total;
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

bool byte_overlap(const void* a, int64_t a_bytes, const void* b, int64_t b_bytes) {
  if (a == nullptr || b == nullptr || a_bytes <= 0 || b_bytes <= 0) return false;
  const uintptr_t a0 = reinterpret_cast<uintptr_t>(a), b0 = reinterpret_cast<uintptr_t>(b);
  return a0 < b0 + static_cast<uintptr_t>(b_bytes) && b0 < a0 + static_cast<uintptr_t>(a_bytes);
}

// Per device: the SM count, and the dynamic shared memory granted so far to
// each CTA shape's kernel (above the default it needs an opt-in per kernel
// and device).
struct TopkDevice {
  int sms = 0;
  size_t granted[2] = {0, 0};  // 512- and 1024-thread kernels
};

int topk_device(int* dev, TopkDevice** out) {
  static TopkDevice devices[64];
  if (cudaGetDevice(dev) != cudaSuccess || *dev < 0 || *dev >= 64) {
    const cudaError_t err = cudaGetLastError();
    return -static_cast<int>(err == cudaSuccess ? cudaErrorInvalidDevice : err);
  }
  *out = &devices[*dev];
  return SILKERN_OK;
}

int topk_prepare(int threads, size_t smem_bytes, int* sms) {
  static std::mutex mutex;
  int dev = 0;
  TopkDevice* d = nullptr;
  const int rc = topk_device(&dev, &d);
  if (rc != SILKERN_OK) return rc;
  std::lock_guard<std::mutex> lock(mutex);
  if (d->sms == 0) {
    int n = 0;
    const cudaError_t err = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (err != cudaSuccess) {
      (void)cudaGetLastError();
      return -static_cast<int>(err);
    }
    d->sms = n;
  }
  *sms = d->sms;
  if (threads == 0) return SILKERN_OK;
  const int slot = threads == kLargeCta ? 1 : 0;
  if (d->granted[slot] >= smem_bytes) return SILKERN_OK;
  const cudaError_t err = cudaFuncSetAttribute(
      threads == kLargeCta ? topk_localize_kernel<kLargeCta> : topk_localize_kernel<kSmallCta>,
      cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem_bytes));
  if (err != cudaSuccess) {
    (void)cudaGetLastError();
    return -static_cast<int>(err);
  }
  d->granted[slot] = smem_bytes;
  return SILKERN_OK;
}

int align16(int64_t v) { return static_cast<int>((v + 15) & ~int64_t{15}); }

int topk_launch(const float* logits, int64_t stride, int64_t width, const int32_t* seq_lens,
                const int32_t* req_ids, const int32_t* table, int64_t table_rows, int64_t table_width,
                int32_t* positions, int32_t* out, int32_t* counts, int64_t batch, int32_t top_k,
                int32_t block_size, int32_t dcp_size, int32_t dcp_rank, int32_t interleave, int32_t compact,
                int32_t cap_req, int32_t stage_req, int32_t threads_req, int32_t* status, cudaStream_t stream) {
  if (!logits || !seq_lens || !req_ids || !table || !out || !counts) return SILKERN_E_NULL;
  if (batch < 1 || batch > INT32_MAX || width < 1 || width > SILKERN_TOPK_MAX_WIDTH || stride < width ||
      top_k < 1 || top_k > SILKERN_MAX_ROW_WIDTH || table_rows < 1 || table_width < 1 || table_width > INT32_MAX) {
    return SILKERN_E_SHAPE;
  }
  if (dcp_size < 1 || dcp_rank < 0 || dcp_rank >= dcp_size || interleave < 1) return SILKERN_E_DCP;
  if (block_size < 1 || block_size % interleave != 0) return SILKERN_E_BLOCK_SIZE;

  // Inputs and outputs, in bytes, must not overlap (outputs among themselves either).
  const int64_t logit_bytes = ((batch - 1) * stride + width) * 4;
  struct Range {
    const void* p;
    int64_t bytes;
  };
  const Range inputs[4] = {{logits, logit_bytes}, {seq_lens, batch * 4}, {req_ids, batch * 4},
                           {table, table_rows * table_width * 4}};
  const Range outputs[3] = {{positions, batch * top_k * 4}, {out, batch * top_k * 4}, {counts, batch * 4}};
  for (const Range& o : outputs) {
    for (const Range& in : inputs) {
      if (byte_overlap(o.p, o.bytes, in.p, in.bytes)) return SILKERN_E_ALIAS;
    }
  }
  for (int a = 0; a < 3; ++a) {
    for (int b = a + 1; b < 3; ++b) {
      if (byte_overlap(outputs[a].p, outputs[a].bytes, outputs[b].p, outputs[b].bytes)) return SILKERN_E_ALIAS;
    }
  }

  int stage;
  if (stage_req < 0) {
    stage = table_width <= kTableStageMax ? 1 : 0;
  } else {
    if (stage_req > 1 || (stage_req == 1 && table_width > kTableStageMax)) return SILKERN_E_GEOMETRY;
    stage = stage_req;
  }
  // Candidate list: room for the usual ~1.5 x top_k candidates plus the
  // floor bin's spill, within the shared-memory budget, never below top_k
  // (the whole-row path lists exactly top_k). The explicit entry point may
  // shrink it to force that path.
  const int64_t nblocks = (width + kBlockCols - 1) / kBlockCols;
  const int64_t fixed = align16(nblocks * 16) + align16(nblocks * 4) + (stage ? align16(table_width * 4) : 0);
  const int64_t cap_max = (kTopkSmemBudget - fixed) / 8 / 4 * 4;
  int64_t cap = int64_t{3} * top_k + 2048;
  if (cap > cap_max) cap = cap_max;
  if (cap_req != 0) {
    if (cap_req > cap_max || cap_req >= 65536) return SILKERN_E_GEOMETRY;
    cap = cap_req;
  }
  if (cap < top_k) return SILKERN_E_GEOMETRY;
  TopkParams p{};
  p.off_boff = align16(nblocks * 16);
  p.off_key = p.off_boff + align16(nblocks * 4);
  p.off_pos = p.off_key + align16(cap * 4);
  p.off_table = p.off_pos + align16(cap * 4);
  const int64_t smem = p.off_table + (stage ? align16(table_width * 4) : 0);
  // CTA shape: 1024 threads when every row gets an SM of its own
  if (threads_req != 0 && threads_req != kSmallCta && threads_req != kLargeCta) return SILKERN_E_GEOMETRY;
  int sms = 0;
  int rc = topk_prepare(0, 0, &sms);
  if (rc != SILKERN_OK) return rc;
  const int threads = threads_req != 0 ? threads_req : (batch <= sms ? kLargeCta : kSmallCta);
  rc = topk_prepare(threads, static_cast<size_t>(smem), &sms);
  if (rc != SILKERN_OK) return rc;

  p.logits = logits;
  p.seq_lens = seq_lens;
  p.req_ids = req_ids;
  p.table = table;
  p.positions = positions;
  p.out = out;
  p.counts = counts;
  p.status = status;
  p.stride = stride;
  p.table_rows = table_rows;
  p.table_width = static_cast<uint32_t>(table_width);
  p.width = static_cast<int32_t>(width);
  p.k = top_k;
  p.cap = static_cast<int32_t>(cap);
  p.vec = ((reinterpret_cast<uintptr_t>(logits) & 15u) == 0 && stride % 4 == 0) ? 1 : 0;
  p.stage = stage;
  p.compact = (compact != 0 && dcp_size > 1) ? 1 : 0;
  p.dcp_rank = static_cast<uint32_t>(dcp_rank);
  p.dcp_size = static_cast<uint32_t>(dcp_size);
  p.interleave = static_cast<uint32_t>(interleave);
  p.block_size = block_size;
  p.div_il = make_fastdiv(p.interleave);
  p.div_dcp = make_fastdiv(p.dcp_size);
  p.div_bs = make_fastdiv(static_cast<uint32_t>(block_size));
  auto pow2_shift = [](uint32_t v, uint32_t* shift) {
    if ((v & (v - 1u)) != 0u) return false;
    uint32_t s = 0;
    while ((1u << s) < v) ++s;
    *shift = s;
    return true;
  };
  p.pow2 = (pow2_shift(p.interleave, &p.il_shift) && pow2_shift(p.dcp_size, &p.dcp_shift) &&
            pow2_shift(static_cast<uint32_t>(block_size), &p.bs_shift))
               ? 1
               : 0;
  // Early prefetch from half a row per SM: 256 rows of up to 65536 scores
  // measured 28.5 -> 25.3 us per call, 148 rows 17.9 -> 16.4; at 64 rows
  // and below it was slower (64 rows: 16.9 against 16.3).
  p.early_prefetch = 2 * batch >= static_cast<int64_t>(sms) ? 1 : 0;

  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(batch), 1, 1);
  cfg.blockDim = dim3(static_cast<unsigned>(threads), 1, 1);
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cfg.stream = stream;
  cudaLaunchAttribute attrs[1];
  attrs[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attrs;
  cfg.numAttrs = 1;
  const cudaError_t err = threads == kLargeCta ? cudaLaunchKernelEx(&cfg, topk_localize_kernel<kLargeCta>, p)
                                               : cudaLaunchKernelEx(&cfg, topk_localize_kernel<kSmallCta>, p);
  if (err != cudaSuccess) {
    (void)cudaGetLastError();
    return -static_cast<int>(err);
  }
  return SILKERN_OK;
}

}  // namespace
}  // namespace silkern

extern "C" int silkern_topk_localize_v1(const float* logits, int64_t logits_stride, int64_t logits_width,
                                        const int32_t* seq_lens, const int32_t* req_ids,
                                        const int32_t* block_table, int64_t table_rows, int64_t table_width,
                                        int32_t* positions, int32_t* out, int32_t* counts, int64_t batch,
                                        int32_t top_k, int32_t block_size, int32_t dcp_size, int32_t dcp_rank,
                                        int32_t dcp_interleave, int32_t compact_valid_to_front,
                                        int32_t* status, void* stream) {
  return silkern::topk_launch(logits, logits_stride, logits_width, seq_lens, req_ids, block_table, table_rows,
                              table_width, positions, out, counts, batch, top_k, block_size, dcp_size, dcp_rank,
                              dcp_interleave, compact_valid_to_front, 0, -1, 0, status,
                              static_cast<cudaStream_t>(stream));
}

extern "C" int silkern_topk_localize_explicit_v2(
    const float* logits, int64_t logits_stride, int64_t logits_width, const int32_t* seq_lens,
    const int32_t* req_ids, const int32_t* block_table, int64_t table_rows, int64_t table_width,
    int32_t* positions, int32_t* out, int32_t* counts, int64_t batch, int32_t top_k, int32_t block_size,
    int32_t dcp_size, int32_t dcp_rank, int32_t dcp_interleave, int32_t compact_valid_to_front,
    int32_t candidate_capacity, int32_t stage_table, int32_t cta_threads, int32_t* status, void* stream) {
  if (candidate_capacity < 0 || stage_table < -1 || cta_threads < 0) return SILKERN_E_GEOMETRY;
  return silkern::topk_launch(logits, logits_stride, logits_width, seq_lens, req_ids, block_table, table_rows,
                              table_width, positions, out, counts, batch, top_k, block_size, dcp_size, dcp_rank,
                              dcp_interleave, compact_valid_to_front, candidate_capacity, stage_table, cta_threads,
                              status, static_cast<cudaStream_t>(stream));
}

extern "C" int silkern_topk_localize_explicit_v1(
    const float* logits, int64_t logits_stride, int64_t logits_width, const int32_t* seq_lens,
    const int32_t* req_ids, const int32_t* block_table, int64_t table_rows, int64_t table_width,
    int32_t* positions, int32_t* out, int32_t* counts, int64_t batch, int32_t top_k, int32_t block_size,
    int32_t dcp_size, int32_t dcp_rank, int32_t dcp_interleave, int32_t compact_valid_to_front,
    int32_t candidate_capacity, int32_t stage_table, int32_t* status, void* stream) {
  return silkern_topk_localize_explicit_v2(logits, logits_stride, logits_width, seq_lens, req_ids, block_table,
                                           table_rows, table_width, positions, out, counts, batch, top_k,
                                           block_size, dcp_size, dcp_rank, dcp_interleave,
                                           compact_valid_to_front, candidate_capacity, stage_table, 0, status,
                                           stream);
}
