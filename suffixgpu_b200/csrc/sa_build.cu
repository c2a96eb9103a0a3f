// Suffix-array construction for sm_100a: prefix doubling over the still
// tied suffixes, each round sorted with a hand-written stable LSD radix
// sort.
//
// Result: identical to suffix_gpu/suffix_array.py:15-63 (the suffix array
// is unique: suffixes at distinct positions differ, end of string sorts
// first). The reference re-sorts all n packed (rank, rank[i+k]) keys with
// torch.argsort for ceil(log2 n) rounds; here
//   * ranks are group starts (the SA index of the first suffix of each
//     group of equal 2^r-prefixes), so a suffix whose group has one member
//     is final and leaves the active set (Larsson-Sadakane doubling);
//   * a round sorts only the active suffixes by the packed key
//     (group start << SB) | (i + h < n ? rank[i + h] + 1 : 0);
//     group starts are contiguous in SA order, so the sorted active list
//     maps one-to-one onto the active SA slots;
//   * one scan pass then writes SA entries, new group-start ranks and the
//     next active list; the build stops when no group is left (no fixed
//     round count).
// Radix sort: 8-bit digits; per 4096-key tile a digit histogram, a
// per-digit scan over tiles, and a stable scatter that ranks each 32-key
// warp round with 8 ballots (no __match_any_sync, which is slow on
// sm_100a).
// Segmented rounds: the active list is in SA order, so it is already
// grouped; a round only has to order each group by its second key. Groups
// of at most kSegHalo suffixes (on copy-heavy text nearly all of them:
// 10 M of 16 M suffixes stay active for 8 rounds, in groups of a few) are
// ranked in shared memory by the block whose tile holds their head, in one
// pass; only the suffixes of larger groups are compacted, radix-sorted by
// (group, second key) and scattered back into their groups' slots.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <mutex>

#include "sg_common.cuh"

namespace sg {

constexpr int kSortThreads = 256;
constexpr int kSortWarps = kSortThreads / 32;
constexpr int kSortItems = 16;                    // keys per thread
constexpr int kTile = kSortThreads * kSortItems;  // 4096 keys per tile
// Small lists (fewer than two 4096-element tiles per SM: the rebuild's
// tail sorts, short corpora) use 1024-element tiles in the sort and scan
// passes, so that their blocks still cover the SMs.
constexpr int kItemsSmall = 4;

// ---------------------------------------------------------------------------
// radix sort passes
// ---------------------------------------------------------------------------
template <int ITEMS>
__global__ void __launch_bounds__(kSortThreads)
    rs_hist_kernel(const uint64_t* __restrict__ keys, int64_t m, int shift,
                   uint32_t* __restrict__ tile_hist, int ntiles,
                   uint32_t* __restrict__ totals) {
  __shared__ uint32_t h[kSortWarps][256];
  const int t = threadIdx.x, warp = warp_id();
  for (int i = t; i < kSortWarps * 256; i += kSortThreads) (&h[0][0])[i] = 0;
  __syncthreads();
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kSortThreads * ITEMS;
#pragma unroll
  for (int r = 0; r < ITEMS; ++r) {
    const int64_t idx = base + r * kSortThreads + t;
    if (idx < m) atomicAdd(&h[warp][(keys[idx] >> shift) & 255], 1u);
  }
  __syncthreads();
  uint32_t s = 0;
#pragma unroll
  for (int w = 0; w < kSortWarps; ++w) s += h[w][t];
  tile_hist[static_cast<int64_t>(t) * ntiles + blockIdx.x] = s;
  if (s) atomicAdd(&totals[t], s);
}

// Block d: exclusive scan of digit d's per-tile counts, offset by the
// number of keys with a smaller digit.
__global__ void __launch_bounds__(kSortThreads)
    rs_scan_kernel(uint32_t* __restrict__ tile_hist, int ntiles,
                   const uint32_t* __restrict__ totals) {
  __shared__ uint32_t warp_sums[kSortWarps];
  const int d = blockIdx.x, t = threadIdx.x;
  const int warp = warp_id(), lane = lane_id();
  // digit start = sum of totals[0..d)
  uint32_t v = t < d ? totals[t] : 0u;
  v = __reduce_add_sync(SG_FULL_MASK, v);
  if (lane == 0) warp_sums[warp] = v;
  __syncthreads();
  uint32_t carry = 0;
#pragma unroll
  for (int w = 0; w < kSortWarps; ++w) carry += warp_sums[w];
  __syncthreads();
  uint32_t* row = tile_hist + static_cast<int64_t>(d) * ntiles;
  for (int c0 = 0; c0 < ntiles; c0 += kSortThreads) {
    const int i = c0 + t;
    const uint32_t x = i < ntiles ? row[i] : 0u;
    const uint32_t inc =
        static_cast<uint32_t>(warp_incl_scan(static_cast<int>(x)));
    if (lane == 31) warp_sums[warp] = inc;
    __syncthreads();
    uint32_t pre = 0, tot = 0;
#pragma unroll
    for (int w = 0; w < kSortWarps; ++w) {
      const uint32_t y = warp_sums[w];
      if (w < warp) pre += y;
      tot += y;
    }
    if (i < ntiles) row[i] = carry + pre + inc - x;
    carry += tot;
    __syncthreads();
  }
}

__global__ void zero_u32_kernel(uint32_t* p, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) p[i] = 0u;
}

template <int ITEMS>
__global__ void __launch_bounds__(kSortThreads)
    rs_scatter_kernel(const uint64_t* __restrict__ kin,
                      const uint32_t* __restrict__ vin,
                      uint64_t* __restrict__ kout, uint32_t* __restrict__ vout,
                      int64_t m, int shift,
                      const uint32_t* __restrict__ offs, int ntiles) {
  __shared__ uint32_t wcnt[kSortWarps][256];
  __shared__ uint32_t s_off[256];
  const int t = threadIdx.x, warp = warp_id(), lane = lane_id();
  const unsigned lt_mask = (1u << lane) - 1u;
  for (int i = lane; i < 256; i += 32) wcnt[warp][i] = 0u;
  s_off[t] = offs[static_cast<int64_t>(t) * ntiles + blockIdx.x];
  // warp w owns keys [base, base + 512) of the tile, 32 per round in order
  const int64_t base =
      static_cast<int64_t>(blockIdx.x) * kSortThreads * ITEMS + warp * (32 * ITEMS);
  uint64_t key[ITEMS];
  uint32_t val[ITEMS];
  uint32_t loc[ITEMS];
#pragma unroll
  for (int r = 0; r < ITEMS; ++r) {
    const int64_t idx = base + r * 32 + lane;
    key[r] = idx < m ? kin[idx] : 0ull;
    val[r] = idx < m ? vin[idx] : 0u;
  }
  __syncwarp();
  // stable rank of every key among this warp's keys with the same digit
#pragma unroll
  for (int r = 0; r < ITEMS; ++r) {
    const int64_t idx = base + r * 32 + lane;
    const bool valid = idx < m;
    const uint32_t d = static_cast<uint32_t>(key[r] >> shift) & 255u;
    unsigned peers = __ballot_sync(SG_FULL_MASK, valid);
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      const unsigned bal =
          __ballot_sync(SG_FULL_MASK, valid && ((d >> b) & 1u));
      peers &= ((d >> b) & 1u) ? bal : ~bal;
    }
    const int leader = valid ? __ffs(peers) - 1 : lane;
    uint32_t old = 0;
    if (valid && lane == leader) {
      old = wcnt[warp][d];
      wcnt[warp][d] = old + __popc(peers);
    }
    old = __shfl_sync(SG_FULL_MASK, old, leader);
    loc[r] = old + __popc(peers & lt_mask);
    __syncwarp();
  }
  __syncthreads();
  // exclusive prefix over warps, per digit (thread t = digit t)
  {
    uint32_t run = 0;
#pragma unroll
    for (int w = 0; w < kSortWarps; ++w) {
      const uint32_t c = wcnt[w][t];
      wcnt[w][t] = run;
      run += c;
    }
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < ITEMS; ++r) {
    const int64_t idx = base + r * 32 + lane;
    if (idx < m) {
      const uint32_t d = static_cast<uint32_t>(key[r] >> shift) & 255u;
      const uint32_t pos = s_off[d] + wcnt[warp][d] + loc[r];
      kout[pos] = key[r];
      vout[pos] = val[r];
    }
  }
}

// ---------------------------------------------------------------------------
// doubling rounds
// ---------------------------------------------------------------------------
constexpr int kScanThreads = 256;
constexpr int kScanItems = 16;

__global__ void init_keys_kernel(const int32_t* __restrict__ tok, int64_t n,
                                 uint64_t* __restrict__ keys,
                                 uint32_t* __restrict__ vals) {
  const int64_t i =
      static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) {
    // order-preserving map of signed int32 to unsigned
    keys[i] = static_cast<uint32_t>(tok[i]) ^ 0x80000000u;
    vals[i] = static_cast<uint32_t>(i);
  }
}

__global__ void make_keys_kernel(const uint32_t* __restrict__ act,
                                 const int32_t* __restrict__ sa,
                                 const uint32_t* __restrict__ rank, int64_t n,
                                 int64_t m, int64_t h, int sb,
                                 uint64_t* __restrict__ keys,
                                 uint32_t* __restrict__ vals) {
  const int64_t t =
      static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (t >= m) return;
  const int64_t i = sa[act[t]];
  const uint64_t second =
      i + h < n ? static_cast<uint64_t>(rank[i + h]) + 1 : 0;
  keys[t] = (static_cast<uint64_t>(rank[i]) << sb) | second;
  vals[t] = static_cast<uint32_t>(i);
}

// Dense token ids for the two-token pass. After the first-token sort,
// block b counts the heads (first element of each run of equal tokens) of
// its elements; blk_max is zeroed so that round_scan_blocks_kernel serves.
template <int ITEMS>
__global__ void __launch_bounds__(kScanThreads)
    dense_count_kernel(const uint64_t* __restrict__ K, int64_t m,
                       uint32_t* __restrict__ blk_max,
                       uint32_t* __restrict__ blk_sum) {
  __shared__ uint32_t ss[kSortWarps];
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kScanThreads * ITEMS;
  uint32_t sum = 0;
  for (int r = 0; r < ITEMS; ++r) {
    const int64_t t = base + r * kScanThreads + threadIdx.x;
    if (t < m) sum += (t == 0 || K[t] != K[t - 1]) ? 1u : 0u;
  }
  sum = __reduce_add_sync(SG_FULL_MASK, sum);
  if (lane_id() == 0) ss[warp_id()] = sum;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t b = 0;
    for (int w = 0; w < kSortWarps; ++w) b += ss[w];
    blk_max[blockIdx.x] = 0;
    blk_sum[blockIdx.x] = b;
  }
}

// dense[V[t]] = number of distinct tokens below K[t]: the order-preserving
// id of position V[t]'s token among the D distinct ones (0 .. D - 1).
template <int ITEMS>
__global__ void __launch_bounds__(kScanThreads)
    dense_write_kernel(const uint64_t* __restrict__ K,
                       const uint32_t* __restrict__ V, int64_t m,
                       const uint32_t* __restrict__ blk_sum,
                       uint32_t* __restrict__ dense) {
  __shared__ uint32_t ws[kSortWarps];
  const int lane = lane_id(), warp = warp_id();
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kScanThreads * ITEMS;
  uint32_t carry = blk_sum[blockIdx.x];
  for (int r = 0; r < ITEMS; ++r) {
    const int64_t t = base + r * kScanThreads + threadIdx.x;
    const bool head = t < m && (t == 0 || K[t] != K[t - 1]);
    const unsigned bal = __ballot_sync(SG_FULL_MASK, head);
    if (lane == 0) ws[warp] = __popc(bal);
    __syncthreads();
    uint32_t pre = carry, tot = carry;
    for (int w = 0; w < kSortWarps; ++w) {
      if (w < warp) pre += ws[w];
      tot += ws[w];
    }
    if (t < m) dense[V[t]] = pre + __popc(bal & ((2u << lane) - 1u)) - 1u;
    carry = tot;
    __syncthreads();
  }
}

// Dense token ids without sorting, when the tokens other than the PAD
// sentinel (int32 max) span a range [lo, hi] of at most 64 n values: a
// presence bitmap over the range, per-word prefix popcounts, and each
// token's id = the number of distinct values below it (PAD, the largest
// value, gets the top id). The same ids as the first-token sort gives,
// without its four digit passes over all n suffixes.
__global__ void range_init_kernel(int32_t* r) {
  r[0] = INT32_MAX;  // min of the non-PAD tokens
  r[1] = INT32_MIN;  // max of the non-PAD tokens
  r[2] = 0;          // a PAD token occurs
}

__global__ void __launch_bounds__(256)
    token_range_kernel(const int32_t* __restrict__ tok, int64_t n,
                       int32_t* __restrict__ r) {
  __shared__ int s_lo[8], s_hi[8];
  __shared__ unsigned s_pad[8];
  int lo = INT32_MAX, hi = INT32_MIN;
  unsigned pad = 0;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x +
                   threadIdx.x;
       i < n; i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int v = tok[i];
    if (v == INT32_MAX) {
      pad = 1;
    } else {
      lo = min(lo, v);
      hi = max(hi, v);
    }
  }
  lo = __reduce_min_sync(SG_FULL_MASK, lo);
  hi = __reduce_max_sync(SG_FULL_MASK, hi);
  pad = __reduce_or_sync(SG_FULL_MASK, pad);
  if (lane_id() == 0) {
    s_lo[warp_id()] = lo;
    s_hi[warp_id()] = hi;
    s_pad[warp_id()] = pad;
  }
  __syncthreads();
  if (threadIdx.x == 0) {  // one set of atomics per block
    for (int w = 1; w < 8; ++w) {
      lo = min(lo, s_lo[w]);
      hi = max(hi, s_hi[w]);
      pad |= s_pad[w];
    }
    if (lo != INT32_MAX) atomicMin(&r[0], lo);
    if (hi != INT32_MIN) atomicMax(&r[1], hi);
    if (pad) atomicOr(&r[2], 1);
  }
}

// Bits are set only when not yet set (frequent tokens would otherwise
// pile atomics onto a few words); a bitmap of at most kSmemWords words is
// built in the block's shared memory first and OR-ed out once.
constexpr int kSmemWords = 12288;  // 48 KB

__global__ void __launch_bounds__(256)
    bitmap_set_kernel(const int32_t* __restrict__ tok, int64_t n, int64_t lo,
                      int64_t nw, uint32_t* __restrict__ bm) {
  __shared__ uint32_t sbm[kSmemWords];
  const bool local = nw <= kSmemWords;
  if (local) {
    for (int k = threadIdx.x; k < nw; k += blockDim.x) sbm[k] = 0u;
    __syncthreads();
  }
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x +
                   threadIdx.x;
       i < n; i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int v = tok[i];
    if (v == INT32_MAX) continue;
    const uint64_t off = static_cast<uint64_t>(static_cast<int64_t>(v) - lo);
    const uint32_t bit = 1u << (off & 31);
    uint32_t* word = local ? &sbm[off >> 5] : &bm[off >> 5];
    if (!(*reinterpret_cast<volatile uint32_t*>(word) & bit))
      atomicOr(word, bit);
  }
  if (local) {
    __syncthreads();
    for (int k = threadIdx.x; k < nw; k += blockDim.x)
      if (sbm[k]) atomicOr(&bm[k], sbm[k]);
  }
}

constexpr int kWordsPerBlock = 4096;  // bitmap words per scan block

// Per block of kWordsPerBlock words: the number of set bits (blk_max is
// zeroed so that round_scan_blocks_kernel serves).
__global__ void __launch_bounds__(256)
    bitmap_count_kernel(const uint32_t* __restrict__ bm, int64_t W,
                        uint32_t* __restrict__ blk_max,
                        uint32_t* __restrict__ blk_sum) {
  __shared__ uint32_t ss[8];
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kWordsPerBlock;
  uint32_t c = 0;
  for (int k = threadIdx.x; k < kWordsPerBlock; k += 256) {
    const int64_t w = base + k;
    if (w < W) c += __popc(bm[w]);
  }
  c = __reduce_add_sync(SG_FULL_MASK, c);
  if (lane_id() == 0) ss[warp_id()] = c;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t t = 0;
    for (int w = 0; w < 8; ++w) t += ss[w];
    blk_max[blockIdx.x] = 0;
    blk_sum[blockIdx.x] = t;
  }
}

// pre[w] = set bits in the words before w (block offsets from blk_sum after
// round_scan_blocks_kernel); thread t scans 16 consecutive words.
__global__ void __launch_bounds__(256)
    bitmap_prefix_kernel(const uint32_t* __restrict__ bm, int64_t W,
                         const uint32_t* __restrict__ blk_sum,
                         uint32_t* __restrict__ pre) {
  __shared__ uint32_t ws[8];
  constexpr int kPer = kWordsPerBlock / 256;
  const int64_t w0 = static_cast<int64_t>(blockIdx.x) * kWordsPerBlock +
                     static_cast<int64_t>(threadIdx.x) * kPer;
  uint32_t c[kPer];
  uint32_t mine = 0;
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    c[k] = w0 + k < W ? __popc(bm[w0 + k]) : 0u;
    mine += c[k];
  }
  const uint32_t inc =
      static_cast<uint32_t>(warp_incl_scan(static_cast<int>(mine)));
  if (lane_id() == 31) ws[warp_id()] = inc;
  __syncthreads();
  uint32_t run = blk_sum[blockIdx.x] + inc - mine;
  for (int w = 0; w < warp_id(); ++w) run += ws[w];
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    if (w0 + k < W) pre[w0 + k] = run;
    run += c[k];
  }
}

__global__ void __launch_bounds__(256)
    bitmap_dense_kernel(const int32_t* __restrict__ tok, int64_t n,
                        int64_t lo, const uint32_t* __restrict__ bm,
                        const uint32_t* __restrict__ pre,
                        const int64_t* __restrict__ n_values,
                        uint32_t* __restrict__ dense) {
  const uint32_t pad_id = static_cast<uint32_t>(*n_values);
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x +
                   threadIdx.x;
       i < n; i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int v = tok[i];
    uint32_t id = pad_id;
    if (v != INT32_MAX) {
      const uint64_t off =
          static_cast<uint64_t>(static_cast<int64_t>(v) - lo);
      const uint64_t w = off >> 5;
      id = pre[w] + __popc(bm[w] & ((1u << (off & 31)) - 1u));
    }
    dense[i] = id;
  }
}

// Keys of the two-token pass: (dense[i] << B) | (dense[i+1] + 1, or 0 at
// the end of the string), value i.
__global__ void make2_keys_kernel(const uint32_t* __restrict__ dense,
                                  int64_t n, int B,
                                  uint64_t* __restrict__ keys,
                                  uint32_t* __restrict__ vals) {
  const int64_t i =
      static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint64_t second = i + 1 < n ? static_cast<uint64_t>(dense[i + 1]) + 1 : 0;
  keys[i] = (static_cast<uint64_t>(dense[i]) << B) | second;
  vals[i] = static_cast<uint32_t>(i);
}

// Element t of the sorted active list: head of a new group? still tied?
__device__ __forceinline__ void round_flags(const uint64_t* K, int64_t m,
                                            int64_t t, bool& head,
                                            bool& keep) {
  const uint64_t k = K[t];
  head = (t == 0) || K[t - 1] != k;
  const bool next_head = (t == m - 1) || K[t + 1] != k;
  keep = !(head && next_head);
}

// Per scan block: max of the new group starts and count of elements that
// stay active.
template <int ITEMS>
__global__ void __launch_bounds__(kScanThreads)
    round_reduce_kernel(const uint64_t* __restrict__ K,
                        const uint32_t* __restrict__ act, int64_t m,
                        uint32_t* __restrict__ blk_max,
                        uint32_t* __restrict__ blk_sum) {
  __shared__ uint32_t sm[kSortWarps], ss[kSortWarps];
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kScanThreads * ITEMS;
  uint32_t mx = 0, sum = 0;
  for (int r = 0; r < ITEMS; ++r) {
    const int64_t t = base + r * kScanThreads + threadIdx.x;
    if (t < m) {
      bool head, keep;
      round_flags(K, m, t, head, keep);
      const uint32_t a = act ? act[t] : static_cast<uint32_t>(t);
      if (head) mx = max(mx, a);
      sum += keep;
    }
  }
  mx = __reduce_max_sync(SG_FULL_MASK, mx);
  sum = __reduce_add_sync(SG_FULL_MASK, sum);
  if (lane_id() == 0) {
    sm[warp_id()] = mx;
    ss[warp_id()] = sum;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t a = 0, b = 0;
    for (int w = 0; w < kSortWarps; ++w) {
      a = max(a, sm[w]);
      b += ss[w];
    }
    blk_max[blockIdx.x] = a;
    blk_sum[blockIdx.x] = b;
  }
}

// Exclusive max-scan and sum-scan of the block aggregates (one block of
// 1024 threads); writes the next active count.
__global__ void __launch_bounds__(1024)
    round_scan_blocks_kernel(uint32_t* blk_max, uint32_t* blk_sum, int nblk,
                             int64_t* next_m) {
  __shared__ uint32_t wm[32], ws[32];
  __shared__ uint32_t carry_m, carry_s;
  const int lane = lane_id(), warp = warp_id();
  if (threadIdx.x == 0) {
    carry_m = 0;
    carry_s = 0;
  }
  __syncthreads();
  for (int c0 = 0; c0 < nblk; c0 += 1024) {
    const int i = c0 + threadIdx.x;
    const uint32_t xm = i < nblk ? blk_max[i] : 0u;
    const uint32_t xs = i < nblk ? blk_sum[i] : 0u;
    uint32_t im = xm, is = xs;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t a = __shfl_up_sync(SG_FULL_MASK, im, o);
      const uint32_t b = __shfl_up_sync(SG_FULL_MASK, is, o);
      if (lane >= o) {
        im = max(im, a);
        is += b;
      }
    }
    uint32_t em = __shfl_up_sync(SG_FULL_MASK, im, 1);
    if (lane == 0) em = 0;
    const uint32_t es = is - xs;
    if (lane == 31) {
      wm[warp] = im;
      ws[warp] = is;
    }
    __syncthreads();
    uint32_t pm = carry_m, ps = carry_s;
    for (int w = 0; w < warp; ++w) {
      pm = max(pm, wm[w]);
      ps += ws[w];
    }
    if (i < nblk) {
      blk_max[i] = max(pm, em);
      blk_sum[i] = ps + es;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      uint32_t a = carry_m, b = carry_s;
      for (int w = 0; w < 32; ++w) {
        a = max(a, wm[w]);
        b += ws[w];
      }
      carry_m = a;
      carry_s = b;
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) *next_m = carry_s;
}

// Writes sa[act[t]] = V[t], rank[V[t]] = start of t's group (the act value
// of its group's first element: act is increasing, so a max-scan over
// head-marked act values finds it) and compacts the still-tied elements
// into act_next, all in element order.
template <int ITEMS>
__global__ void __launch_bounds__(kScanThreads)
    round_apply_kernel(const uint64_t* __restrict__ K,
                       const uint32_t* __restrict__ V,
                       const uint32_t* __restrict__ act, int64_t m,
                       const uint32_t* __restrict__ blk_max,
                       const uint32_t* __restrict__ blk_sum,
                       int32_t* __restrict__ sa, uint32_t* __restrict__ rank,
                       uint32_t* __restrict__ act_next) {
  __shared__ uint32_t wm[kSortWarps], ws[kSortWarps];
  const int lane = lane_id(), warp = warp_id();
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kScanThreads * ITEMS;
  uint32_t carry_m = blk_max[blockIdx.x];
  uint32_t carry_s = blk_sum[blockIdx.x];
  for (int r = 0; r < ITEMS; ++r) {
    const int64_t t = base + r * kScanThreads + threadIdx.x;
    bool head = false, keep = false;
    uint32_t a = 0;
    if (t < m) {
      round_flags(K, m, t, head, keep);
      a = act ? act[t] : static_cast<uint32_t>(t);
    }
    uint32_t im = head ? a : 0u, is = keep ? 1u : 0u;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t x = __shfl_up_sync(SG_FULL_MASK, im, o);
      const uint32_t y = __shfl_up_sync(SG_FULL_MASK, is, o);
      if (lane >= o) {
        im = max(im, x);
        is += y;
      }
    }
    if (lane == 31) {
      wm[warp] = im;
      ws[warp] = is;
    }
    __syncthreads();
    uint32_t pm = carry_m, ps = carry_s, tm = carry_m, ts = carry_s;
#pragma unroll
    for (int w = 0; w < kSortWarps; ++w) {
      if (w < warp) {
        pm = max(pm, wm[w]);
        ps += ws[w];
      }
      tm = max(tm, wm[w]);
      ts += ws[w];
    }
    if (t < m) {
      const uint32_t v = V[t];
      sa[a] = static_cast<int32_t>(v);
      rank[v] = max(pm, im);
      if (keep) act_next[ps + is - 1] = a;
    }
    carry_m = tm;
    carry_s = ts;
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// segmented rounds
// ---------------------------------------------------------------------------
constexpr int kSegThreads = 256;
constexpr int kSegTile = 2048;   // active-list elements owned by a block
constexpr int kSegHalo = 256;    // largest group ranked on chip
constexpr int kSegItems = 11;    // window elements per thread
constexpr int kSegWin = kSegTile + 2 * kSegHalo + 2;  // (+ one each side)
constexpr int kSegWinPad = (kSegWin + 3) & ~3;       // 16-byte rows
constexpr size_t kSegSmem = sizeof(uint64_t) * kSegWin + 8 * kSegWinPad;
static_assert(kSegThreads * kSegItems >= kSegWin, "window does not fit");

// Exclusive prefix max / suffix min over the threads of a block (one value
// per thread): warp scans with shuffles, then the warps' totals.
__device__ __forceinline__ int block_excl_prefix_max(int v, int* buf) {
  const int lane = lane_id(), warp = warp_id();
  int inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int x = __shfl_up_sync(SG_FULL_MASK, inc, o);
    if (lane >= o) inc = max(inc, x);
  }
  if (lane == 31) buf[warp] = inc;
  __syncthreads();
  int carry = INT32_MIN;
  for (int w = 0; w < warp; ++w) carry = max(carry, buf[w]);
  int ex = __shfl_up_sync(SG_FULL_MASK, inc, 1);
  if (lane == 0) ex = INT32_MIN;
  __syncthreads();  // buf is reused by the next scan
  return max(carry, ex);
}

__device__ __forceinline__ int block_excl_suffix_min(int v, int* buf) {
  const int lane = lane_id(), warp = warp_id();
  constexpr int kWarps = kSegThreads / 32;
  int inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int x = __shfl_down_sync(SG_FULL_MASK, inc, o);
    if (lane + o < 32) inc = min(inc, x);
  }
  if (lane == 0) buf[warp] = inc;
  __syncthreads();
  int carry = INT32_MAX;
  for (int w = warp + 1; w < kWarps; ++w) carry = min(carry, buf[w]);
  int ex = __shfl_down_sync(SG_FULL_MASK, inc, 1);
  if (lane == 31) ex = INT32_MAX;
  __syncthreads();
  return min(carry, ex);
}

// Element w of the window is element x = t0 - kSegHalo - 1 + w of the
// active list (sentinel groups outside the list). A block owns x in
// [t0, t0 + kSegTile): it flags each owned element that belongs to a large
// group (for the global path) and writes every element of the small groups
// whose head it owns, in (second key, list position) order, at the group's
// slots. A small group's members all lie within kSegHalo of its head, so
// the window holds every group that the block must see whole.
__global__ void __launch_bounds__(kSegThreads)
    seg_local_kernel(const uint64_t* __restrict__ K,
                     const uint32_t* __restrict__ V, int64_t m, int sb,
                     uint64_t* __restrict__ Kout, uint32_t* __restrict__ Vout,
                     uint8_t* __restrict__ large) {
  extern __shared__ __align__(16) unsigned char seg_smem[];
  uint64_t* sk = reinterpret_cast<uint64_t*>(seg_smem);   // [kSegWin]
  int* first = reinterpret_cast<int*>(sk + kSegWin);      // [kSegWinPad]
  int* last = first + kSegWinPad;                         // [kSegWinPad]
  __shared__ int sbuf[kSegThreads];
  const int t = threadIdx.x;
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * kSegTile;
  const int64_t wbase = t0 - kSegHalo - 1;
  const uint64_t kmask = (uint64_t(1) << sb) - 1;
  // group ids of real keys are < 2^31 <= 2^(63 - sb); the two sentinels
  // (before / after the list) have distinct larger ids
  const uint64_t before_key = uint64_t(1) << 63;
  const uint64_t after_key = (uint64_t(3) << 62);
  for (int w = t; w < kSegWin; w += kSegThreads) {
    const int64_t x = wbase + w;
    sk[w] = (x >= 0 && x < m) ? K[x] : (x < 0 ? before_key : after_key);
  }
  __syncthreads();
  // first[w]: head of w's group (<= 0: at or before the window start);
  // last[w]: its last element (>= kSegWin - 1: at or after the window end)
  const int w0 = t * kSegItems;
  int run = INT32_MIN;
#pragma unroll
  for (int q = 0; q < kSegItems; ++q) {
    const int w = w0 + q;
    if (w < kSegWin) {
      if (w > 0 && (sk[w] >> sb) != (sk[w - 1] >> sb)) run = w;
      first[w] = run;
    }
  }
  const int pre = block_excl_prefix_max(run, sbuf);
#pragma unroll
  for (int q = 0; q < kSegItems; ++q) {
    const int w = w0 + q;
    if (w < kSegWin) {
      const int f = max(first[w], pre);
      first[w] = f < 0 ? 0 : f;
    }
  }
  int rrun = INT32_MAX;
#pragma unroll
  for (int q = kSegItems - 1; q >= 0; --q) {
    const int w = w0 + q;
    if (w < kSegWin) {
      if (w < kSegWin - 1 && (sk[w] >> sb) != (sk[w + 1] >> sb)) rrun = w;
      last[w] = rrun;
    }
  }
  const int suf = block_excl_suffix_min(rrun, sbuf);
  // final bounds packed as first | last << 16 (both < kSegWin < 2^16);
  // `last` then holds the 32-bit second keys (below 2^sb <= 2^31) that the
  // ranking loop reads four at a time
#pragma unroll
  for (int q = 0; q < kSegItems; ++q) {
    const int w = w0 + q;
    if (w < kSegWin) {
      const int l = min(last[w], suf);
      first[w] |= (l > kSegWin - 1 ? kSegWin - 1 : l) << 16;
      last[w] = static_cast<int>(static_cast<uint32_t>(sk[w] & kmask));
    }
  }
  __syncthreads();
  const uint32_t* k32 = reinterpret_cast<const uint32_t*>(last);
  // owned elements and the forward halo
  const int own0 = kSegHalo + 1, own1 = own0 + kSegTile;
  for (int w = own0 + t; w < kSegWin - 1; w += kSegThreads) {
    const int64_t x = wbase + w;
    if (x >= m) break;
    const int fl = first[w];
    const int f = fl & 0xffff, l = fl >> 16;
    const bool small = f > 0 && l < kSegWin - 1 && l - f + 1 <= kSegHalo;
    if (w < own1) large[x] = small ? 0 : 1;
    if (!small || f < own0 || f >= own1) continue;  // another block's group
    // rank in the group by (second key, list position)
    const uint32_t kw = k32[w];
    int rank = 0;
    int u = f;
    for (; u <= l && (u & 3); ++u) {
      const uint32_t ku = k32[u];
      rank += (ku < kw) || (ku == kw && u < w);
    }
    for (; u + 3 <= l; u += 4) {
      const uint4 q4 = *reinterpret_cast<const uint4*>(k32 + u);
      rank += (q4.x < kw) || (q4.x == kw && u < w);
      rank += (q4.y < kw) || (q4.y == kw && u + 1 < w);
      rank += (q4.z < kw) || (q4.z == kw && u + 2 < w);
      rank += (q4.w < kw) || (q4.w == kw && u + 3 < w);
    }
    for (; u <= l; ++u) {
      const uint32_t ku = k32[u];
      rank += (ku < kw) || (ku == kw && u < w);
    }
    const int64_t pos = wbase + f + rank;
    Kout[pos] = sk[w];
    Vout[pos] = V[x];
  }
}

// Per scan block: number of flagged elements (blk_max zeroed so that the
// shared scan kernel can be reused).
template <int ITEMS>
__global__ void __launch_bounds__(kScanThreads)
    flag_count_kernel(const uint8_t* __restrict__ flag, int64_t m,
                      uint32_t* __restrict__ blk_max,
                      uint32_t* __restrict__ blk_sum) {
  __shared__ uint32_t ss[kSortWarps];
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kScanThreads * ITEMS;
  uint32_t sum = 0;
  for (int r = 0; r < ITEMS; ++r) {
    const int64_t t = base + r * kScanThreads + threadIdx.x;
    if (t < m) sum += flag[t];
  }
  sum = __reduce_add_sync(SG_FULL_MASK, sum);
  if (lane_id() == 0) ss[warp_id()] = sum;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t b = 0;
    for (int w = 0; w < kSortWarps; ++w) b += ss[w];
    blk_max[blockIdx.x] = 0;
    blk_sum[blockIdx.x] = b;
  }
}

// Flagged elements in order: LK[u] = K[t], LV[u] = V[t], LT[u] = t.
template <int ITEMS>
__global__ void __launch_bounds__(kScanThreads)
    flag_compact_kernel(const uint8_t* __restrict__ flag,
                        const uint64_t* __restrict__ K,
                        const uint32_t* __restrict__ V, int64_t m,
                        const uint32_t* __restrict__ blk_sum,
                        uint64_t* __restrict__ LK, uint32_t* __restrict__ LV,
                        uint32_t* __restrict__ LT) {
  __shared__ uint32_t ws[kSortWarps];
  const int lane = lane_id(), warp = warp_id();
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kScanThreads * ITEMS;
  uint32_t carry = blk_sum[blockIdx.x];
  for (int r = 0; r < ITEMS; ++r) {
    const int64_t t = base + r * kScanThreads + threadIdx.x;
    const bool f = t < m && flag[t];
    const unsigned bal = __ballot_sync(SG_FULL_MASK, f);
    if (lane == 0) ws[warp] = __popc(bal);
    __syncthreads();
    uint32_t pre = carry, tot = carry;
    for (int w = 0; w < kSortWarps; ++w) {
      if (w < warp) pre += ws[w];
      tot += ws[w];
    }
    if (f) {
      const uint32_t u = pre + __popc(bal & ((1u << lane) - 1u));
      LK[u] = K[t];
      LV[u] = V[t];
      LT[u] = static_cast<uint32_t>(t);
    }
    carry = tot;
    __syncthreads();
  }
}

// Sorted large-group elements back to their slots.
__global__ void flag_scatter_kernel(const uint64_t* __restrict__ SK,
                                    const uint32_t* __restrict__ SV,
                                    const uint32_t* __restrict__ LT,
                                    int64_t ml, uint64_t* __restrict__ Kout,
                                    uint32_t* __restrict__ Vout) {
  const int64_t u = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (u < ml) {
    const uint32_t pos = LT[u];
    Kout[pos] = SK[u];
    Vout[pos] = SV[u];
  }
}

// ---------------------------------------------------------------------------
// host driver
// ---------------------------------------------------------------------------
static int bitlen(uint64_t x) {
  int b = 0;
  while (x) {
    ++b;
    x >>= 1;
  }
  return b;
}

struct SaWorkspace {
  uint64_t* K[2];
  uint32_t* V[2];
  uint32_t* rank;
  uint32_t* act[2];
  uint64_t* LK;      // large-group elements: keys, values, list positions
  uint32_t* LV;
  uint32_t* LT;
  uint8_t* flag;     // element of a large group
  uint32_t* tile_hist;
  uint32_t* totals;
  uint32_t* blk_max;
  uint32_t* blk_sum;
  int64_t* m_dev;
  size_t bytes;
};

static size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

static SaWorkspace carve(void* base, int64_t n) {
  SaWorkspace w{};
  const size_t un = static_cast<size_t>(n > 0 ? n : 1);
  // per-tile / per-block arrays sized for the small tiles
  const size_t small = static_cast<size_t>(kSortThreads) * kItemsSmall;
  const size_t ntiles = (un + small - 1) / small;
  const size_t nblk = (un + small - 1) / small;
  char* p = static_cast<char*>(base);
  size_t o = 0;
  auto take = [&](size_t bytes) {
    char* r = p ? p + o : nullptr;
    o = align256(o + bytes);
    return r;
  };
  w.K[0] = reinterpret_cast<uint64_t*>(take(8 * un));
  w.K[1] = reinterpret_cast<uint64_t*>(take(8 * un));
  w.V[0] = reinterpret_cast<uint32_t*>(take(4 * un));
  w.V[1] = reinterpret_cast<uint32_t*>(take(4 * un));
  w.rank = reinterpret_cast<uint32_t*>(take(4 * un));
  w.act[0] = reinterpret_cast<uint32_t*>(take(4 * un));
  w.act[1] = reinterpret_cast<uint32_t*>(take(4 * un));
  w.LK = reinterpret_cast<uint64_t*>(take(8 * un));
  w.LV = reinterpret_cast<uint32_t*>(take(4 * un));
  w.LT = reinterpret_cast<uint32_t*>(take(4 * un));
  w.flag = reinterpret_cast<uint8_t*>(take(un));
  w.tile_hist = reinterpret_cast<uint32_t*>(take(4 * 256 * ntiles));
  w.totals = reinterpret_cast<uint32_t*>(take(4 * 256));
  w.blk_max = reinterpret_cast<uint32_t*>(take(4 * nblk));
  w.blk_sum = reinterpret_cast<uint32_t*>(take(4 * nblk));
  w.m_dev = reinterpret_cast<int64_t*>(take(8));
  w.bytes = o;
  return w;
}

// Whether a list of m elements takes the small tiles.
static bool small_tiles(int64_t m) {
  return (m + kTile - 1) / kTile < 2 * static_cast<int64_t>(num_sms());
}

static int elems_per_block(int64_t m) {
  return kSortThreads * (small_tiles(m) ? kItemsSmall : kSortItems);
}

template <int ITEMS>
static void radix_pass(SaWorkspace& w, const uint64_t* kin,
                       const uint32_t* vin, uint64_t* kout, uint32_t* vout,
                       int64_t m, int shift, cudaStream_t st) {
  const int ntiles = static_cast<int>(
      (m + kSortThreads * ITEMS - 1) / (kSortThreads * ITEMS));
  zero_u32_kernel<<<1, 256, 0, st>>>(w.totals, 256);
  rs_hist_kernel<ITEMS><<<ntiles, kSortThreads, 0, st>>>(
      kin, m, shift, w.tile_hist, ntiles, w.totals);
  rs_scan_kernel<<<256, kSortThreads, 0, st>>>(w.tile_hist, ntiles,
                                               w.totals);
  rs_scatter_kernel<ITEMS><<<ntiles, kSortThreads, 0, st>>>(
      kin, vin, kout, vout, m, shift, w.tile_hist, ntiles);
}

// Stable LSD sort of (kb[cur], vb[cur]) by the low `bits` bits, ping-
// ponging between the two buffer pairs; returns the index holding the
// result.
static int radix_sort_pair(SaWorkspace& w, uint64_t* const kb[2],
                           uint32_t* const vb[2], int cur, int64_t m,
                           int bits, cudaStream_t st) {
  const bool small = small_tiles(m);
  for (int shift = 0; shift < bits; shift += 8) {
    if (small)
      radix_pass<kItemsSmall>(w, kb[cur], vb[cur], kb[1 - cur], vb[1 - cur],
                              m, shift, st);
    else
      radix_pass<kSortItems>(w, kb[cur], vb[cur], kb[1 - cur], vb[1 - cur],
                             m, shift, st);
    cur = 1 - cur;
  }
  return cur;
}

static int radix_sort(SaWorkspace& w, int cur, int64_t m, int bits,
                      cudaStream_t st) {
  return radix_sort_pair(w, w.K, w.V, cur, m, bits, st);
}

// Host landing slots for the counts a build reads back each round. A
// device-to-host copy into pageable memory is staged by the driver and
// keeps the calling thread inside the runtime until the stream has drained;
// the drafter launches its decode step from another thread while a
// background rebuild waits here, so the counts land in page-locked memory
// instead: a pool of slots allocated once per process, one slot per build
// in flight (a build that finds the pool empty uses its stack).
constexpr int kCountSlots = 64;
static std::mutex g_count_mu;
static int64_t* g_count_pool = nullptr;
static bool g_count_pool_failed = false;
static uint64_t g_count_used = 0;  // bit i: slot i taken

class CountSlot {
 public:
  // use_pool false: the reads land in the slot's own stack array (the
  // allocation-free build may not make the pool's one host allocation)
  explicit CountSlot(bool use_pool = true) {
    if (!use_pool) return;
    std::lock_guard<std::mutex> lk(g_count_mu);
    if (!g_count_pool && !g_count_pool_failed) {
      void* p = nullptr;
      if (cudaHostAlloc(&p, kCountSlots * 64, cudaHostAllocDefault) ==
          cudaSuccess) {
        g_count_pool = static_cast<int64_t*>(p);
      } else {
        cudaGetLastError();
        g_count_pool_failed = true;
      }
    }
    if (!g_count_pool) return;
    for (int i = 0; i < kCountSlots; ++i) {
      if (!(g_count_used >> i & 1)) {
        g_count_used |= uint64_t(1) << i;
        idx_ = i;
        ptr_ = g_count_pool + i * 8;  // one 64-byte line per slot
        return;
      }
    }
  }
  ~CountSlot() {
    if (idx_ < 0) return;
    std::lock_guard<std::mutex> lk(g_count_mu);
    g_count_used &= ~(uint64_t(1) << idx_);
  }
  CountSlot(const CountSlot&) = delete;
  CountSlot& operator=(const CountSlot&) = delete;
  int64_t* get() { return ptr_ ? ptr_ : fallback_; }  // 64 bytes

 private:
  int idx_ = -1;
  int64_t* ptr_ = nullptr;
  int64_t fallback_[8] = {};
};

// Reads `bytes` (<= 64, one slot) of device memory into *out (host sync),
// through the build's slot.
static int read_small(const void* dev, void* out, size_t bytes,
                      CountSlot& slot, cudaStream_t st) {
  if (bytes > 64) return SG_ERR_INVALID;
  int64_t* land = slot.get();
  cudaError_t e = cudaMemcpyAsync(land, dev, bytes, cudaMemcpyDeviceToHost,
                                  st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return SG_ERR_CUDA;
  }
  std::memcpy(out, land, bytes);
  return SG_OK;
}

// Reads a device count into *out (host sync), through the build's slot.
static int read_count(const int64_t* dev, int64_t* out, CountSlot& slot,
                      cudaStream_t st) {
  return read_small(dev, out, sizeof(int64_t), slot, st);
}

// One read through a slot of its own, for callers outside a build loop.
int read_device_i64(const int64_t* dev, int64_t* out, cudaStream_t st) {
  CountSlot slot;
  return read_count(dev, out, slot, st);
}

// Dense ids of the first-token sort (K[kcur], V[kcur]; n elements) into
// w.rank; returns the number D of distinct tokens through *d (host sync).
static int dense_ids(SaWorkspace& w, int kcur, int64_t n, CountSlot& slot,
                     cudaStream_t st, int64_t* d) {
  const bool small = small_tiles(n);
  const int nblk = static_cast<int>((n + elems_per_block(n) - 1) /
                                    elems_per_block(n));
  if (small)
    dense_count_kernel<kItemsSmall><<<nblk, kScanThreads, 0, st>>>(
        w.K[kcur], n, w.blk_max, w.blk_sum);
  else
    dense_count_kernel<kScanItems><<<nblk, kScanThreads, 0, st>>>(
        w.K[kcur], n, w.blk_max, w.blk_sum);
  round_scan_blocks_kernel<<<1, 1024, 0, st>>>(w.blk_max, w.blk_sum, nblk,
                                               w.m_dev);
  if (small)
    dense_write_kernel<kItemsSmall><<<nblk, kScanThreads, 0, st>>>(
        w.K[kcur], w.V[kcur], n, w.blk_sum, w.rank);
  else
    dense_write_kernel<kScanItems><<<nblk, kScanThreads, 0, st>>>(
        w.K[kcur], w.V[kcur], n, w.blk_sum, w.rank);
  return read_count(w.m_dev, d, slot, st);
}

// Orders the active list (K[0], V[0]; m elements, grouped) by
// (group, second key) into (K[1], V[1]): small groups on chip, large ones
// through the global radix sort.
static int segmented_sort(SaWorkspace& w, int64_t m, int sb, int bits,
                          CountSlot& slot, cudaStream_t st) {
  const int nseg = static_cast<int>((m + kSegTile - 1) / kSegTile);
  seg_local_kernel<<<nseg, kSegThreads, kSegSmem, st>>>(
      w.K[0], w.V[0], m, sb, w.K[1], w.V[1], w.flag);
  const bool small = small_tiles(m);
  const int nblk = static_cast<int>((m + elems_per_block(m) - 1) /
                                    elems_per_block(m));
  if (small)
    flag_count_kernel<kItemsSmall><<<nblk, kScanThreads, 0, st>>>(
        w.flag, m, w.blk_max, w.blk_sum);
  else
    flag_count_kernel<kScanItems><<<nblk, kScanThreads, 0, st>>>(
        w.flag, m, w.blk_max, w.blk_sum);
  round_scan_blocks_kernel<<<1, 1024, 0, st>>>(w.blk_max, w.blk_sum, nblk,
                                               w.m_dev);
  int64_t ml = 0;
  const int rc = read_count(w.m_dev, &ml, slot, st);
  if (rc != SG_OK) return rc;
  if (ml == 0) return SG_OK;
  if (small)
    flag_compact_kernel<kItemsSmall><<<nblk, kScanThreads, 0, st>>>(
        w.flag, w.K[0], w.V[0], m, w.blk_sum, w.LK, w.LV, w.LT);
  else
    flag_compact_kernel<kScanItems><<<nblk, kScanThreads, 0, st>>>(
        w.flag, w.K[0], w.V[0], m, w.blk_sum, w.LK, w.LV, w.LT);
  uint64_t* const kb[2] = {w.LK, w.K[0]};
  uint32_t* const vb[2] = {w.LV, w.V[0]};
  const int c = radix_sort_pair(w, kb, vb, 0, ml, bits, st);
  flag_scatter_kernel<<<static_cast<unsigned>((ml + 255) / 256), 256, 0,
                        st>>>(kb[c], vb[c], w.LT, ml, w.K[1], w.V[1]);
  return SG_OK;
}

// One apply pass; returns the next active count (host sync).
static int apply_round(SaWorkspace& w, int kcur, const uint32_t* act,
                       uint32_t* act_next, int64_t m, int32_t* sa,
                       CountSlot& slot, cudaStream_t st, int64_t* next_m,
                       int* err) {
  const bool small = small_tiles(m);
  const int nblk = static_cast<int>((m + elems_per_block(m) - 1) /
                                    elems_per_block(m));
  if (small)
    round_reduce_kernel<kItemsSmall><<<nblk, kScanThreads, 0, st>>>(
        w.K[kcur], act, m, w.blk_max, w.blk_sum);
  else
    round_reduce_kernel<kScanItems><<<nblk, kScanThreads, 0, st>>>(
        w.K[kcur], act, m, w.blk_max, w.blk_sum);
  round_scan_blocks_kernel<<<1, 1024, 0, st>>>(w.blk_max, w.blk_sum, nblk,
                                               w.m_dev);
  if (small)
    round_apply_kernel<kItemsSmall><<<nblk, kScanThreads, 0, st>>>(
        w.K[kcur], w.V[kcur], act, m, w.blk_max, w.blk_sum, sa, w.rank,
        act_next);
  else
    round_apply_kernel<kScanItems><<<nblk, kScanThreads, 0, st>>>(
        w.K[kcur], w.V[kcur], act, m, w.blk_max, w.blk_sum, sa, w.rank,
        act_next);
  const int rc = read_count(w.m_dev, next_m, slot, st);
  if (rc != SG_OK) {
    *err = rc;
    return 0;
  }
  return 1;
}

}  // namespace sg

using namespace sg;

extern "C" size_t sg_suffix_array_workspace_size(int64_t n) {
  if (n < 0) return 0;
  return carve(nullptr, n).bytes;
}

namespace sg {

// The build behind both entry points; host_pool false keeps the per-round
// count read-backs out of the page-locked slot pool (no host allocation).
static int build_suffix_array(const int32_t* tokens, int64_t n,
                              int32_t* sa_out, void* workspace,
                              size_t ws_bytes, int32_t* rounds_out,
                              sg_stream_t stream, bool host_pool) {
  sg::NvtxScope nvtx_range("sg_build_suffix_array");
  if (n < 0) return SG_ERR_INVALID;
  if (n >= (int64_t(1) << 31) - 1) return SG_ERR_UNSUPPORTED;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (rounds_out) *rounds_out = 0;
  if (n == 0) return SG_OK;
  if (!tokens || !sa_out) return SG_ERR_INVALID;
  if (n == 1) {
    cudaError_t e = cudaMemsetAsync(sa_out, 0, sizeof(int32_t), st);
    if (e != cudaSuccess) {
      set_cuda_error(e);
      return SG_ERR_CUDA;
    }
    return SG_OK;
  }
  if (!workspace || ws_bytes < carve(nullptr, n).bytes)
    return SG_ERR_WORKSPACE;
  SaWorkspace w = carve(workspace, n);
  CountSlot slot(host_pool);

  int kcur = 0;
  int err = SG_OK;
  int64_t m = 0;
  int acur = 0;
  int rounds = 0;
  // Dense token ids (w.rank): from a bitmap when the tokens' range allows
  // it, else from a sort by the first token.
  int64_t n_distinct = 0;
  bool dense_done = false;
  {
    int32_t* r = reinterpret_cast<int32_t*>(w.tile_hist);
    const unsigned grid = static_cast<unsigned>(
        std::min<int64_t>((n + 255) / 256, 8 * static_cast<int64_t>(num_sms())));
    range_init_kernel<<<1, 1, 0, st>>>(r);
    token_range_kernel<<<grid, 256, 0, st>>>(tokens, n, r);
    int32_t rng[3] = {0, 0, 0};  // min, max of the non-PAD tokens, PAD seen
    int rc = read_small(r, rng, sizeof(rng), slot, st);
    if (rc != SG_OK) return rc;
    const int64_t lo = rng[0], hi = rng[1];
    const bool pad = rng[2] != 0;
    const int64_t range = hi >= lo ? hi - lo + 1 : 0;
    if (range <= 64 * n && range < (int64_t(1) << 31) - 2) {
      uint32_t* bm = reinterpret_cast<uint32_t*>(w.LK);     // <= 8n bytes
      uint32_t* pre = reinterpret_cast<uint32_t*>(w.K[1]);  // <= 8n bytes
      const int64_t nw = (range + 31) / 32;
      cudaError_t e = cudaSuccess;
      if (nw > 0) {
        e = cudaMemsetAsync(bm, 0, static_cast<size_t>(nw) * 4, st);
        // few blocks when each ORs a whole shared bitmap out at its end
        const unsigned gset =
            nw <= kSmemWords
                ? std::min<unsigned>(grid, 2u * static_cast<unsigned>(num_sms()))
                : grid;
        bitmap_set_kernel<<<gset, 256, 0, st>>>(tokens, n, lo, nw, bm);
        const int nb = static_cast<int>((nw + kWordsPerBlock - 1) /
                                        kWordsPerBlock);
        bitmap_count_kernel<<<nb, 256, 0, st>>>(bm, nw, w.blk_max, w.blk_sum);
        round_scan_blocks_kernel<<<1, 1024, 0, st>>>(w.blk_max, w.blk_sum,
                                                     nb, w.m_dev);
        bitmap_prefix_kernel<<<nb, 256, 0, st>>>(bm, nw, w.blk_sum, pre);
      } else {
        e = cudaMemsetAsync(w.m_dev, 0, sizeof(int64_t), st);
      }
      if (e != cudaSuccess) {
        set_cuda_error(e);
        return SG_ERR_CUDA;
      }
      bitmap_dense_kernel<<<grid, 256, 0, st>>>(tokens, n, lo, bm, pre,
                                                w.m_dev, w.rank);
      int64_t values = 0;
      rc = read_count(w.m_dev, &values, slot, st);
      if (rc != SG_OK) return rc;
      n_distinct = values + (pad ? 1 : 0);
      dense_done = true;
    }
  }
  if (!dense_done) {
    // initial pass: sort by the first token
    init_keys_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0,
                       st>>>(tokens, n, w.K[0], w.V[0]);
    kcur = radix_sort(w, 0, n, 32, st);
  }
  // Two-token pass in place of the first doubling round: with the D
  // distinct tokens renumbered 0 .. D - 1 in order, a suffix's first two
  // tokens pack into 2 * bitlen(D) <= 62 bits, and one sort of all n
  // suffixes by them leaves the same groups and ranks as that round (whose
  // active list, on copy-heavy text, is most of the corpus) at the price of
  // ceil(2 * bitlen(D) / 8) digit passes.
  if (!dense_done) {
    const int rc0 = dense_ids(w, kcur, n, slot, st, &n_distinct);
    if (rc0 != SG_OK) return rc0;
  }
  if (n_distinct == n && !dense_done) {
    // every first token differs: sorted already, no common prefixes
    if (!apply_round(w, kcur, nullptr, w.act[acur], n, sa_out, slot, st, &m,
                     &err))
      return err;
  } else {
    const int B = bitlen(static_cast<uint64_t>(n_distinct));  // ids + 1 <= D
    make2_keys_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0,
                        st>>>(w.rank, n, B, w.K[0], w.V[0]);
    kcur = radix_sort(w, 0, n, 2 * B, st);
    if (!apply_round(w, kcur, nullptr, w.act[acur], n, sa_out, slot, st, &m,
                     &err))
      return err;
    // every first token distinct: no common prefixes, no doubling round
    rounds = n_distinct == n ? 0 : 1;
  }
  const int sb = bitlen(static_cast<uint64_t>(n));        // rank[i+h]+1 <= n
  const int pb = bitlen(static_cast<uint64_t>(n - 1));    // group start < n
  for (int64_t h = 2; m > 0; h <<= 1) {
    if (h >= n) return SG_ERR_CUDA;  // cannot happen for a correct build
    make_keys_kernel<<<static_cast<unsigned>((m + 255) / 256), 256, 0, st>>>(
        w.act[acur], sa_out, w.rank, n, m, h, sb, w.K[0], w.V[0]);
    const int rc = segmented_sort(w, m, sb, pb + sb, slot, st);
    if (rc != SG_OK) return rc;
    kcur = 1;
    int64_t m_next = 0;
    if (!apply_round(w, kcur, w.act[acur], w.act[1 - acur], m, sa_out, slot,
                     st, &m_next, &err))
      return err;
    acur = 1 - acur;
    m = m_next;
    ++rounds;
  }
  if (rounds_out) *rounds_out = rounds;
  return check_launch();
}

}  // namespace sg

extern "C" int sg_build_suffix_array(const int32_t* tokens, int64_t n,
                                     int32_t* sa_out, void* workspace,
                                     size_t ws_bytes, int32_t* rounds_out,
                                     sg_stream_t stream) {
  return sg::build_suffix_array(tokens, n, sa_out, workspace, ws_bytes,
                                rounds_out, stream, /*host_pool=*/true);
}

// ---------------------------------------------------------------------------
// Allocation-free variant
// ---------------------------------------------------------------------------
// Some callers cannot allocate device memory at all: a serving engine that
// reserves all free GPU memory for its KV cache at start-up and forbids
// later cudaMalloc calls, or a plugin host that owns every allocation and
// only hands its plugins input and output buffers. For them the suffix-array
// build can run on a scratch array compiled into this library. The array is
// a file-scope __device__ variable: every GPU that loads the library holds
// its kSaNoAllocScratchBytes until the process exits, whether or not the
// entry point is used.
namespace sg {

constexpr size_t kSaNoAllocScratchBytes = size_t(8) << 20;  // 8 MiB

static __device__ __align__(256) unsigned char
    g_sa_noalloc_scratch[kSaNoAllocScratchBytes];

// Device address of the scratch array, looked up once per device. In host
// code the array's name is only a host-side stand-in, so kernels must be
// given the address cudaGetSymbolAddress returns for the current device.
static std::mutex g_noalloc_mu;
static void* g_noalloc_ptr[64] = {nullptr};

static int noalloc_scratch(void** out) {
  const int dev = current_device();
  if (dev < 0 || dev >= 64) return SG_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_sa_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      set_cuda_error(e);
      return SG_ERR_CUDA;
    }
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return SG_OK;
}

// Largest n whose build workspace fits the scratch array.
static int64_t noalloc_max_tokens() {
  int64_t lo = 0, hi = static_cast<int64_t>(kSaNoAllocScratchBytes);
  while (lo < hi) {
    const int64_t mid = lo + (hi - lo + 1) / 2;
    if (carve(nullptr, mid).bytes <= kSaNoAllocScratchBytes) {
      lo = mid;
    } else {
      hi = mid - 1;
    }
  }
  return lo;
}

}  // namespace sg

extern "C" int sg_build_suffix_array_noalloc(const int32_t* tokens,
                                             int64_t n, int32_t* sa_out,
                                             int32_t* rounds_out,
                                             sg_stream_t stream) {
  if (n < 0) return SG_ERR_INVALID;
  static const int64_t max_n = sg::noalloc_max_tokens();
  if (n > max_n) return SG_ERR_UNSUPPORTED;  // input beyond the scratch size
  void* scratch = nullptr;
  // First call on a device: looks up the scratch address (no allocation).
  const int rc = sg::noalloc_scratch(&scratch);
  if (rc != SG_OK) return rc;
  // The build zeroes the per-pass digit totals itself and writes every
  // other scratch region before reading it, so the previous call's leftover
  // contents need no clearing. Its count read-backs land on this thread's
  // stack, not in the page-locked pool (whose creation allocates).
  return sg::build_suffix_array(tokens, n, sa_out, scratch,
                                sg::kSaNoAllocScratchBytes, rounds_out, stream,
                                /*host_pool=*/false);
}
