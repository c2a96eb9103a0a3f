// Suffix-array shards for the multi-GPU global drafter (benchmark config 5).
//
// The reference has one suffix array over the whole corpus and samples a
// match interval in suffix-array order: with ilen suffixes in [start, end)
// and ilen > R it takes start + floor(j * ilen / R), else start + j
// (suffix_gpu/global_index.py:339-352). Split by corpus position, each GPU
// keeps the suffixes that start in its part of the corpus, in the same
// order, each with its global rank (its index in the whole suffix array):
//
// * sg_shard_extract: a shard's (position, global rank) lists from the
//   whole suffix array, one stable compaction;
// * sg_shard_bounds (sa_search.cu): each shard's per-(row, length)
//   intervals; summed over the shards they are the whole-corpus intervals;
// * sg_shard_resolve: per row and cap the reference's longest found length
//   (from the summed intervals), and for each of its samples the position
//   if the sample's global rank is one of this shard's suffixes (else 0:
//   exactly one shard owns each sample, so a sum over the shards fills in
//   every sample), plus, for the rows this GPU drafts, the per-cap plan
//   that points the fused global step at those samples;
// * sg_shard_pack_rows: the rows' tails, tail lengths and drafting flags in
//   the packed layout the two kernels above read (and the collectives
//   move).
#include <cuda_runtime.h>

#include "sg_common.cuh"

namespace sg {

constexpr int kExtractThreads = 256;
constexpr int kExtractItems = 16;
constexpr int kExtractTile = kExtractThreads * kExtractItems;

// Per tile: how many suffix-array entries fall in [lo, hi).
__global__ void __launch_bounds__(kExtractThreads)
    extract_count_kernel(const int32_t* __restrict__ sa, int64_t n,
                         int64_t lo, int64_t hi, uint32_t* __restrict__ cnt) {
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kExtractTile;
  int c = 0;
#pragma unroll 4
  for (int k = 0; k < kExtractItems; ++k) {
    const int64_t i = base + k * kExtractThreads + threadIdx.x;
    if (i < n) {
      const int64_t p = sa[i];
      c += p >= lo && p < hi;
    }
  }
  c = __reduce_add_sync(SG_FULL_MASK, c);
  __shared__ int ws[kExtractThreads / 32];
  if (lane_id() == 0) ws[warp_id()] = c;
  __syncthreads();
  if (threadIdx.x == 0) {
    int t = 0;
    for (int w = 0; w < kExtractThreads / 32; ++w) t += ws[w];
    cnt[blockIdx.x] = static_cast<uint32_t>(t);
  }
}

// Exclusive scan of the tile counts, in place (one block).
__global__ void __launch_bounds__(1024)
    extract_scan_kernel(uint32_t* __restrict__ cnt, int ntiles) {
  __shared__ uint32_t carry;
  __shared__ uint32_t wsum[32];
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (int base = 0; base < ntiles; base += 1024) {
    const int i = base + threadIdx.x;
    const uint32_t v = i < ntiles ? cnt[i] : 0;
    uint32_t x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(SG_FULL_MASK, x, o);
      if (lane_id() >= o) x += y;
    }
    if (lane_id() == 31) wsum[warp_id()] = x;
    __syncthreads();
    if (warp_id() == 0) {
      uint32_t s = wsum[lane_id()];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(SG_FULL_MASK, s, o);
        if (lane_id() >= o) s += y;
      }
      wsum[lane_id()] = s;
    }
    __syncthreads();
    const uint32_t before = carry + (warp_id() ? wsum[warp_id() - 1] : 0);
    if (i < ntiles) cnt[i] = before + x - v;
    __syncthreads();
    if (threadIdx.x == 1023) carry = before + x;
    __syncthreads();
  }
}

// Stable scatter: entry i of the suffix array with its position in
// [lo, hi) goes to slot (tile offset + its rank within the tile) with its
// global rank i. Items are taken in order per warp (ballot prefix).
__global__ void __launch_bounds__(kExtractThreads)
    extract_scatter_kernel(const int32_t* __restrict__ sa, int64_t n,
                           int64_t lo, int64_t hi,
                           const uint32_t* __restrict__ off,
                           int32_t* __restrict__ out_pos,
                           int32_t* __restrict__ out_rank) {
  __shared__ uint32_t wcnt[kExtractThreads / 32];
  __shared__ uint32_t s_base;
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kExtractTile;
  if (threadIdx.x == 0) s_base = off[blockIdx.x];
  // chunk k of the tile: 256 consecutive entries; warps take them in
  // order within the chunk, chunks in order
  for (int k = 0; k < kExtractItems; ++k) {
    const int64_t i = base + static_cast<int64_t>(k) * kExtractThreads +
                      threadIdx.x;
    int32_t p = 0;
    bool take = false;
    if (i < n) {
      p = sa[i];
      take = p >= lo && p < hi;
    }
    const unsigned bal = __ballot_sync(SG_FULL_MASK, take);
    if (lane_id() == 0) wcnt[warp_id()] = __popc(bal);
    __syncthreads();
    uint32_t before = s_base;
    for (int w = 0; w < warp_id(); ++w) before += wcnt[w];
    if (take) {
      const uint32_t slot =
          before + __popc(bal & ((1u << lane_id()) - 1u));
      out_pos[slot] = p;
      out_rank[slot] = static_cast<int32_t>(i);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      uint32_t t = 0;
      for (int w = 0; w < kExtractThreads / 32; ++w) t += wcnt[w];
      s_base += t;
    }
    __syncthreads();
  }
}

// Packed rows: [tail (M), tail length, drafting flag] per row.
__global__ void pack_rows_kernel(const int32_t* __restrict__ tails,
                                 const int64_t* __restrict__ tail_len,
                                 const uint8_t* __restrict__ row_mask, int B,
                                 int M, int32_t* __restrict__ rows) {
  const int W = M + 2;
  const int64_t total = static_cast<int64_t>(B) * W;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x +
                   threadIdx.x;
       i < total; i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int b = static_cast<int>(i / W), j = static_cast<int>(i % W);
    int32_t v;
    if (j < M) {
      v = tails[static_cast<int64_t>(b) * M + j];
    } else if (j == M) {
      v = static_cast<int32_t>(tail_len[b]);
    } else {
      v = row_mask ? (row_mask[b] != 0) : 1;
    }
    rows[i] = v;
  }
}

constexpr int kResolveThreads = 256;
constexpr int kResolveMaxCaps = 16;

// One block per (row, cap), for every row of the job. The cap's best
// length (suffix_match_backoff, sa_search.py:150-163: the longest length
// <= cap and <= the tail length whose summed interval is not empty); caps
// whose best length equals the previous cap's share its samples. Every
// sample slot [row, cap, j < R] gets the sample's corpus position when
// this shard holds the suffix of that global rank, else 0. A shard holding
// few suffixes of the interval walks them (a suffix of global rank
// start + d is sample j when d == floor(j * ilen / R)); otherwise each
// sample's global rank is searched among them. For the rows this GPU
// drafts ([own_lo, own_lo + own_n)) the fused global step's per-cap inputs
// are written: SA length, and a [start, end) range of the sample block
// (min(ilen, R) entries, so the step reads them in order).
__global__ void __launch_bounds__(kResolveThreads)
    shard_resolve_kernel(const int32_t* __restrict__ gb,
                         const int32_t* __restrict__ lb,
                         const int32_t* __restrict__ rows, int M,
                         const int64_t* __restrict__ caps, int C, int R,
                         const int32_t* __restrict__ shard_pos,
                         const int32_t* __restrict__ shard_rank,
                         int32_t* __restrict__ samples, int own_lo, int own_n,
                         int64_t* __restrict__ sa_len,
                         int64_t* __restrict__ sa_start,
                         int64_t* __restrict__ sa_end) {
  extern __shared__ int32_t s_out[];  // [R]
  __shared__ int s_best[kResolveMaxCaps], s_src;
  const int b = blockIdx.x, c = blockIdx.y;
  const int32_t* row = rows + static_cast<int64_t>(b) * (M + 2);
  const int32_t* g = gb + static_cast<int64_t>(b) * M * 2;
  const int32_t* l = lb + static_cast<int64_t>(b) * M * 2;
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    const int tl = row[M], active = row[M + 1];
    if (lane < C && lane <= c) {
      int best = 0;
      if (active) {
        const int64_t cap = caps[lane];
        for (int len = 1; len <= M; ++len)
          if (len <= cap && len <= tl && g[2 * len - 1] > g[2 * len - 2])
            best = len;
      }
      s_best[lane] = best;
    }
    __syncwarp();
    if (lane == 0) {
      // first cap of the run of caps with this best length
      int src = c;
      while (src > 0 && s_best[src - 1] == s_best[c]) --src;
      s_src = src;
    }
  }
  __syncthreads();
  const int best = s_best[c];
  const int src = s_src;
  const int64_t own = static_cast<int64_t>(b) - own_lo;
  int64_t start = 0, ilen = 0;
  if (best > 0) {
    start = g[2 * best - 2];
    ilen = static_cast<int64_t>(g[2 * best - 1]) - start;
  }
  const int64_t cnt = ilen < R ? ilen : R;
  if (own >= 0 && own < own_n && threadIdx.x == 0) {
    const int64_t o = own * C + c;
    sa_len[o] = best;
    const int64_t st = best > 0 ? (own * C + src) * R : 0;
    sa_start[o] = st;
    sa_end[o] = best > 0 ? st + cnt : 0;
  }
  int32_t* out = samples + (static_cast<int64_t>(b) * C + c) * R;
  if (best == 0 || src != c) {
    for (int j = threadIdx.x; j < R; j += kResolveThreads) out[j] = 0;
    return;
  }
  const int64_t lo = l[2 * best - 2], hi = l[2 * best - 1];
  if (hi - lo <= 4 * static_cast<int64_t>(R)) {
    for (int j = threadIdx.x; j < R; j += kResolveThreads) s_out[j] = 0;
    __syncthreads();
    for (int64_t k = lo + threadIdx.x; k < hi; k += kResolveThreads) {
      const int64_t d = static_cast<int64_t>(shard_rank[k]) - start;
      int64_t j;
      if (ilen > R) {
        j = (d * R + ilen - 1) / ilen;  // smallest j with j * ilen / R >= d
        if (j >= R || (j * ilen) / R != d) continue;
      } else {
        j = d;
      }
      s_out[j] = shard_pos[k];
    }
    __syncthreads();
    for (int j = threadIdx.x; j < R; j += kResolveThreads) out[j] = s_out[j];
    return;
  }
  for (int j = threadIdx.x; j < R; j += kResolveThreads) {
    int32_t v = 0;
    if (j < cnt) {
      const int64_t want =
          start + (ilen > R ? (static_cast<int64_t>(j) * ilen) / R : j);
      // this shard's suffixes of the interval, ascending global ranks
      int64_t a = lo, z = hi;
      while (a < z) {
        const int64_t m = (a + z) >> 1;
        if (shard_rank[m] < want) {
          a = m + 1;
        } else {
          z = m;
        }
      }
      if (a < hi && shard_rank[a] == want) v = shard_pos[a];
    }
    out[j] = v;
  }
}

}  // namespace sg

using namespace sg;

extern "C" size_t sg_shard_extract_workspace_size(int64_t n) {
  if (n < 0) return 0;
  return static_cast<size_t>(ceil_div(n > 0 ? n : 1, kExtractTile)) * 4;
}

extern "C" int sg_shard_extract(const int32_t* sa, int64_t n, int64_t lo,
                                int64_t hi, int32_t* shard_pos,
                                int32_t* shard_rank, void* workspace,
                                size_t workspace_bytes, sg_stream_t stream) {
  sg::NvtxScope nvtx_range("sg_shard_extract");
  if (n < 0 || n > INT32_MAX || lo < 0 || hi < lo || hi > n)
    return SG_ERR_INVALID;
  if (n == 0 || hi == lo) return SG_OK;
  if (!sa || !shard_pos || !shard_rank) return SG_ERR_INVALID;
  const int64_t ntiles = ceil_div(n, kExtractTile);
  if (!workspace || workspace_bytes < sg_shard_extract_workspace_size(n))
    return SG_ERR_WORKSPACE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  uint32_t* cnt = static_cast<uint32_t*>(workspace);
  extract_count_kernel<<<static_cast<unsigned>(ntiles), kExtractThreads, 0,
                         st>>>(sa, n, lo, hi, cnt);
  extract_scan_kernel<<<1, 1024, 0, st>>>(cnt, static_cast<int>(ntiles));
  extract_scatter_kernel<<<static_cast<unsigned>(ntiles), kExtractThreads, 0,
                           st>>>(sa, n, lo, hi, cnt, shard_pos, shard_rank);
  return check_launch();
}

extern "C" int sg_shard_pack_rows(const int32_t* tails,
                                  const int64_t* tail_len,
                                  const uint8_t* row_mask, int32_t batch,
                                  int32_t max_len, int32_t* rows,
                                  sg_stream_t stream) {
  if (batch < 0 || max_len < 1) return SG_ERR_INVALID;
  if (batch == 0) return SG_OK;
  if (!tails || !tail_len || !rows) return SG_ERR_INVALID;
  const int64_t total = static_cast<int64_t>(batch) * (max_len + 2);
  const int64_t blocks = ceil_div(total, 256);
  pack_rows_kernel<<<static_cast<unsigned>(blocks < 1024 ? blocks : 1024),
                     256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      tails, tail_len, row_mask, batch, max_len, rows);
  return check_launch();
}

extern "C" int sg_shard_resolve(const int32_t* bounds_sum,
                                const int32_t* bounds_local,
                                const int32_t* rows, int32_t batch,
                                int32_t max_len, const int64_t* caps,
                                int32_t num_caps, int32_t max_occ,
                                const int32_t* shard_pos,
                                const int32_t* shard_rank, int32_t* samples,
                                int32_t own_lo, int32_t own_n,
                                int64_t* sa_len, int64_t* sa_start,
                                int64_t* sa_end, sg_stream_t stream) {
  sg::NvtxScope nvtx_range("sg_shard_resolve");
  if (batch < 0 || max_len < 1 || num_caps < 1 ||
      num_caps > kResolveMaxCaps || max_occ < 1 || own_lo < 0 || own_n < 0 ||
      own_lo + own_n > batch)
    return SG_ERR_INVALID;
  if (batch == 0) return SG_OK;
  if (!bounds_sum || !bounds_local || !rows || !caps || !samples ||
      (own_n > 0 && (!sa_len || !sa_start || !sa_end)))
    return SG_ERR_INVALID;
  const size_t smem = static_cast<size_t>(max_occ) * 4;
  static int cache[64] = {0};
  const int rc = ensure_dyn_smem(shard_resolve_kernel, smem, cache);
  if (rc != SG_OK) return rc;
  shard_resolve_kernel<<<dim3(static_cast<unsigned>(batch),
                              static_cast<unsigned>(num_caps)),
                         kResolveThreads, smem,
                         reinterpret_cast<cudaStream_t>(stream)>>>(
      bounds_sum, bounds_local, rows, max_len, caps, num_caps, max_occ,
      shard_pos, shard_rank, samples, own_lo, own_n, sa_len, sa_start,
      sa_end);
  return check_launch();
}
