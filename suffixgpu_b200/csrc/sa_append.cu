// Incremental suffix-array rebuild for the global index: the suffix array
// of a new snapshot from the previous snapshot's suffix array, without
// re-sorting the kept corpus.
//
// A rebuild of GlobalIndex._launch_rebuild (suffix_gpu/global_index.py:
// 147-223) forms the snapshot  S = Y . Z [. PAD]: Y is the previous active
// corpus with its oldest documents evicted, Z the absorbed delta documents,
// PAD the sentinel column. The reference sorts all of S from scratch
// (suffix_array.py:15-63). Here:
//   * Let L bound the longest common prefix of two distinct suffixes of the
//     previous snapshot (a build reports rounds with L < 2^rounds) and
//     W = 2^rounds. Two suffixes that start in Y with more than W tokens of
//     Y left first differ inside Y, so they keep the relative order they
//     had in the previous suffix array ("kept" suffixes, A, read off the
//     previous array in one order-preserving compaction).
//   * The suffixes that start in the last W tokens of Y or later ("tail"
//     suffixes, B) are sorted by the full builder as the suffixes of the
//     string S[|Y| - W ..): their order is decided inside that string.
//   * Merge: every tail suffix finds the number of kept suffixes smaller
//     than it by a binary search over A with warp-wide suffix comparisons
//     on S (the comparison starts at the smaller of the two boundary LCPs,
//     Manber-Myers) cut at depth W: kept suffixes differ from each other
//     within W tokens, so at most one of them (the "twin") shares W tokens
//     with a tail suffix, and only a comparison with the twin needs to go
//     deeper. A kept suffix is longer than every tail suffix, so a full
//     comparison ends at the latest where the tail suffix ends. Both lists
//     are then scattered into place.
// The result is the unique suffix array of S, identical to a full build.
// The new bound: the longest common prefix of two adjacent suffixes of S is
// one of a kept pair (< 2^prev_rounds), a tail pair (the tail build's
// rounds) or a tail suffix and its kept neighbour (measured by the merge).
#include <cuda_runtime.h>

#include "sg_common.cuh"

namespace sg {

constexpr int kAppThreads = 256;
constexpr int kAppItems = 16;
constexpr int kAppBlock = kAppThreads * kAppItems;  // entries per block
constexpr int kAppWarps = kAppThreads / 32;

__device__ __forceinline__ int block_sum_256(int v, int* red) {
  v = __reduce_add_sync(SG_FULL_MASK, v);
  if (lane_id() == 0) red[warp_id()] = v;
  __syncthreads();
  int s = 0;
#pragma unroll
  for (int w = 0; w < kAppWarps; ++w) s += red[w];
  __syncthreads();
  return s;
}

// Block b: how many previous-array entries of its 4096 hold a position in
// [lo, hi) (the kept suffixes).
__global__ void __launch_bounds__(kAppThreads)
    append_count_kernel(const int32_t* __restrict__ prev_sa, int64_t prev_n,
                        int64_t lo, int64_t hi, int32_t* __restrict__ blk) {
  __shared__ int red[kAppWarps];
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kAppBlock;
  int c = 0;
#pragma unroll
  for (int r = 0; r < kAppItems; ++r) {
    const int64_t i = base + r * kAppThreads + threadIdx.x;
    if (i < prev_n) {
      const int64_t p = prev_sa[i];
      c += (p >= lo && p < hi) ? 1 : 0;
    }
  }
  c = block_sum_256(c, red);
  if (threadIdx.x == 0) blk[blockIdx.x] = c;
}

// In place: blk[i] <- sum of blk[0..i) (one block of 1024 threads).
__global__ void __launch_bounds__(1024)
    append_scan_kernel(int32_t* __restrict__ blk, int nblk) {
  __shared__ int wsum[32];
  __shared__ int carry;
  const int lane = lane_id(), warp = warp_id();
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (int c0 = 0; c0 < nblk; c0 += 1024) {
    const int i = c0 + threadIdx.x;
    const int x = i < nblk ? blk[i] : 0;
    const int inc = warp_incl_scan(x);
    if (lane == 31) wsum[warp] = inc;
    __syncthreads();
    int pre = carry, tot = 0;
    for (int w = 0; w < 32; ++w) {
      if (w < warp) pre += wsum[w];
      tot += wsum[w];
    }
    if (i < nblk) blk[i] = pre + inc - x;
    __syncthreads();
    if (threadIdx.x == 0) carry += tot;
    __syncthreads();
  }
}

// Order-preserving compaction of the kept positions, shifted to the new
// snapshot's coordinates: kept[rank] = p - lo.
__global__ void __launch_bounds__(kAppThreads)
    append_compact_kernel(const int32_t* __restrict__ prev_sa, int64_t prev_n,
                          int64_t lo, int64_t hi,
                          const int32_t* __restrict__ blk,
                          int32_t* __restrict__ kept) {
  __shared__ int wcnt[kAppWarps];
  const int lane = lane_id(), warp = warp_id();
  const unsigned lt = (1u << lane) - 1u;
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kAppBlock;
  int64_t out = blk[blockIdx.x];
#pragma unroll 1
  for (int r = 0; r < kAppItems; ++r) {
    const int64_t i = base + r * kAppThreads + threadIdx.x;
    int64_t p = -1;
    if (i < prev_n) p = prev_sa[i];
    const bool keep = p >= lo && p < hi;
    const unsigned bal = __ballot_sync(SG_FULL_MASK, keep);
    if (lane == 0) wcnt[warp] = __popc(bal);
    __syncthreads();
    int pre = 0, tot = 0;
#pragma unroll
    for (int w = 0; w < kAppWarps; ++w) {
      const int c = wcnt[w];
      if (w < warp) pre += c;
      tot += c;
    }
    if (keep)
      kept[out + pre + __popc(bal & lt)] = static_cast<int32_t>(p - lo);
    out += tot;
    __syncthreads();
  }
}

// One 32-token step of a comparison of suffix a (kept) with suffix t
// (tail, a < t) at offsets [off, off + 32), cut at lim. Suffix t is the
// shorter one: where it has ended (t + o >= m) suffix a still has a token
// (a + o < m), so the first such offset is a difference that makes a > t
// (the end of a string sorts first); there every load is skipped. Returns
// 0 if no difference below lim, else -1 / 1 with *l at the difference.
__device__ __forceinline__ int cmp_step32(const int32_t* __restrict__ s,
                                          int64_t m, int64_t a, int64_t t,
                                          int64_t off, int64_t lim,
                                          int64_t* l) {
  const int lane = lane_id();
  const int64_t o = off + lane;
  const bool t_end = t + o >= m;
  int32_t va = 0, vt = 0;
  if (!t_end && o < lim) {
    va = s[a + o];
    vt = s[t + o];
  }
  const unsigned d =
      __ballot_sync(SG_FULL_MASK, o < lim && (t_end || va != vt));
  if (!d) return 0;
  const int b = __ffs(d) - 1;
  const bool e = __shfl_sync(SG_FULL_MASK, t_end, b);
  const int32_t xa = __shfl_sync(SG_FULL_MASK, va, b);
  const int32_t xt = __shfl_sync(SG_FULL_MASK, vt, b);
  *l = off + b;
  return (e || xa > xt) ? 1 : -1;
}

// Warp-wide three-way comparison of suffix a (kept) with suffix t (tail,
// t > a) from offset *l (a prefix both are known to share) up to offset
// lim: -1 if a < t, 1 if a > t, 0 if they agree through lim - 1. *l leaves
// as the longest common prefix (lim for 0). Most comparisons of a binary
// search end within a few tokens, so the first step reads 32 tokens per
// side; longer ones continue 128 tokens per step (four independent 32-token
// loads per side in flight). With lim > m - t the result is never 0.
__device__ __forceinline__ int warp_cmp_upto(const int32_t* __restrict__ s,
                                             int64_t m, int64_t a, int64_t t,
                                             int64_t* l, int64_t lim) {
  int64_t off = *l;
  if (off < lim) {
    const int c = cmp_step32(s, m, a, t, off, lim, l);
    if (c) return c;
    off += 32;
  }
  const int lane = lane_id();
  for (; off < lim; off += 128) {
    const int64_t o0 = off + lane, o1 = o0 + 32, o2 = o0 + 64, o3 = o0 + 96;
    const bool e0 = t + o0 >= m, e1 = t + o1 >= m, e2 = t + o2 >= m,
               e3 = t + o3 >= m;
    int32_t a0 = 0, t0 = 0, a1 = 0, t1 = 0, a2 = 0, t2 = 0, a3 = 0, t3 = 0;
    if (!e0 && o0 < lim) { a0 = s[a + o0]; t0 = s[t + o0]; }
    if (!e1 && o1 < lim) { a1 = s[a + o1]; t1 = s[t + o1]; }
    if (!e2 && o2 < lim) { a2 = s[a + o2]; t2 = s[t + o2]; }
    if (!e3 && o3 < lim) { a3 = s[a + o3]; t3 = s[t + o3]; }
    const unsigned d0 = __ballot_sync(SG_FULL_MASK, o0 < lim && (e0 || a0 != t0));
    const unsigned d1 = __ballot_sync(SG_FULL_MASK, o1 < lim && (e1 || a1 != t1));
    const unsigned d2 = __ballot_sync(SG_FULL_MASK, o2 < lim && (e2 || a2 != t2));
    const unsigned d3 = __ballot_sync(SG_FULL_MASK, o3 < lim && (e3 || a3 != t3));
    if (d0 | d1 | d2 | d3) {
      // first differing 32-token chunk j and lane b; values from lane b
      const int j = d0 ? 0 : d1 ? 1 : d2 ? 2 : 3;
      const unsigned d = j == 0 ? d0 : j == 1 ? d1 : j == 2 ? d2 : d3;
      const int b = __ffs(d) - 1;
      const bool ej = j == 0 ? e0 : j == 1 ? e1 : j == 2 ? e2 : e3;
      const int32_t aj = j == 0 ? a0 : j == 1 ? a1 : j == 2 ? a2 : a3;
      const int32_t tj = j == 0 ? t0 : j == 1 ? t1 : j == 2 ? t2 : t3;
      const bool e = __shfl_sync(SG_FULL_MASK, ej, b);
      const int32_t xa = __shfl_sync(SG_FULL_MASK, aj, b);
      const int32_t xt = __shfl_sync(SG_FULL_MASK, tj, b);
      *l = off + 32 * j + b;
      return (e || xa > xt) ? 1 : -1;
    }
  }
  *l = lim;
  return 0;
}

// Warp per tail suffix k: pos[k] = number of kept suffixes smaller than it.
// Binary search over the kept list with comparisons cut at depth W (every
// other kept suffix differs from one that shares W tokens with t within
// those W tokens, so a cut comparison is exact unless it meets that one
// "twin"). On the twin a = kept[mid]: pos = mid + (a < t), from one full
// comparison. The largest LCP with a kept neighbour goes into *lcp_max.
__global__ void __launch_bounds__(kAppThreads)
    append_rank_kernel(const int32_t* __restrict__ s, int64_t m,
                       const int32_t* __restrict__ kept, int64_t n_kept,
                       const int32_t* __restrict__ tail, int64_t n_tail,
                       int64_t t0, int64_t wlen, int32_t* __restrict__ pos,
                       unsigned long long* __restrict__ lcp_max) {
  const int64_t k =
      static_cast<int64_t>(blockIdx.x) * kAppWarps + warp_id();
  if (k >= n_tail) return;
  const int64_t t = t0 + tail[k];
  int64_t lo = 0, hi = n_kept;
  int64_t llcp = 0, rlcp = 0;  // LCP of t with kept[lo - 1] / kept[hi]
  int64_t res = -1, best = 0;
  while (lo < hi) {
    const int64_t mid = (lo + hi) >> 1;
    const int64_t a = kept[mid];
    int64_t l = llcp < rlcp ? llcp : rlcp;
    const int c = warp_cmp_upto(s, m, a, t, &l, wlen);
    if (c == 0) {  // the twin: decide the side with one full comparison
      const int c2 = warp_cmp_upto(s, m, a, t, &l, m - t + 1);
      res = mid + (c2 < 0 ? 1 : 0);
      best = l;
      break;
    }
    if (c < 0) {
      lo = mid + 1;
      llcp = l;
    } else {
      hi = mid;
      rlcp = l;
    }
  }
  if (res < 0) {
    res = lo;
    if (lo > 0) best = llcp;
    if (lo < n_kept && rlcp > best) best = rlcp;
  }
  if (lane_id() == 0) {
    pos[k] = static_cast<int32_t>(res);
    atomicMax(lcp_max, static_cast<unsigned long long>(best));
  }
}

__global__ void append_place_tail_kernel(const int32_t* __restrict__ tail,
                                         const int32_t* __restrict__ pos,
                                         int64_t n_tail, int64_t t0,
                                         int32_t* __restrict__ sa_out) {
  const int64_t k = static_cast<int64_t>(blockIdx.x) * blockDim.x +
                    threadIdx.x;
  if (k < n_tail)
    sa_out[k + pos[k]] = static_cast<int32_t>(t0 + tail[k]);
}

// Number of entries of the non-decreasing pos[0..n) that are <= r.
__device__ __forceinline__ int64_t count_le(const int32_t* __restrict__ pos,
                                            int64_t n, int64_t r) {
  int64_t lo = 0, hi = n;
  while (lo < hi) {
    const int64_t mid = (lo + hi) >> 1;
    if (pos[mid] <= r)
      lo = mid + 1;
    else
      hi = mid;
  }
  return lo;
}

// Kept suffix of rank r goes after the r kept and the count_le(r) tail
// suffixes smaller than it. The block narrows the tail range once for its
// 4096 ranks.
__global__ void __launch_bounds__(kAppThreads)
    append_place_kept_kernel(const int32_t* __restrict__ kept, int64_t n_kept,
                             const int32_t* __restrict__ pos, int64_t n_tail,
                             int32_t* __restrict__ sa_out) {
  __shared__ int64_t range[2];
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * kAppBlock;
  int64_t r1 = r0 + kAppBlock;
  if (r1 > n_kept) r1 = n_kept;
  if (threadIdx.x == 0) range[0] = count_le(pos, n_tail, r0 - 1);
  if (threadIdx.x == 32) range[1] = count_le(pos, n_tail, r1 - 1);
  __syncthreads();
  const int64_t cb = range[0], cn = range[1] - range[0];
#pragma unroll 4
  for (int i = 0; i < kAppItems; ++i) {
    const int64_t r = r0 + i * kAppThreads + threadIdx.x;
    if (r < r1)
      sa_out[r + cb + count_le(pos + cb, cn, r)] = kept[r];
  }
}

struct AppendWorkspace {
  int32_t* kept;
  int32_t* tail;
  int32_t* pos;
  int32_t* blk;
  unsigned long long* lcp_max;
  void* build_ws;
  size_t build_bytes;
  size_t bytes;
};

static AppendWorkspace carve_append(void* base, int64_t n) {
  AppendWorkspace w{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    char* p = base ? static_cast<char*>(base) + off : nullptr;
    off += (bytes + 255) & ~size_t(255);
    return p;
  };
  const int64_t nblk = ceil_div(n, kAppBlock) + 1;
  w.kept = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * n));
  w.tail = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * n));
  w.pos = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * n));
  w.blk = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * nblk));
  w.lcp_max =
      reinterpret_cast<unsigned long long*>(take(sizeof(unsigned long long)));
  w.build_bytes = sg_suffix_array_workspace_size(n);
  w.build_ws = take(w.build_bytes);
  w.bytes = off;
  return w;
}

static int bits_for(int64_t v) {  // smallest R with v < 2^R
  int r = 0;
  while (r < 62 && (int64_t(1) << r) <= v) ++r;
  return r;
}

}  // namespace sg

using namespace sg;

extern "C" size_t sg_suffix_array_append_workspace_size(int64_t n) {
  if (n < 0) return 0;
  return carve_append(nullptr, n).bytes;
}

extern "C" int sg_suffix_array_append(
    const int32_t* tokens, int64_t n, const int32_t* prev_sa, int64_t prev_n,
    int64_t evicted, int64_t kept_len, int32_t prev_rounds, int32_t* sa_out,
    void* workspace, size_t ws_bytes, int32_t* rounds_out,
    sg_stream_t stream) {
  sg::NvtxScope nvtx_range("sg_suffix_array_append");
  if (n < 0 || prev_n < 0 || evicted < 0 || kept_len < 0 || prev_rounds < 0)
    return SG_ERR_INVALID;
  if (n >= (int64_t(1) << 31) - 1 || prev_n >= (int64_t(1) << 31) - 1)
    return SG_ERR_UNSUPPORTED;
  if (kept_len > n || evicted + kept_len > prev_n) return SG_ERR_INVALID;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (rounds_out) *rounds_out = 0;
  if (n == 0) return SG_OK;
  if (!tokens || !sa_out || (kept_len > 0 && !prev_sa)) return SG_ERR_INVALID;
  if (!workspace || ws_bytes < carve_append(nullptr, n).bytes)
    return SG_ERR_WORKSPACE;
  AppendWorkspace w = carve_append(workspace, n);

  // kept suffixes: more than W tokens of the kept corpus left
  const int64_t wlen = prev_rounds >= 31 ? (int64_t(1) << 31)
                                         : (int64_t(1) << prev_rounds);
  const int64_t n_kept = kept_len > wlen ? kept_len - wlen : 0;
  const int64_t t0 = n_kept;  // first tail position
  const int64_t n_tail = n - t0;

  int32_t tail_rounds = 0;
  if (n_kept == 0) {
    // nothing to keep: a full build
    return sg_build_suffix_array(tokens, n, sa_out, w.build_ws,
                                 w.build_bytes, rounds_out, stream);
  }
  const int rc = sg_build_suffix_array(tokens + t0, n_tail, w.tail,
                                       w.build_ws, w.build_bytes,
                                       &tail_rounds, stream);
  if (rc != SG_OK) return rc;

  const int nblk = static_cast<int>(ceil_div(prev_n, kAppBlock));
  const int64_t lo = evicted, hi = evicted + n_kept;
  append_count_kernel<<<nblk, kAppThreads, 0, st>>>(prev_sa, prev_n, lo, hi,
                                                    w.blk);
  append_scan_kernel<<<1, 1024, 0, st>>>(w.blk, nblk);
  append_compact_kernel<<<nblk, kAppThreads, 0, st>>>(prev_sa, prev_n, lo,
                                                      hi, w.blk, w.kept);
  cudaError_t e =
      cudaMemsetAsync(w.lcp_max, 0, sizeof(unsigned long long), st);
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return SG_ERR_CUDA;
  }
  append_rank_kernel<<<static_cast<unsigned>(ceil_div(n_tail, kAppWarps)),
                       kAppThreads, 0, st>>>(tokens, n, w.kept, n_kept,
                                             w.tail, n_tail, t0, wlen, w.pos,
                                             w.lcp_max);
  append_place_tail_kernel<<<static_cast<unsigned>(ceil_div(n_tail, 256)),
                             256, 0, st>>>(w.tail, w.pos, n_tail, t0, sa_out);
  append_place_kept_kernel<<<static_cast<unsigned>(
                                 ceil_div(n_kept, kAppBlock)),
                             kAppThreads, 0, st>>>(w.kept, n_kept, w.pos,
                                                   n_tail, sa_out);
  int st_launch = check_launch();
  if (st_launch != SG_OK) return st_launch;
  int64_t lcp_ab = 0;
  const int rr = read_device_i64(reinterpret_cast<const int64_t*>(w.lcp_max),
                                 &lcp_ab, st);
  if (rr != SG_OK) return rr;
  int rounds = prev_rounds;
  if (tail_rounds > rounds) rounds = tail_rounds;
  const int rab = bits_for(lcp_ab);
  if (rab > rounds) rounds = rab;
  if (rounds_out) *rounds_out = rounds;
  return SG_OK;
}
