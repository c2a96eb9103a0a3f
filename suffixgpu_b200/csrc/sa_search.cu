// Suffix-array interval search for sm_100a.
//
// Reproduces suffix_gpu/sa_search.py: search_interval (:66-107, Triton
// _sa_search_kernel triton_kernels.py:56-94) and suffix_match_backoff
// (:110-163). The lower bound (first suffix with cmp >= 0) and the upper
// bound (first with cmp > 0) run the reference's fixed
// ceil(log2(n + 1))-iteration loop with the same midpoint rule and the
// same comparator (_cmp_pattern, :25-63: corpus tokens past the end read
// -1, pattern positions past its length always match), so the bounds are
// identical to the reference's for any SA.
//
// One warp runs both bounds of a pattern: lane j holds pattern column j
// (and j + 32, ...), so a probe reads the suffix's columns with one
// coalesced load and finds the first mismatch with a ballot; the two
// bounds share their probes until one compares equal. The backoff variant
// searches every suffix length 1..M of each row's tail on one cluster of 8
// CTAs (one warp per length); CTA 0 gathers the intervals through
// distributed shared memory and keeps, per cap, the longest found length
// <= cap. Patterns wider than 128 columns use one thread per bound.
#include <cooperative_groups.h>
#include <cuda_runtime.h>

#include "sg_common.cuh"

namespace sg {

// _cmp_pattern (sa_search.py:25-63) for the suffix at SA index `mid` and a
// pattern of width M read through pat(j), valid length plen:
// -1 suffix < pattern, 0 suffix starts with pattern, 1 suffix > pattern.
// Columns j >= plen always match; lcp = min(leading matches over the M
// columns, plen); a full match (lcp >= plen) compares equal; otherwise the
// suffix token at lcp (-1 past the end) is compared with pat(min(lcp, M-1)).
template <class PatFn>
__device__ __forceinline__ int sa_cmp(const int32_t* __restrict__ sa,
                                      const int32_t* __restrict__ corpus,
                                      int64_t n, int64_t mid, PatFn pat,
                                      int64_t plen, int M) {
  const int64_t pos = sa[mid];
  const int lim = plen < M ? (plen > 0 ? static_cast<int>(plen) : 0) : M;
  int lcp = 0;
  int tok = 0;
  for (; lcp < lim; ++lcp) {
    const int64_t x = pos + lcp;
    tok = x < n ? corpus[x] : -1;
    if (tok != pat(lcp)) break;
  }
  if (lcp == lim) {
    // every column up to min(plen, M) matched
    if (plen <= M) return 0;
    // plen > M: lcp = M, not a full match; compare with pat(M - 1)
    const int64_t x = pos + M;
    tok = x < n ? corpus[x] : -1;
    const int pc = pat(M - 1);
    return tok < pc ? -1 : (tok > pc ? 1 : 0);
  }
  const int pc = pat(lcp);
  return tok < pc ? -1 : 1;
}

template <class PatFn>
__device__ __forceinline__ int64_t sa_bound(const int32_t* __restrict__ sa,
                                            const int32_t* __restrict__ corpus,
                                            int64_t n, int iters, PatFn pat,
                                            int64_t plen, int M, bool upper) {
  int64_t lo = 0, hi = n;
  for (int it = 0; it < iters; ++it) {
    int64_t mid = (lo + hi) >> 1;
    if (mid > n - 1) mid = n - 1;
    const int c = sa_cmp(sa, corpus, n, mid, pat, plen, M);
    const bool right = c < 0 || (upper && c == 0);
    if (right) {
      lo = mid + 1;
    } else {
      hi = mid;
    }
  }
  return lo;
}

__host__ __device__ inline int sa_iters(int64_t n) {
  // ceil(log2(n + 1)), at least 1
  int it = 0;
  while ((int64_t(1) << it) < n + 1) ++it;
  return it < 1 ? 1 : it;
}

// search_interval: thread per (row, bound); pattern rows in global memory.
__global__ void sa_search_kernel(const int32_t* __restrict__ sa,
                                 const int32_t* __restrict__ corpus,
                                 int64_t n, const int32_t* __restrict__ pat,
                                 int M, const int64_t* __restrict__ plen,
                                 int B, int iters, int64_t* __restrict__ start,
                                 int64_t* __restrict__ end) {
  extern __shared__ int pbuf[];  // [blockDim.x][M]
  const int gid = blockIdx.x * blockDim.x + threadIdx.x;
  if (gid >= 2 * B) return;
  const int row = gid % B;
  const bool upper = gid >= B;
  int* p = pbuf + threadIdx.x * M;
  for (int j = 0; j < M; ++j) p[j] = pat[static_cast<int64_t>(row) * M + j];
  auto pf = [&](int j) -> int { return p[j]; };
  const int64_t r = sa_bound(sa, corpus, n, iters, pf, plen[row], M, upper);
  (upper ? end : start)[row] = r;
}

// suffix_match_backoff: block per row, thread per (length, bound).
__global__ void sa_backoff_kernel(const int32_t* __restrict__ sa,
                                  const int32_t* __restrict__ corpus,
                                  int64_t n, const int32_t* __restrict__ query,
                                  int Q, const int64_t* __restrict__ qlen,
                                  int M, const int64_t* __restrict__ caps,
                                  int C, const uint8_t* __restrict__ row_mask,
                                  int iters, int64_t* __restrict__ out_len,
                                  int64_t* __restrict__ out_start,
                                  int64_t* __restrict__ out_end) {
  extern __shared__ int smem_i[];
  int* qs = smem_i;                       // [Q] query row
  int64_t* st = reinterpret_cast<int64_t*>(smem_i + ((Q + 1) & ~1));  // [M]
  int64_t* en = st + M;                   // [M]
  const int b = blockIdx.x;
  const bool active = !row_mask || row_mask[b];
  const int64_t ql = qlen[b];
  for (int j = threadIdx.x; j < Q; j += blockDim.x)
    qs[j] = query[static_cast<int64_t>(b) * Q + j];
  __syncthreads();
  for (int task = threadIdx.x; task < 2 * M; task += blockDim.x) {
    const int l = task % M + 1;  // pattern length
    const bool upper = task >= M;
    int64_t r = 0;
    if (active && l <= ql) {
      // pattern_l[j] = query[qlen - l + j] for j < l (indices >= 0 here;
      // the gather clamps them to the query width like the reference)
      const int64_t o = ql - l;
      auto pf = [&](int j) -> int {
        const int64_t x = o + j;
        return qs[x < Q ? x : Q - 1];
      };
      r = sa_bound(sa, corpus, n, iters, pf, l, M, upper);
    }
    (upper ? en : st)[l - 1] = r;
  }
  __syncthreads();
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    const int64_t cap = caps[c];
    int64_t best = 0;
    if (active) {
      for (int l = 1; l <= M; ++l)
        if (l <= cap && l <= ql && en[l - 1] > st[l - 1]) best = l;
    }
    const int64_t o = static_cast<int64_t>(b) * C + c;
    out_len[o] = best;
    out_start[o] = best > 0 ? st[best - 1] : 0;
    out_end[o] = best > 0 ? en[best - 1] : 0;
  }
}


// ---------------------------------------------------------------------------
// Warp-per-bound search
// ---------------------------------------------------------------------------
namespace cg = cooperative_groups;

constexpr int kSWarps = 8;   // warps per block of the search_interval kernel
constexpr int kSCG = 8;      // CTAs per row of the backoff cluster kernel
constexpr int kSMaxCols = 4; // pattern columns per lane (width <= 128)

// The columns of the suffix at corpus position pos that a probe compares:
// lane j reads column j + 32 k into tok[k] (columns >= lim read 0; past
// the corpus end -1); lane 0 also reads column M into tm when the pattern
// is longer than its width M (the reference then compares that token).
// Positions are below n < 2^31 - 1, so index arithmetic is 32-bit (the
// search is bound by instruction issue: thousands of warps probe at once).
template <int NC>
__device__ __forceinline__ void load_probe(const int32_t* __restrict__ corpus,
                                           uint32_t n, uint32_t pos, int lim,
                                           int64_t plen, int M, int (&tok)[NC],
                                           int& tm) {
  const int lane = lane_id();
#pragma unroll
  for (int k = 0; k < NC; ++k) {
    const int j = lane + 32 * k;
    tok[k] = 0;
    if (j < lim) {
      const uint32_t x = pos + static_cast<uint32_t>(j);
      tok[k] = x < n ? corpus[x] : -1;
    }
  }
  tm = 0;
  if (plen > M && lane == 0) {
    const uint32_t x = pos + static_cast<uint32_t>(M);
    tm = x < n ? corpus[x] : -1;
  }
}

// _cmp_pattern on a loaded probe, with lane j holding pattern column
// j + 32 k in pc[k] (columns >= lim are ignored). Warp-uniform result.
template <int NC>
__device__ __forceinline__ int cmp_probe(const int (&tok)[NC], int tm,
                                         const int (&pc)[NC], int lim,
                                         int64_t plen, int M) {
  const int lane = lane_id();
#pragma unroll
  for (int k = 0; k < NC; ++k) {
    const int j = lane + 32 * k;
    const unsigned bal = __ballot_sync(SG_FULL_MASK, j < lim && tok[k] != pc[k]);
    if (bal) {  // first mismatching column: compare token with pattern
      const int f = __ffs(bal) - 1;
      const int tv = __shfl_sync(SG_FULL_MASK, tok[k], f);
      const int pv = __shfl_sync(SG_FULL_MASK, pc[k], f);
      return tv < pv ? -1 : 1;
    }
  }
  if (plen <= M) return 0;  // every column up to min(plen, M) matched
  // plen > M: the token at column M against pattern column M - 1
  const int tv = __shfl_sync(SG_FULL_MASK, tm, 0);
  int src = 0;
#pragma unroll
  for (int k = 0; k < NC; ++k)
    if (k == ((M - 1) >> 5)) src = pc[k];
  const int pv = __shfl_sync(SG_FULL_MASK, src, (M - 1) & 31);
  return tv < pv ? -1 : (tv > pv ? 1 : 0);
}

__device__ __forceinline__ uint32_t sa_mid(uint32_t lo, uint32_t hi,
                                           uint32_t n) {
  const uint32_t m = (lo + hi) >> 1;
  return m > n - 1 ? n - 1 : m;
}

// Both bounds of one pattern (lower: first suffix with cmp >= 0, upper:
// first with cmp > 0) by the reference's midpoint rule. The two searches
// take the same steps until a probe compares equal, so they share those
// probes; from there the lower bound continues below the equal probe and
// the upper bound above it, both probes of a step loaded together. Once a
// bound's range is empty every further step of the reference's fixed
// ceil(log2(n + 1)) count leaves it unchanged, so its loop stops there.
// n: entries of sa; nc: tokens of corpus (equal for a whole-corpus suffix
// array; a shard's suffix array holds fewer entries than the corpus).
template <int NC>
__device__ __forceinline__ void warp_bounds_cols(
    const int32_t* __restrict__ sa, const int32_t* __restrict__ corpus,
    uint32_t n, uint32_t nc, int iters, const int (&pc)[NC], int M, int lim,
    int64_t plen, uint32_t& out_lo, uint32_t& out_hi) {
  uint32_t lo = 0, hi = n;
  int it = 0;
  uint32_t eq = 0;
  bool split = false;
  for (; it < iters && lo < hi; ++it) {
    const uint32_t mid = sa_mid(lo, hi, n);
    int tok[NC], tm;
    load_probe<NC>(corpus, nc, static_cast<uint32_t>(sa[mid]), lim, plen, M,
                   tok, tm);
    const int c = cmp_probe<NC>(tok, tm, pc, lim, plen, M);
    if (c < 0) {
      lo = mid + 1;
    } else if (c > 0) {
      hi = mid;
    } else {
      eq = mid;
      split = true;
      ++it;
      break;
    }
  }
  if (!split) {
    out_lo = out_hi = lo;
    return;
  }
  uint32_t llo = lo, lhi = eq, ulo = eq + 1, uhi = hi;
  for (; it < iters && (llo < lhi || ulo < uhi); ++it) {
    const bool dl = llo < lhi, du = ulo < uhi;
    const uint32_t ml = sa_mid(llo, lhi, n), mu = sa_mid(ulo, uhi, n);
    // (a finished bound loads nothing: zero columns, no column M)
    int tl[NC], tml, tu[NC], tmu;
    load_probe<NC>(corpus, nc, static_cast<uint32_t>(sa[ml]), dl ? lim : 0,
                   dl ? plen : 0, M, tl, tml);
    load_probe<NC>(corpus, nc, static_cast<uint32_t>(sa[mu]), du ? lim : 0,
                   du ? plen : 0, M, tu, tmu);
    if (dl) {
      if (cmp_probe<NC>(tl, tml, pc, lim, plen, M) < 0)
        llo = ml + 1;
      else
        lhi = ml;
    }
    if (du) {
      if (cmp_probe<NC>(tu, tmu, pc, lim, plen, M) <= 0)
        ulo = mu + 1;
      else
        uhi = mu;
    }
  }
  out_lo = llo;
  out_hi = ulo;
}

// Both bounds; patterns of at most 32 compared columns take the one-column
// path (half of the backoff lengths for 64-token tails).
template <int NC>
__device__ __forceinline__ void warp_bounds(
    const int32_t* __restrict__ sa, const int32_t* __restrict__ corpus,
    int64_t n, int iters, const int (&pc)[NC], int M, int64_t plen,
    int64_t& lower, int64_t& upper, int64_t nc = -1) {
  const int lim = plen < M ? (plen > 0 ? static_cast<int>(plen) : 0) : M;
  const uint32_t un = static_cast<uint32_t>(n);
  const uint32_t unc = static_cast<uint32_t>(nc < 0 ? n : nc);
  uint32_t a, b;
  if (NC > 1 && lim <= 32 && plen <= M) {
    const int pc1[1] = {pc[0]};
    warp_bounds_cols<1>(sa, corpus, un, unc, iters, pc1, M, lim, plen, a, b);
  } else {
    warp_bounds_cols<NC>(sa, corpus, un, unc, iters, pc, M, lim, plen, a, b);
  }
  lower = a;
  upper = b;
}

// search_interval: one warp per pattern row.
template <int NC>
__global__ void __launch_bounds__(kSWarps * 32)
    sa_search_warp_kernel(const int32_t* __restrict__ sa,
                          const int32_t* __restrict__ corpus, int64_t n,
                          const int32_t* __restrict__ pat, int M,
                          const int64_t* __restrict__ plen, int B, int iters,
                          int64_t* __restrict__ start,
                          int64_t* __restrict__ end) {
  const int row = blockIdx.x * kSWarps + warp_id();
  if (row >= B) return;  // warp-uniform
  const int lane = lane_id();
  int pc[NC];
#pragma unroll
  for (int k = 0; k < NC; ++k) {
    const int j = lane + 32 * k;
    pc[k] = j < M ? pat[static_cast<int64_t>(row) * M + j] : 0;
  }
  int64_t lo, hi;
  warp_bounds<NC>(sa, corpus, n, iters, pc, M, plen[row], lo, hi);
  if (lane == 0) {
    start[row] = lo;
    end[row] = hi;
  }
}

// suffix_match_backoff: one cluster of kSCG CTAs per row, one warp per
// pattern length; CTA 0 gathers the intervals and selects per cap.
template <int NC>
__global__ void __cluster_dims__(kSCG, 1, 1) __launch_bounds__(512)
    sa_backoff_cluster_kernel(const int32_t* __restrict__ sa,
                              const int32_t* __restrict__ corpus, int64_t n,
                              const int32_t* __restrict__ query, int Q,
                              const int64_t* __restrict__ qlen, int M,
                              const int64_t* __restrict__ caps, int C,
                              const uint8_t* __restrict__ row_mask, int iters,
                              int64_t* __restrict__ out_len,
                              int64_t* __restrict__ out_start,
                              int64_t* __restrict__ out_end) {
  cg::cluster_group cluster = cg::this_cluster();
  __shared__ long long s_res[2 * 16];   // this CTA's intervals, one per warp
  __shared__ long long s_all[2 * 128];  // CTA 0: every length's interval
  const int g = static_cast<int>(cluster.block_rank());
  const int b = blockIdx.x / kSCG;
  const int wpc = blockDim.x >> 5;
  const int warp = warp_id(), lane = lane_id();
  const bool active = !row_mask || row_mask[b];
  const int64_t ql = qlen[b];
  const int task = g * wpc + warp;
  if (task < M) {
    const int l = task + 1;  // pattern length
    int64_t lo = 0, hi = 0;
    if (active && l <= ql) {
      // pattern_l[j] = query[qlen - l + j] for j < l (the gather clamps
      // indices to the query width like the reference)
      int pc[NC];
      const int64_t o = ql - l;
#pragma unroll
      for (int k = 0; k < NC; ++k) {
        const int j = lane + 32 * k;
        const int64_t x = o + j;
        pc[k] = j < l ? query[static_cast<int64_t>(b) * Q + (x < Q ? x : Q - 1)] : 0;
      }
      warp_bounds<NC>(sa, corpus, n, iters, pc, M, l, lo, hi);
    }
    if (lane == 0) {
      s_res[2 * warp] = lo;
      s_res[2 * warp + 1] = hi;
    }
  }
  cluster.sync();  // every CTA's intervals are published
  if (g == 0) {
    for (int i = threadIdx.x; i < 2 * M; i += blockDim.x) {
      const int t = i >> 1;  // length index
      s_all[i] = *cluster.map_shared_rank(&s_res[2 * (t % wpc) + (i & 1)],
                                          t / wpc);
    }
  }
  cluster.sync();  // remote reads done; s_all visible to CTA 0
  if (g == 0) {
    for (int c = threadIdx.x; c < C; c += blockDim.x) {
      const int64_t cap = caps[c];
      int64_t best = 0;
      if (active) {
        for (int l = 1; l <= M; ++l)
          if (l <= cap && l <= ql && s_all[2 * l - 1] > s_all[2 * l - 2]) best = l;
      }
      const int64_t o = static_cast<int64_t>(b) * C + c;
      out_len[o] = best;
      out_start[o] = best > 0 ? s_all[2 * best - 2] : 0;
      out_end[o] = best > 0 ? s_all[2 * best - 1] : 0;
    }
  }
}

// Shard search: every (row, length) interval of the rows' tails over one
// shard's suffix array (the whole-corpus suffix array restricted to the
// suffixes that start in the shard, in the same order). One warp per
// (row, length); rows are packed as [tail (M tokens, oldest first), tail
// length, drafting flag] int32. The bounds count the shard's suffixes
// below the pattern (lower) and not above it (upper), so summing them over
// all shards gives the whole-corpus interval.
// Whether length l's bounds are needed by the per-cap selection, given the
// row's longest matching length lstar over all shards (sg_shard_longest
// summed with a MAX; M + 1 = every length): found lengths are then exactly
// 1..lstar, so cap c selects min(cap_c, lstar).
__device__ __forceinline__ bool length_needed(int l, int lstar, int M,
                                              const int64_t* caps, int C) {
  if (lstar > M) return true;
  for (int c = 0; c < C; ++c) {
    const int64_t want = caps[c] < lstar ? caps[c] : lstar;
    if (want == l) return true;
  }
  return false;
}

template <int NC>
__global__ void __launch_bounds__(kSWarps * 32)
    shard_bounds_kernel(const int32_t* __restrict__ sa, int64_t ns,
                        const int32_t* __restrict__ corpus, int64_t nc,
                        const int32_t* __restrict__ rows, int B, int W, int M,
                        int iters, const int32_t* __restrict__ lstar,
                        const int64_t* __restrict__ caps, int C,
                        int32_t* __restrict__ out) {
  const int64_t w = static_cast<int64_t>(blockIdx.x) * kSWarps + warp_id();
  if (w >= static_cast<int64_t>(B) * M) return;  // warp-uniform
  const int b = static_cast<int>(w / M), l = static_cast<int>(w % M) + 1;
  const int lane = lane_id();
  const int32_t* row = rows + static_cast<int64_t>(b) * W;
  const int tl = row[M], active = row[M + 1];
  int64_t lo = 0, hi = 0;
  const bool needed = !lstar || length_needed(l, lstar[b], M, caps, C);
  if (active && l <= tl && ns > 0 && needed) {
    int pc[NC];
    const int o = tl - l;
#pragma unroll
    for (int k = 0; k < NC; ++k) {
      const int j = lane + 32 * k;
      const int x = o + j;
      pc[k] = j < l ? row[x < M ? x : M - 1] : 0;
    }
    warp_bounds<NC>(sa, corpus, ns, sa_iters(ns), pc, M, l, lo, hi, nc);
  }
  (void)iters;
  if (lane == 0) {
    out[2 * w] = static_cast<int32_t>(lo);
    out[2 * w + 1] = static_cast<int32_t>(hi);
  }
}

// The longest l <= tail length with the tail's last l tokens starting some
// suffix of this shard (0: none), one block of kSWarps warps per packed
// row. Found lengths form a prefix 1..L (a match of l tokens at p leaves
// one of l - 1 tokens at p + 1) unless a pattern can match past the corpus
// end, where tokens read -1: rows whose tail holds a -1 report M + 1
// (every length needed). The search keeps found(a) and !found(z + 1) and
// probes kSWarps lengths of (a, z] at once per round (one per warp), so a
// 64-token tail takes two rounds. The row's longest over all shards is the
// MAX of the shards' values.
template <int NC>
__global__ void __launch_bounds__(kSWarps * 32)
    shard_longest_kernel(const int32_t* __restrict__ sa, int64_t ns,
                         const int32_t* __restrict__ corpus, int64_t nc,
                         const int32_t* __restrict__ rows, int W, int M,
                         int32_t* __restrict__ out) {
  __shared__ int s_found[kSWarps], s_len[kSWarps];
  __shared__ int s_a, s_z;
  const int b = blockIdx.x;
  const int warp = warp_id(), lane = lane_id();
  const int32_t* row = rows + static_cast<int64_t>(b) * W;
  const int tl = row[M] < M ? row[M] : M, active = row[M + 1];
  if (threadIdx.x < 32) {
    bool minus_one = false;
    for (int j = lane; j < tl; j += 32) minus_one |= row[j] == -1;
    minus_one = __any_sync(SG_FULL_MASK, minus_one);
    if (lane == 0) {
      s_a = 0;
      s_z = (active && tl > 0 && ns > 0) ? tl : 0;
      if (active && tl > 0 && minus_one) s_a = s_z = M + 1;
    }
  }
  __syncthreads();
  while (s_a < s_z) {  // block-uniform
    const int a = s_a, z = s_z, span = z - a;
    // probe lengths a < l_0 < ... <= z, spread over the span
    const int l = span <= kSWarps
                      ? (warp < span ? a + warp + 1 : 0)
                      : a + static_cast<int>((static_cast<int64_t>(warp + 1) *
                                              span + kSWarps - 1) / kSWarps);
    int found = 0;
    if (l > 0) {
      int pc[NC];
      const int o = tl - l;
#pragma unroll
      for (int k = 0; k < NC; ++k) {
        const int j = lane + 32 * k;
        pc[k] = j < l ? row[o + j] : 0;
      }
      int64_t lo, hi;
      warp_bounds<NC>(sa, corpus, ns, sa_iters(ns), pc, M, l, lo, hi, nc);
      found = hi > lo;
    }
    if (lane == 0) {
      s_found[warp] = found;
      s_len[warp] = l;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int na = a, nz = z;
      for (int w = 0; w < kSWarps; ++w) {
        if (s_len[w] == 0) continue;
        if (s_found[w]) {
          if (s_len[w] > na) na = s_len[w];
        } else if (s_len[w] - 1 < nz) {
          nz = s_len[w] - 1;
        }
      }
      s_a = na;
      s_z = nz;
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) out[b] = s_a;
}

template <int NC>
static int launch_search_warp(const int32_t* sa, const int32_t* corpus,
                              int64_t n, const int32_t* pattern, int batch,
                              int width, const int64_t* plen, int64_t* st,
                              int64_t* en, cudaStream_t stream) {
  const int64_t blocks = (static_cast<int64_t>(batch) + kSWarps - 1) / kSWarps;
  sa_search_warp_kernel<NC><<<static_cast<unsigned>(blocks), kSWarps * 32, 0,
                              stream>>>(sa, corpus, n, pattern, width, plen,
                                        batch, sa_iters(n), st, en);
  return check_launch();
}

template <int NC>
static int launch_backoff_cluster(const int32_t* sa, const int32_t* corpus,
                                  int64_t n, const int32_t* query, int batch,
                                  int qw, const int64_t* qlen, int M,
                                  const int64_t* caps, int C,
                                  const uint8_t* row_mask, int64_t* ol,
                                  int64_t* os, int64_t* oe,
                                  cudaStream_t stream) {
  const int wpc = (M + kSCG - 1) / kSCG;  // <= 16 for M <= 128
  sa_backoff_cluster_kernel<NC><<<batch * kSCG, wpc * 32, 0, stream>>>(
      sa, corpus, n, query, qw, qlen, M, caps, C, row_mask, sa_iters(n), ol,
      os, oe);
  return check_launch();
}

}  // namespace sg

using namespace sg;

extern "C" int sg_sa_search(const int32_t* sa, const int32_t* corpus,
                            int64_t n, const int32_t* pattern, int32_t batch,
                            int32_t width, const int64_t* pattern_len,
                            int64_t* out_start, int64_t* out_end,
                            sg_stream_t stream) {
  sg::NvtxScope nvtx_range("sg_sa_search");
  if (n < 1 || batch < 0 || width < 1) return SG_ERR_INVALID;
  if (batch == 0) return SG_OK;
  if (!sa || !corpus || !pattern || !pattern_len || !out_start || !out_end)
    return SG_ERR_INVALID;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (width <= 32 * kSMaxCols) {
    if (width <= 32)
      return launch_search_warp<1>(sa, corpus, n, pattern, batch, width,
                                   pattern_len, out_start, out_end, st);
    if (width <= 64)
      return launch_search_warp<2>(sa, corpus, n, pattern, batch, width,
                                   pattern_len, out_start, out_end, st);
    return launch_search_warp<4>(sa, corpus, n, pattern, batch, width,
                                 pattern_len, out_start, out_end, st);
  }
  const int th = 64;
  const size_t smem = static_cast<size_t>(th) * width * 4;
  static int cache[64] = {0};
  int rc = ensure_dyn_smem(sa_search_kernel, smem, cache);
  if (rc != SG_OK) return rc;
  sa_search_kernel<<<(2 * batch + th - 1) / th, th, smem,
                     reinterpret_cast<cudaStream_t>(stream)>>>(
      sa, corpus, n, pattern, width, pattern_len, batch, sa_iters(n),
      out_start, out_end);
  return check_launch();
}

extern "C" int sg_suffix_match_backoff(
    const int32_t* sa, const int32_t* corpus, int64_t n, const int32_t* query,
    int32_t batch, int32_t query_width, const int64_t* query_len,
    int32_t max_len, const int64_t* caps, int32_t num_caps,
    const uint8_t* row_mask, int64_t* out_len, int64_t* out_start,
    int64_t* out_end, sg_stream_t stream) {
  sg::NvtxScope nvtx_range("sg_suffix_match_backoff");
  if (n < 1 || batch < 0 || query_width < 1 || max_len < 1 || num_caps < 1)
    return SG_ERR_INVALID;
  if (batch == 0) return SG_OK;
  if (!sa || !corpus || !query || !query_len || !caps || !out_len ||
      !out_start || !out_end)
    return SG_ERR_INVALID;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (max_len <= 32 * kSMaxCols && static_cast<int64_t>(batch) * kSCG <= INT32_MAX) {
    if (max_len <= 32)
      return launch_backoff_cluster<1>(sa, corpus, n, query, batch,
                                       query_width, query_len, max_len, caps,
                                       num_caps, row_mask, out_len, out_start,
                                       out_end, st);
    if (max_len <= 64)
      return launch_backoff_cluster<2>(sa, corpus, n, query, batch,
                                       query_width, query_len, max_len, caps,
                                       num_caps, row_mask, out_len, out_start,
                                       out_end, st);
    return launch_backoff_cluster<4>(sa, corpus, n, query, batch,
                                     query_width, query_len, max_len, caps,
                                     num_caps, row_mask, out_len, out_start,
                                     out_end, st);
  }
  const int th = 2 * max_len < 1024 ? ((2 * max_len + 31) & ~31) : 1024;
  const size_t smem = 4 * static_cast<size_t>((query_width + 1) & ~1) +
                      16 * static_cast<size_t>(max_len);
  static int cache[64] = {0};
  int rc = ensure_dyn_smem(sa_backoff_kernel, smem, cache);
  if (rc != SG_OK) return rc;
  sa_backoff_kernel<<<batch, th, smem,
                      reinterpret_cast<cudaStream_t>(stream)>>>(
      sa, corpus, n, query, query_width, query_len, max_len, caps, num_caps,
      row_mask, sa_iters(n), out_len, out_start, out_end);
  return check_launch();
}

extern "C" int sg_shard_longest(const int32_t* shard_sa, int64_t shard_n,
                                const int32_t* corpus, int64_t corpus_n,
                                const int32_t* rows, int32_t batch,
                                int32_t max_len, int32_t* out_len,
                                sg_stream_t stream) {
  sg::NvtxScope nvtx_range("sg_shard_longest");
  if (shard_n < 0 || corpus_n < 1 || corpus_n > INT32_MAX ||
      shard_n > corpus_n || batch < 0 || max_len < 1 ||
      max_len > 32 * kSMaxCols)
    return SG_ERR_INVALID;
  if (batch == 0) return SG_OK;
  if ((shard_n > 0 && !shard_sa) || !corpus || !rows || !out_len)
    return SG_ERR_INVALID;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const unsigned blocks = static_cast<unsigned>(batch);
  const int W = max_len + 2;
  if (max_len <= 32)
    shard_longest_kernel<1><<<blocks, kSWarps * 32, 0, st>>>(
        shard_sa, shard_n, corpus, corpus_n, rows, W, max_len, out_len);
  else if (max_len <= 64)
    shard_longest_kernel<2><<<blocks, kSWarps * 32, 0, st>>>(
        shard_sa, shard_n, corpus, corpus_n, rows, W, max_len, out_len);
  else
    shard_longest_kernel<4><<<blocks, kSWarps * 32, 0, st>>>(
        shard_sa, shard_n, corpus, corpus_n, rows, W, max_len, out_len);
  return check_launch();
}

extern "C" int sg_shard_bounds(const int32_t* shard_sa, int64_t shard_n,
                               const int32_t* corpus, int64_t corpus_n,
                               const int32_t* rows, int32_t batch,
                               int32_t max_len, const int32_t* longest,
                               const int64_t* caps, int32_t num_caps,
                               int32_t* out_bounds, sg_stream_t stream) {
  sg::NvtxScope nvtx_range("sg_shard_bounds");
  if (shard_n < 0 || corpus_n < 1 || corpus_n > INT32_MAX ||
      shard_n > corpus_n || batch < 0 || max_len < 1 ||
      max_len > 32 * kSMaxCols || (longest && (!caps || num_caps < 1)))
    return SG_ERR_INVALID;
  if (batch == 0) return SG_OK;
  if ((shard_n > 0 && !shard_sa) || !corpus || !rows || !out_bounds)
    return SG_ERR_INVALID;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int64_t warps = static_cast<int64_t>(batch) * max_len;
  const unsigned blocks = static_cast<unsigned>((warps + kSWarps - 1) / kSWarps);
  const int W = max_len + 2;
  const int it = sa_iters(shard_n > 0 ? shard_n : 1);
  if (max_len <= 32)
    shard_bounds_kernel<1><<<blocks, kSWarps * 32, 0, st>>>(
        shard_sa, shard_n, corpus, corpus_n, rows, batch, W, max_len, it,
        longest, caps, num_caps, out_bounds);
  else if (max_len <= 64)
    shard_bounds_kernel<2><<<blocks, kSWarps * 32, 0, st>>>(
        shard_sa, shard_n, corpus, corpus_n, rows, batch, W, max_len, it,
        longest, caps, num_caps, out_bounds);
  else
    shard_bounds_kernel<4><<<blocks, kSWarps * 32, 0, st>>>(
        shard_sa, shard_n, corpus, corpus_n, rows, batch, W, max_len, it,
        longest, caps, num_caps, out_bounds);
  return check_launch();
}
