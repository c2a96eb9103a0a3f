// Suffix-array interval search for sm_100a.
//
// Reproduces suffix_gpu/sa_search.py: search_interval (:66-107, Triton
// _sa_search_kernel triton_kernels.py:56-94) and suffix_match_backoff
// (:110-163). The lower bound (first suffix with cmp >= 0) and the upper
// bound (first with cmp > 0) run the reference's fixed
// ceil(log2(n + 1))-iteration loop with the same midpoint rule and the
// same comparator (_cmp_pattern, :25-63: corpus tokens past the end read
// -1, pattern positions past its length always match), so the bounds are
// identical to the reference's for any SA. The backoff variant searches
// every suffix length 1..M of each row's tail in one block (one thread per
// length and bound, tail in shared memory) and keeps, per cap, the longest
// found length <= cap.
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

}  // namespace sg

using namespace sg;

extern "C" int sg_sa_search(const int32_t* sa, const int32_t* corpus,
                            int64_t n, const int32_t* pattern, int32_t batch,
                            int32_t width, const int64_t* pattern_len,
                            int64_t* out_start, int64_t* out_end,
                            sg_stream_t stream) {
  if (n < 1 || batch < 0 || width < 1) return SG_ERR_INVALID;
  if (batch == 0) return SG_OK;
  if (!sa || !corpus || !pattern || !pattern_len || !out_start || !out_end)
    return SG_ERR_INVALID;
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
  if (n < 1 || batch < 0 || query_width < 1 || max_len < 1 || num_caps < 1)
    return SG_ERR_INVALID;
  if (batch == 0) return SG_OK;
  if (!sa || !corpus || !query || !query_len || !caps || !out_len ||
      !out_start || !out_end)
    return SG_ERR_INVALID;
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
