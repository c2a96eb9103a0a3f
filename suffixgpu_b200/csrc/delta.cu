// Delta-buffer brute-force match for sm_100a.
//
// Reproduces GlobalIndex._delta_match_backoff (suffix_gpu/global_index.py:
// 465-546): for each query row, match_back over delta positions
// i in [0, delta_capacity] against the newest-first tail (fill -3), masked
// to i <= delta_len; lo = min(max_i mb, cap) per cap; the earliest R
// positions with mb >= lo (lo > 0), returned as start positions
// max(i - lo, 0), zero-padded, count clamped to R.
//
// The reference materialises mb as [B, delta_capacity + 1] int32 (16.8 MB
// for 64 rows x 65537) and sorts position keys per cap. Here one CTA per row
// streams the delta through shared memory in 4096-position tiles (plus a
// halo of max_len tokens) twice: pass 1 keeps only the maximum; pass 2
// appends, per warp, the positions whose match reaches the smallest cap
// length to an ordered list, and one warp per cap walks the lists in order,
// stopping at R. delta_len is read from device memory (no host sync).
#include <cuda_runtime.h>

#include "sg_common.cuh"

namespace sg {

constexpr int kDThreads = 256;
constexpr int kDWarps = kDThreads / 32;
constexpr int kDTile = 4096;
constexpr int kDSeg = kDTile / kDWarps;  // positions per warp per tile
constexpr int kDMaxCaps = 16;

struct DeltaSmem {
  int* pat;   // [M]
  int* tile;  // [M + kDTile]: tile[j] = delta[p0 - M + j] (-1 before 0)
  int* lpos;  // [kDTile] per-warp ordered hit positions (warp w: w*kDSeg..)
  int* lmb;   // [kDTile] their match lengths
};

// match_back at position i (tile-relative k = i - p0), given tok(i-1) ==
// pat[0] already checked.
__device__ __forceinline__ int delta_extend(const DeltaSmem& s, int k,
                                            int M) {
  int m = 1;
  for (int t = 1; t < M; ++t) {
    if (s.tile[M + k - 1 - t] != s.pat[t]) break;
    ++m;
  }
  return m;
}

__device__ void load_tile(const DeltaSmem& s, const int32_t* delta,
                          int64_t dcap, int64_t p0, int M) {
  for (int j = threadIdx.x; j < M + kDTile; j += kDThreads) {
    const int64_t y = p0 - M + j;
    s.tile[j] = (y >= 0 && y < dcap) ? delta[y] : -1;
  }
}

__global__ void __launch_bounds__(kDThreads)
    delta_match_kernel(const int32_t* __restrict__ delta, int64_t dcap,
                       const int64_t* __restrict__ dlen_dev,
                       const int32_t* __restrict__ query, int Q,
                       const int64_t* __restrict__ qlen, int M,
                       const int64_t* __restrict__ caps, int C, int R,
                       const uint8_t* __restrict__ row_mask,
                       int64_t* __restrict__ out_len,
                       int64_t* __restrict__ out_pos,
                       int64_t* __restrict__ out_cnt) {
  extern __shared__ int smem_d[];
  DeltaSmem s;
  s.pat = smem_d;
  s.tile = s.pat + ((M + 3) & ~3);
  s.lpos = s.tile + ((M + kDTile + 3) & ~3);
  s.lmb = s.lpos + kDTile;
  __shared__ long long s_lo[kDMaxCaps];
  __shared__ int s_cnt[kDMaxCaps];
  __shared__ int s_wlen[kDWarps];
  __shared__ int s_done;

  const int b = blockIdx.x;
  const int t = threadIdx.x, warp = warp_id(), lane = lane_id();
  const unsigned lt_mask = (1u << lane) - 1u;
  const bool active = !row_mask || row_mask[b];
  const int64_t ql = qlen[b];
  int64_t dlen = *dlen_dev;
  if (dlen > dcap) dlen = dcap;  // valid end positions i <= dlen <= dcap
  // pattern, newest-first, -3 before the query start
  for (int i = t; i < M; i += kDThreads) {
    const int64_t x = ql - 1 - i;
    const int64_t xc = x < 0 ? 0 : (x > Q - 1 ? Q - 1 : x);
    s.pat[i] = x >= 0 ? query[static_cast<int64_t>(b) * Q + xc] : -3;
  }
  __syncthreads();
  const int pat0 = s.pat[0];
  const int64_t n_pos = active && dlen >= 0 ? dlen + 1 : 0;  // i in [0, dlen]

  // ---- pass 1: longest match ---------------------------------------------
  int best = 0;
  for (int64_t p0 = 0; p0 < n_pos; p0 += kDTile) {
    load_tile(s, delta, dcap, p0, M);
    __syncthreads();
    for (int k = t; k < kDTile; k += kDThreads) {
      if (p0 + k >= n_pos) break;
      if (s.tile[M + k - 1] == pat0) best = max(best, delta_extend(s, k, M));
    }
    best = __reduce_max_sync(SG_FULL_MASK, best);
    const int blk = __syncthreads_or(best == M);
    if (blk) {
      best = M;
      break;
    }
  }
  {
    __shared__ int s_best[kDWarps];
    if (lane == 0) s_best[warp] = best;
    __syncthreads();
    int bb = 0;
    for (int w = 0; w < kDWarps; ++w) bb = max(bb, s_best[w]);
    best = bb;
  }
  // per-cap lengths; the smallest positive one gates pass 2
  int lo_min = 0;
  for (int c = 0; c < C; ++c) {
    const int64_t cp = caps[c];
    const int64_t lo = best < cp ? best : cp;  // min(lo_full, cap)
    if (t == 0) {
      s_lo[c] = lo;
      s_cnt[c] = 0;
    }
    if (lo > 0 && (lo_min == 0 || lo < lo_min)) lo_min = static_cast<int>(lo);
  }
  if (t == 0) s_done = 0;
  __syncthreads();

  // ---- pass 2: earliest R occurrences per cap ----------------------------
  if (lo_min > 0) {
    for (int64_t p0 = 0; p0 < n_pos; p0 += kDTile) {
      load_tile(s, delta, dcap, p0, M);
      __syncthreads();
      // warp w: positions [w*kDSeg, (w+1)*kDSeg) of the tile, in order
      int nh = 0;
      for (int k0 = warp * kDSeg; k0 < (warp + 1) * kDSeg; k0 += 32) {
        const int k = k0 + lane;
        int m = 0;
        if (p0 + k < n_pos && s.tile[M + k - 1] == pat0)
          m = delta_extend(s, k, M);
        const bool hit = m >= lo_min;
        const unsigned bal = __ballot_sync(SG_FULL_MASK, hit);
        if (hit) {
          const int at = warp * kDSeg + nh + __popc(bal & lt_mask);
          s.lpos[at] = k;
          s.lmb[at] = m;
        }
        nh += __popc(bal);
      }
      if (lane == 0) s_wlen[warp] = nh;
      __syncthreads();
      // warp c appends cap c's hits in position order
      for (int c = warp; c < C; c += kDWarps) {
        const int lo = s_lo[c] > 0 ? static_cast<int>(s_lo[c]) : 0;
        int cnt = s_cnt[c];
        if (lo <= 0 || cnt >= R) continue;
        int64_t* op = out_pos + (static_cast<int64_t>(b) * C + c) * R;
        for (int w = 0; w < kDWarps && cnt < R; ++w) {
          const int len = s_wlen[w];
          for (int i0 = 0; i0 < len && cnt < R; i0 += 32) {
            const int i = i0 + lane;
            const int at = w * kDSeg + i;
            const bool hit = i < len && s.lmb[at] >= lo;
            const unsigned bal = __ballot_sync(SG_FULL_MASK, hit);
            const int r = cnt + __popc(bal & lt_mask);
            if (hit && r < R) {
              const int64_t end = p0 + s.lpos[at];
              op[r] = end - lo > 0 ? end - lo : 0;
            }
            cnt += __popc(bal);
          }
        }
        if (lane == 0) s_cnt[c] = cnt < R ? cnt : R;
      }
      __syncthreads();
      int all = 1;
      for (int c = 0; c < C; ++c) all &= (s_lo[c] <= 0 || s_cnt[c] >= R);
      if (all) break;  // uniform: every thread reads the same smem values
      __syncthreads();
    }
  }
  __syncthreads();
  // outputs: lengths, counts, zero padding
  for (int c = 0; c < C; ++c) {
    const int cnt = s_cnt[c];
    int64_t* op = out_pos + (static_cast<int64_t>(b) * C + c) * R;
    for (int r = cnt + t; r < R; r += kDThreads) op[r] = 0;
    if (t == 0) {
      out_len[static_cast<int64_t>(b) * C + c] = s_lo[c];
      out_cnt[static_cast<int64_t>(b) * C + c] = cnt;
    }
  }
}

}  // namespace sg

using namespace sg;

extern "C" int sg_delta_match_backoff(
    const int32_t* delta, int64_t delta_capacity, const int64_t* delta_len,
    const int32_t* query, int32_t batch, int32_t query_width,
    const int64_t* query_len, int32_t max_len, const int64_t* caps,
    int32_t num_caps, int32_t max_occ, const uint8_t* row_mask,
    int64_t* out_len, int64_t* out_pos, int64_t* out_cnt,
    sg_stream_t stream) {
  if (delta_capacity < 1 || batch < 0 || query_width < 1 || max_len < 1 ||
      num_caps < 1 || num_caps > kDMaxCaps || max_occ < 1)
    return SG_ERR_INVALID;
  if (batch == 0) return SG_OK;
  if (!delta || !delta_len || !query || !query_len || !caps || !out_len ||
      !out_pos || !out_cnt)
    return SG_ERR_INVALID;
  const size_t smem = 4 * (static_cast<size_t>((max_len + 3) & ~3) +
                           ((max_len + kDTile + 3) & ~3) + 2 * kDTile);
  static int cache[64] = {0};
  int rc = ensure_dyn_smem(delta_match_kernel, smem, cache);
  if (rc != SG_OK) return rc;
  delta_match_kernel<<<batch, kDThreads, smem,
                       reinterpret_cast<cudaStream_t>(stream)>>>(
      delta, delta_capacity, delta_len, query, query_width, query_len,
      max_len, caps, num_caps, max_occ, row_mask, out_len, out_pos, out_cnt);
  return check_launch();
}
