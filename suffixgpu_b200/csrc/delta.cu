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
// for 64 rows x 65537) and sorts position keys per cap. Here each row is
// one thread-block cluster of 8 CTAs; CTA g holds the g-th eighth of the
// valid positions (plus a halo of max_len tokens) in shared memory and
// scans it once: per warp an ordered list of the positions whose previous
// token is the pattern's newest one, each extended to its match length,
// and per warp #{hits with match >= L}. The CTAs exchange their longest
// match and then, per cap, their qualifying counts through distributed
// shared memory, so each CTA writes its earliest hits at the right output
// offset directly. delta_len is read from device memory (no host sync).
// Capacities whose eighth does not fit in shared memory use a one-CTA-per-
// row kernel that streams the delta in tiles twice (longest match, then
// the ordered occurrences).
#include <cooperative_groups.h>
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


// ---------------------------------------------------------------------------
// Cluster kernel: one cluster of kCG CTAs per row, one pass over the delta.
// ---------------------------------------------------------------------------
namespace cg = cooperative_groups;

constexpr int kCG = 8;             // CTAs per row (cluster size)
constexpr int kCChunkMax = 8256;   // positions per CTA (multiple of 32)
constexpr int kCMaxLen = 255;      // match lengths are packed into 8 bits

struct DeltaClusterLayout {
  int mp, tile, hits, pat, whist, total;  // offsets / sizes in ints
  __host__ __device__ explicit DeltaClusterLayout(int M) {
    mp = (M + 3) & ~3;
    tile = 0;                              // [mp + kCChunkMax + 4]
    hits = tile + mp + kCChunkMax + 4;     // [kCChunkMax]
    pat = hits + kCChunkMax;               // [mp]
    whist = pat + mp;                      // [kDWarps][M + 2]
    total = whist + (M + 2) * kDWarps;
  }
};

__global__ void __cluster_dims__(kCG, 1, 1) __launch_bounds__(kDThreads)
    delta_cluster_kernel(const int32_t* __restrict__ delta, int64_t dcap,
                         const int64_t* __restrict__ dlen_dev,
                         const int32_t* __restrict__ query, int Q,
                         const int64_t* __restrict__ qlen, int M,
                         const int64_t* __restrict__ caps, int C, int R,
                         const uint8_t* __restrict__ row_mask,
                         int64_t* __restrict__ out_len,
                         int64_t* __restrict__ out_pos,
                         int64_t* __restrict__ out_cnt) {
  cg::cluster_group cluster = cg::this_cluster();
  extern __shared__ __align__(16) int smc[];
  const DeltaClusterLayout lay(M);
  int* tile = smc + lay.tile;
  int* hits = smc + lay.hits;
  int* pat = smc + lay.pat;
  int* whist = smc + lay.whist;
  __shared__ int s_max;                   // this CTA's longest match
  __shared__ int s_wmax[kDWarps];
  __shared__ int s_cnt[kDMaxCaps];        // this CTA's qualifying hits
  __shared__ int s_off[kDMaxCaps], s_tot[kDMaxCaps];

  const int g = static_cast<int>(cluster.block_rank());
  const int b = blockIdx.x / kCG;
  const int t = threadIdx.x, warp = warp_id(), lane = lane_id();
  const unsigned lt_mask = (1u << lane) - 1u;
  const int hs = M + 2;
  const bool active = !row_mask || row_mask[b];
  const int64_t ql = qlen[b];
  int64_t dlen = *dlen_dev;
  if (dlen > dcap) dlen = dcap;  // valid end positions i <= dlen <= dcap
  // valid positions [0, n_pos); the host guarantees n_pos <= kCG * kCChunkMax
  const int n_pos = active && dlen >= 0 ? static_cast<int>(dlen + 1) : 0;
  const int ch = ((n_pos + kCG - 1) / kCG + 31) & ~31;
  const int p_begin = g * ch;
  const int p_end = min(p_begin + ch, n_pos);
  const int len = p_end > p_begin ? p_end - p_begin : 0;
  const int start = p_begin - lay.mp;  // delta index of tile[0]

  // pattern, newest-first, -3 before the query start; empty histograms
  for (int i = t; i < M; i += kDThreads) {
    const int64_t x = ql - 1 - i;
    const int64_t xc = x < 0 ? 0 : (x > Q - 1 ? Q - 1 : x);
    pat[i] = x >= 0 ? query[static_cast<int64_t>(b) * Q + xc] : -3;
  }
  for (int i = t; i < hs * kDWarps; i += kDThreads) whist[i] = 0;
  // tokens [start, p_end - 1) with the halo; -1 outside the buffer
  const int ntok = len > 0 ? lay.mp + len : 0;
  const int words = (ntok + 3) >> 2;
  const bool vec = (reinterpret_cast<uintptr_t>(delta) & 15) == 0;
#pragma unroll 4
  for (int wi = t; wi < words; wi += kDThreads) {
    const int64_t y0 = static_cast<int64_t>(start) + 4 * wi;
    int4 v;
    if (vec && y0 >= 0 && y0 + 4 <= dcap) {
      v = *reinterpret_cast<const int4*>(delta + y0);
    } else {
      v.x = (y0 >= 0 && y0 < dcap) ? delta[y0] : -1;
      v.y = (y0 + 1 >= 0 && y0 + 1 < dcap) ? delta[y0 + 1] : -1;
      v.z = (y0 + 2 >= 0 && y0 + 2 < dcap) ? delta[y0 + 2] : -1;
      v.w = (y0 + 3 >= 0 && y0 + 3 < dcap) ? delta[y0 + 3] : -1;
    }
    reinterpret_cast<int4*>(tile)[wi] = v;
  }
  __syncthreads();

  // ---- scan: ordered hit list per warp segment ----------------------------
  const int sw = ch / kDWarps;  // multiple of 4
  const int ws0 = p_begin + warp * sw;
  const int ws1 = min(ws0 + sw, p_end);
  int* my_hits = hits + warp * sw;
  int* my_ge = whist + warp * hs;
  int nh = 0;
  const int pt0 = pat[0];
  {
    const int4* tok4 = reinterpret_cast<const int4*>(tile);
    // token ws0 - 1 (tile index >= mp - 1; the halo holds -1 before 0)
    uint32_t carry = ws0 < ws1 ? (tile[ws0 - 1 - start] == pt0) : 0u;
    for (int c0 = ws0; c0 < ws1; c0 += 1024) {
      // lane l: tokens / end positions [c0 + 32 l, c0 + 32 l + 32); the 8
      // vector loads go in a lane-rotated order (no bank conflicts)
      const int tw = ((c0 - start) >> 2) + 8 * lane;
      uint32_t eq = 0;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int j = (k + lane) & 7;
        if (tw + j < words) {
          const int4 v = tok4[tw + j];
          const uint32_t bits = static_cast<uint32_t>(v.x == pt0) |
                                (static_cast<uint32_t>(v.y == pt0) << 1) |
                                (static_cast<uint32_t>(v.z == pt0) << 2) |
                                (static_cast<uint32_t>(v.w == pt0) << 3);
          eq |= bits << (4 * j);
        }
      }
      const uint32_t up = __shfl_up_sync(SG_FULL_MASK, eq, 1);
      uint32_t hm = (eq << 1) | (lane == 0 ? carry : (up >> 31));
      carry = __shfl_sync(SG_FULL_MASK, eq, 31) >> 31;
      const int p0 = c0 + 32 * lane;
      const int nvalid = ws1 - p0;
      if (nvalid < 32) hm &= nvalid <= 0 ? 0u : ((1u << nvalid) - 1u);
      if (__ballot_sync(SG_FULL_MASK, hm != 0) == 0) continue;
      const int c = __popc(hm);
      int inc = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int x = __shfl_up_sync(SG_FULL_MASK, inc, o);
        if (lane >= o) inc += x;
      }
      int pos = nh + inc - c;
      while (hm) {
        const int bit = __ffs(hm) - 1;
        hm &= hm - 1;
        my_hits[pos++] = p0 + bit;
      }
      nh += __shfl_sync(SG_FULL_MASK, inc, 31);
    }
  }
  __syncwarp();
  // extend every hit; entries become (position - p_begin) << 8 | length
  int h1 = 0, h2 = 0, mmax = 0;
  for (int i = lane; i < nh; i += 32) {
    const int p = my_hits[i];
    const int* tp = tile + (p - 1 - start);  // token p - 1
    int m = 1;
    while (m < M && tp[-m] == pat[m]) ++m;
    h1 += m == 1;
    h2 += m == 2;
    if (m > 2) atomicAdd(&my_ge[m], 1);
    mmax = max(mmax, m);
    my_hits[i] = ((p - p_begin) << 8) | m;
  }
  h1 = warp_sum(h1);
  h2 = warp_sum(h2);
  mmax = __reduce_max_sync(SG_FULL_MASK, mmax);
  __syncwarp();
  {
    // histogram -> #{hits with match >= L}, suffix sums from the top
    int above = 0;
    for (int L0 = ((M - 1) & ~31) + 1; L0 >= 1; L0 -= 32) {
      const int Lx = L0 + lane;
      int v = Lx <= M ? my_ge[Lx] : 0;
      v += Lx == 1 ? h1 : (Lx == 2 ? h2 : 0);
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_down_sync(SG_FULL_MASK, v, o);
        if (lane + o < 32) v += u;
      }
      v += above;
      above = __shfl_sync(SG_FULL_MASK, v, 0);
      if (Lx <= M) my_ge[Lx] = v;
    }
    if (lane == 0) {
      my_ge[M + 1] = 0;
      s_wmax[warp] = mmax;
    }
  }
  __syncthreads();
  if (t == 0) {
    int mx = 0;
    for (int w = 0; w < kDWarps; ++w) mx = max(mx, s_wmax[w]);
    s_max = mx;
  }
  cluster.sync();  // every CTA's s_max is published
  int best = 0;
#pragma unroll
  for (int r = 0; r < kCG; ++r)
    best = max(best, *cluster.map_shared_rank(&s_max, r));
  // per cap: lo = min(best, cap); this CTA's hits with match >= lo
  if (t < C) {
    const int64_t cp = caps[t];
    const int64_t lo = best < cp ? best : cp;
    int k = 0;
    if (lo > 0)
      for (int w = 0; w < kDWarps; ++w) k += whist[w * hs + static_cast<int>(lo)];
    s_cnt[t] = k;
  }
  cluster.sync();  // every CTA's counts are published
  if (t < C) {
    int off = 0, tot = 0;
    for (int r = 0; r < kCG; ++r) {
      const int k = *cluster.map_shared_rank(&s_cnt[t], r);
      if (r < g) off += k;
      tot += k;
    }
    s_off[t] = off;
    s_tot[t] = tot;
  }
  cluster.sync();  // remote reads done (no CTA exits while being read)

  // ---- earliest R occurrences per cap, written at this CTA's offset -------
  for (int c = 0; c < C; ++c) {
    const int64_t cp = caps[c];
    const int lo = best < cp ? best : static_cast<int>(cp > 0 ? cp : 0);
    if (lo <= 0) continue;
    int off = s_off[c];
    for (int w = 0; w < warp; ++w) off += whist[w * hs + lo];
    const int k = my_ge[lo];
    if (k == 0 || off >= R) continue;
    int64_t* op = out_pos + (static_cast<int64_t>(b) * C + c) * R;
    int got = 0;
    for (int i0 = 0; i0 < nh && got < k && off + got < R; i0 += 32) {
      const int i = i0 + lane;
      const int e = i < nh ? my_hits[i] : 0;
      const bool hit = i < nh && (e & 0xff) >= lo;
      const unsigned bal = __ballot_sync(SG_FULL_MASK, hit);
      const int r = off + got + __popc(bal & lt_mask);
      if (hit && r < R) {
        const int64_t end = p_begin + (e >> 8);
        op[r] = end - lo > 0 ? end - lo : 0;
      }
      got += __popc(bal);
    }
  }
  // lengths, counts and zero padding (last CTA of the cluster)
  if (g == kCG - 1) {
    for (int c = 0; c < C; ++c) {
      const int64_t cp = caps[c];
      const int64_t lo = best < cp ? best : cp;
      const int cnt = lo > 0 ? min(s_tot[c], R) : 0;
      int64_t* op = out_pos + (static_cast<int64_t>(b) * C + c) * R;
      for (int r = cnt + t; r < R; r += kDThreads) op[r] = 0;
      if (t == 0) {
        out_len[static_cast<int64_t>(b) * C + c] = lo;
        out_cnt[static_cast<int64_t>(b) * C + c] = cnt;
      }
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
  sg::NvtxScope nvtx_range("sg_delta_match_backoff");
  if (delta_capacity < 1 || batch < 0 || query_width < 1 || max_len < 1 ||
      num_caps < 1 || num_caps > kDMaxCaps || max_occ < 1)
    return SG_ERR_INVALID;
  if (batch == 0) return SG_OK;
  if (!delta || !delta_len || !query || !query_len || !caps || !out_len ||
      !out_pos || !out_cnt)
    return SG_ERR_INVALID;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // one pass per row on a cluster when an eighth of the positions (and the
  // packed 8-bit lengths) fit
  const int64_t chunk = ((delta_capacity + 1 + kCG - 1) / kCG + 31) & ~int64_t(31);
  if (chunk <= kCChunkMax && max_len <= kCMaxLen &&
      static_cast<int64_t>(batch) * kCG <= INT32_MAX) {
    const size_t smem = 4 * static_cast<size_t>(DeltaClusterLayout(max_len).total);
    static int ccache[64] = {0};
    int rc = ensure_dyn_smem(delta_cluster_kernel, smem, ccache);
    if (rc == SG_OK) {
      delta_cluster_kernel<<<batch * kCG, kDThreads, smem, st>>>(
          delta, delta_capacity, delta_len, query, query_width, query_len,
          max_len, caps, num_caps, max_occ, row_mask, out_len, out_pos,
          out_cnt);
      return check_launch();
    }
    if (rc != SG_ERR_UNSUPPORTED) return rc;
  }
  const size_t smem = 4 * (static_cast<size_t>((max_len + 3) & ~3) +
                           ((max_len + kDTile + 3) & ~3) + 2 * kDTile);
  static int cache[64] = {0};
  int rc = ensure_dyn_smem(delta_match_kernel, smem, cache);
  if (rc != SG_OK) return rc;
  delta_match_kernel<<<batch, kDThreads, smem, st>>>(
      delta, delta_capacity, delta_len, query, query_width, query_len,
      max_len, caps, num_caps, max_occ, row_mask, out_len, out_pos, out_cnt);
  return check_launch();
}
