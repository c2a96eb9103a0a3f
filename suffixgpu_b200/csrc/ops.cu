// Standalone operator kernels: the reference's Triton operator layer
// (suffix_gpu/triton_kernels.py:259-402) rebuilt for sm_100a. The fused
// draft kernels do not call these; they serve the operator-level API
// (update_state, GlobalIndex.expand, expand_chain, ...) and its tests.
#include <cuda_runtime.h>

#include "sg_common.cuh"
#include "sg_vote.cuh"

namespace sg {

// ---------------------------------------------------------------------------
// scatter_append (triton_kernels.py:245-256, proposer.py:166-188)
// ---------------------------------------------------------------------------
__global__ void scatter_append_kernel(int32_t* tok, long long stride, int B,
                                      int S, const int32_t* base,
                                      const int32_t* valid_count,
                                      const int32_t* sampled, int T,
                                      int32_t* new_counts) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  const long long bs = base[b];
  long long cnt = 0;
  const int32_t* srow = sampled + static_cast<long long>(b) * T;
  if (valid_count) {
    cnt = valid_count[b];
  } else {
    for (int j = 0; j < T; ++j) cnt += srow[j] != -1;
  }
  int32_t* row = tok + static_cast<long long>(b) * stride;
  for (int j = 0; j < T; ++j) {
    const long long pos = bs + j;
    const int v = srow[j];
    if (j < cnt && v != -1 && pos < S && pos >= 0) row[pos] = v;
  }
  new_counts[b] = static_cast<int32_t>(bs + cnt);
}

// ---------------------------------------------------------------------------
// match_back (triton_kernels.py:39-54, 259-281)
// ---------------------------------------------------------------------------
constexpr int kMbTile = 1024;

__global__ void match_back_kernel(const int32_t* src, long long stride,
                                  long long n_src, const int32_t* pat, int P,
                                  long long n_out, int32_t* out) {
  extern __shared__ int tile[];  // [P + kMbTile]
  const int b = blockIdx.y;
  const long long i0 = static_cast<long long>(blockIdx.x) * kMbTile;
  const int32_t* s = src + (stride ? static_cast<long long>(b) * stride : 0);
  const int32_t* pb = pat + static_cast<long long>(b) * P;
  // tile[j] = src[i0 - P + j] for j < P + kMbTile  (-1 before the start)
  for (int j = threadIdx.x; j < P + kMbTile; j += blockDim.x) {
    const long long y = i0 - P + j;
    tile[j] = (y >= 0 && y < n_src) ? __ldg(s + y) : -1;
  }
  __syncthreads();
  const int p0 = __ldg(pb);
  for (int k = threadIdx.x; k < kMbTile; k += blockDim.x) {
    const long long i = i0 + k;
    if (i >= n_out) break;
    int m = 0;
    // tok[i - 1 - t] = tile[P + k - 1 - t]
    if (tile[P + k - 1] == p0) {
      m = 1;
      for (int t = 1; t < P; ++t) {
        if (tile[P + k - 1 - t] != __ldg(pb + t)) break;
        ++m;
      }
    }
    out[static_cast<long long>(b) * n_out + i] = m;
  }
}

// ---------------------------------------------------------------------------
// first_occurrences (triton_kernels.py:217-243, 362-389)
// ---------------------------------------------------------------------------
constexpr int kFoThreads = 256;

__global__ void __launch_bounds__(kFoThreads)
    first_occ_kernel(const int32_t* mb, long long n_cols, const int64_t* thr,
                     int C, int R, int64_t* out_pos, int64_t* out_cnt) {
  __shared__ int warp_tot[kFoThreads / 32];
  const int row = blockIdx.x;
  const int b = row / C;
  const long long th = thr[row];
  const int32_t* m = mb + static_cast<long long>(b) * n_cols;
  int64_t* op = out_pos + static_cast<long long>(row) * R;
  int found = 0;
  if (th > 0) {
    for (long long off = 0; off < n_cols && found < R;
         off += kFoThreads * 4) {
      int v[4];
      int h = 0;
      const long long i0 = off + threadIdx.x * 4;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const long long i = i0 + k;
        v[k] = (i < n_cols) ? __ldg(m + i) : 0;
        h += v[k] >= th;
      }
      const int inc = warp_incl_scan(h);
      if (lane_id() == 31) warp_tot[warp_id()] = inc;
      __syncthreads();
      int pre = 0, tot = 0;
      for (int w = 0; w < kFoThreads / 32; ++w) {
        const int x = warp_tot[w];
        if (w < warp_id()) pre += x;
        tot += x;
      }
      int slot = found + pre + inc - h;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if (v[k] >= th) {
          if (slot < R) op[slot] = i0 + k;
          ++slot;
        }
      }
      found += tot;
      __syncthreads();
    }
  }
  if (found > R) found = R;
  for (int r = found + threadIdx.x; r < R; r += kFoThreads) op[r] = 0;
  if (threadIdx.x == 0) out_cnt[row] = found;
}

// ---------------------------------------------------------------------------
// expand_chain (expand.py:59-147; triton_kernels.py:140-215, 305-338)
// One warp per row; continuations read from the [N, R, K] block.
// ---------------------------------------------------------------------------
constexpr int kExWarps = 4;

template <int RJ>
__global__ void __launch_bounds__(kExWarps * 32)
    expand_kernel(const int32_t* cont, int N, int R, int K,
                  const int64_t* num_occ, const int64_t* cap, float min_prob,
                  float alpha, int32_t* chain, int64_t* nv_out,
                  int64_t* emit_out, float* score_out, int H) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int warp = warp_id();
  const int row = blockIdx.x * kExWarps + warp;
  const int RA = R > 64 ? R : 64;
  unsigned char* wb = smem + static_cast<size_t>(warp) * (4 * RA + 8 * H);
  VoteScratch vs;
  vs.act = reinterpret_cast<int*>(wb);
  vs.hkey = vs.act + RA;
  vs.hcnt = vs.hkey + H;
  vs.hmask = H - 1;
  vs.hshift = 33 - __ffs(H);
  if (row >= N) return;
  const int32_t* c = cont + static_cast<long long>(row) * R * K;
  long long n_occ = num_occ[row];
  if (n_occ > R) n_occ = R;
  if (n_occ < 0) n_occ = 0;
  const long long cp = cap ? cap[row] : K;
  vote_table_clear(vs);
  auto key_of = [](int i) -> int { return i; };
  auto fn = [&](int r, int d) -> int {
    return __ldg(c + static_cast<long long>(r) * K + d);
  };
  int32_t* ch = chain + static_cast<long long>(row) * K;
  // the operator returns num_valid too, so every depth is expanded
  const ExpandResult er = warp_expand<RJ>(
      key_of, fn, static_cast<int>(n_occ), K, cp, /*stop_at_cap=*/false,
      min_prob, alpha, vs, ch);
  if (lane_id() == 0) {
    nv_out[row] = er.num_valid;
    emit_out[row] = er.emit;
    score_out[row] = er.score;
  }
}

}  // namespace sg

using namespace sg;

extern "C" int sg_scatter_append(int32_t* token_ids, int64_t row_stride,
                                 int32_t batch, int32_t seq_len,
                                 const int32_t* base,
                                 const int32_t* valid_count,
                                 const int32_t* sampled, int32_t sampled_cols,
                                 int32_t* new_counts, sg_stream_t stream) {
  if (batch < 0 || seq_len < 1 || row_stride < seq_len || sampled_cols < 0)
    return SG_ERR_INVALID;
  if (batch == 0) return SG_OK;
  if (!token_ids || !base || !sampled || !new_counts) return SG_ERR_INVALID;
  const int th = 128;
  scatter_append_kernel<<<(batch + th - 1) / th, th, 0,
                          reinterpret_cast<cudaStream_t>(stream)>>>(
      token_ids, row_stride, batch, seq_len, base, valid_count, sampled,
      sampled_cols, new_counts);
  return check_launch();
}

extern "C" int sg_match_back(const int32_t* src, int64_t row_stride,
                             int64_t n_src, const int32_t* pat, int32_t batch,
                             int32_t pat_len, int64_t n_out, int32_t* out,
                             sg_stream_t stream) {
  if (batch < 0 || pat_len < 1 || n_out < 0 || n_src < 0 ||
      n_out > n_src + 1 || (row_stride != 0 && row_stride < n_src))
    return SG_ERR_INVALID;
  if (batch == 0 || n_out == 0) return SG_OK;
  if (!src || !pat || !out) return SG_ERR_INVALID;
  const size_t smem = 4 * static_cast<size_t>(pat_len + kMbTile);
  static int cache[64] = {0};
  const int rc = ensure_dyn_smem(match_back_kernel, smem, cache);
  if (rc != SG_OK) return rc;
  dim3 grid(static_cast<unsigned>(ceil_div(n_out, kMbTile)), batch);
  match_back_kernel<<<grid, 256, smem,
                      reinterpret_cast<cudaStream_t>(stream)>>>(
      src, row_stride, n_src, pat, pat_len, n_out, out);
  return check_launch();
}

extern "C" int sg_first_occurrences(const int32_t* mb, int64_t n_cols,
                                    const int64_t* thr, int32_t rows,
                                    int32_t cands, int32_t max_occ,
                                    int64_t* out_pos, int64_t* out_cnt,
                                    sg_stream_t stream) {
  if (rows < 0 || cands < 1 || max_occ < 1 || n_cols < 0)
    return SG_ERR_INVALID;
  if (rows == 0) return SG_OK;
  if (!mb || !thr || !out_pos || !out_cnt) return SG_ERR_INVALID;
  first_occ_kernel<<<rows, kFoThreads, 0,
                     reinterpret_cast<cudaStream_t>(stream)>>>(
      mb, n_cols, thr, cands, max_occ, out_pos, out_cnt);
  return check_launch();
}

template <int RJ>
static int launch_expand(const int32_t* cont, int N, int R, int K,
                         const int64_t* num_occ, const int64_t* cap,
                         float minp, float alpha, int32_t* chain,
                         int64_t* nv, int64_t* emit, float* score,
                         cudaStream_t st) {
  const int H = static_cast<int>(next_pow2_u32(2 * R > 64 ? 2 * R : 64));
  const size_t smem =
      static_cast<size_t>(kExWarps) * (4 * (R > 64 ? R : 64) + 8 * H);
  static int cache[64] = {0};
  const int rc = ensure_dyn_smem(expand_kernel<RJ>, smem, cache);
  if (rc != SG_OK) return rc;
  expand_kernel<RJ><<<(N + kExWarps - 1) / kExWarps, kExWarps * 32, smem,
                      st>>>(cont, N, R, K, num_occ, cap, minp, alpha, chain,
                            nv, emit, score, H);
  return check_launch();
}

extern "C" int sg_expand_chain(const int32_t* cont, int32_t rows,
                               int32_t max_occ, int32_t k,
                               const int64_t* num_occ, const int64_t* cap,
                               float min_token_prob, float alpha,
                               int32_t* chain, int64_t* num_valid,
                               int64_t* num_emit, float* score,
                               sg_stream_t stream) {
  sg::NvtxScope nvtx_range("sg_expand_chain");
  if (rows < 0 || max_occ < 1 || max_occ > 1024 || k < 1) return SG_ERR_INVALID;
  if (rows == 0) return SG_OK;
  if (!cont || !num_occ || !chain || !num_valid || !num_emit || !score)
    return SG_ERR_INVALID;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (max_occ <= 128)
    return launch_expand<4>(cont, rows, max_occ, k, num_occ, cap,
                            min_token_prob, alpha, chain, num_valid, num_emit,
                            score, st);
  if (max_occ <= 256)
    return launch_expand<8>(cont, rows, max_occ, k, num_occ, cap,
                            min_token_prob, alpha, chain, num_valid, num_emit,
                            score, st);
  return launch_expand<32>(cont, rows, max_occ, k, num_occ, cap,
                           min_token_prob, alpha, chain, num_valid, num_emit,
                           score, st);
}
