// Global-index candidate assembly and final local/global selection for
// sm_100a.
//
// sg_gather_tails: SuffixGPUDrafter._gather_tails (proposer.py:110-125).
// sg_global_candidates: the tail of GlobalIndex._query_backoff
//   (global_index.py:321-370) plus _gather_cont (:443-463): per cap, SA vs
//   delta choice (ties prefer the SA), removal of adjacent caps that resolve
//   to the same (length, source), strided sampling of the SA interval when
//   it holds more than R suffixes, and the [B, C, R, K] continuation block
//   (SEP, PAD and negative tokens become -1), plus the spec cap of every
//   candidate (local_matcher.py:76-81).
// sg_global_combine: the selection of proposer.py:305-331: first-maximum
//   global candidate, taken over the local winner only on a strictly
//   greater score.
#include <cuda_runtime.h>

#include "sg_common.cuh"

namespace sg {

constexpr int kPadToken = 0x7fffffff;
constexpr int kGThreads = 256;
constexpr int kGMaxCaps = 16;

__global__ void gather_tails_kernel(const int32_t* __restrict__ tok,
                                    int64_t stride, int S,
                                    const int32_t* __restrict__ counts, int B,
                                    int P, int32_t* __restrict__ tails,
                                    int64_t* __restrict__ tail_len) {
  const int b = blockIdx.x;
  const int64_t q = counts[b];
  const int64_t tl = q < P ? q : P;
  if (threadIdx.x == 0) tail_len[b] = tl;
  for (int j = threadIdx.x; j < P; j += blockDim.x) {
    int v = 0;
    if (j < tl) {
      int64_t idx = q - tl + j;
      idx = idx < 0 ? 0 : (idx > S - 1 ? S - 1 : idx);
      v = tok[static_cast<int64_t>(b) * stride + idx];
    }
    tails[static_cast<int64_t>(b) * P + j] = v;
  }
}

struct GlobalCandArgs {
  const int64_t* sa_len;
  const int64_t* sa_start;
  const int64_t* sa_end;
  const int64_t* d_len;
  const int64_t* d_pos;
  const int64_t* d_cnt;
  const int32_t* sa;
  const int32_t* corpus;
  int64_t capacity;
  const int32_t* delta;
  int64_t delta_capacity;
  const int64_t* delta_len;  // device scalar
  int B, C, R, K;
  int has_spec_factor;
  float spec_factor, spec_offset;
  int64_t* match_len;  // [B, C]
  int32_t* cont;       // [B, C, R, K]
  int64_t* occ_count;  // [B, C]
  int64_t* spec_cap;   // [B, C] or null
};

__global__ void __launch_bounds__(kGThreads)
    global_candidates_kernel(const GlobalCandArgs a) {
  __shared__ long long s_ml[kGMaxCaps];
  __shared__ int s_src[kGMaxCaps];   // 1 = SA, 2 = delta, 0 = none
  __shared__ long long s_cnt[kGMaxCaps];
  __shared__ long long s_start[kGMaxCaps], s_ilen[kGMaxCaps];
  const int b = blockIdx.x, C = a.C, R = a.R, K = a.K;
  if (threadIdx.x == 0) {
    long long prev_ml = 0;
    int prev_src = 0;
    for (int c = 0; c < C; ++c) {
      const int64_t o = static_cast<int64_t>(b) * C + c;
      const long long sl = a.sa_len[o], dl = a.d_len[o];
      const bool use_sa = sl >= dl && sl > 0;
      const bool use_delta = dl > sl && dl > 0;
      const long long ml = use_sa ? sl : (use_delta ? dl : 0);
      const int src = use_sa ? 1 : (use_delta ? 2 : 0);
      // adjacent caps with the same (length, source) draft the same chain
      const bool dup = c > 0 && ml == prev_ml && src == prev_src && ml > 0;
      prev_ml = ml;
      prev_src = src;
      const long long ilen = a.sa_end[o] - a.sa_start[o];
      s_start[c] = a.sa_start[o];
      s_ilen[c] = ilen;
      s_ml[c] = dup ? 0 : ml;
      s_src[c] = dup ? 0 : src;
      long long cnt = 0;
      if (!dup && use_sa) cnt = ilen < R ? ilen : R;
      if (!dup && use_delta) cnt = a.d_cnt[o];
      s_cnt[c] = cnt;
      a.match_len[o] = s_ml[c];
      a.occ_count[o] = cnt;
      if (a.spec_cap) {
        long long cp = K;
        if (a.has_spec_factor) {
          const float v = __fadd_rn(
              __fmul_rn(a.spec_factor, static_cast<float>(s_ml[c])),
              a.spec_offset);
          cp = static_cast<long long>(floorf(v));
          cp = cp > 0 ? cp : 0;
        }
        a.spec_cap[o] = cp;
      }
    }
  }
  __syncthreads();
  const int64_t dlen = *a.delta_len;
  const int total = C * R;
  for (int cr = threadIdx.x; cr < total; cr += kGThreads) {
    const int c = cr / R, r = cr % R;
    const int64_t o = static_cast<int64_t>(b) * C + c;
    int32_t* out = a.cont + (o * R + r) * K;
    const int src = s_src[c];
    const long long ml = s_ml[c];
    if (src == 0 || r >= s_cnt[c]) {
      for (int j = 0; j < K; ++j) out[j] = -1;
      continue;
    }
    if (src == 1) {
      // strided sample of the SA interval when it is longer than R
      const long long ilen = s_ilen[c], st = s_start[c];
      long long idx = ilen > R ? st + (static_cast<long long>(r) * ilen) / R
                               : st + r;
      idx = idx < 0 ? 0 : (idx > a.capacity - 1 ? a.capacity - 1 : idx);
      const long long pos = a.sa[idx];
      for (int j = 0; j < K; ++j) {
        const long long x = pos + ml + j;
        int v = -1;
        if (x >= 0 && x < a.capacity) {
          const int t = a.corpus[x];
          if (t != kPadToken && t >= 0) v = t;
        }
        out[j] = v;
      }
    } else {
      const long long pos = a.d_pos[o * R + r];
      for (int j = 0; j < K; ++j) {
        const long long x = pos + ml + j;
        int v = -1;
        if (x >= 0 && x < dlen) {
          const long long xc = x < a.delta_capacity ? x : a.delta_capacity - 1;
          const int t = a.delta[xc];
          if (t != kPadToken && t >= 0) v = t;
        }
        out[j] = v;
      }
    }
  }
}

__global__ void global_combine_kernel(int32_t* __restrict__ draft,
                                      int32_t* __restrict__ num_valid,
                                      const float* __restrict__ l_score,
                                      const uint8_t* __restrict__ row_mask,
                                      const int32_t* __restrict__ g_chain,
                                      const int64_t* __restrict__ g_emit,
                                      const float* __restrict__ g_score,
                                      int B, int C, int K) {
  const int b = blockIdx.x;
  __shared__ int s_pick, s_best;
  if (threadIdx.x == 0) {
    int best = 0;
    float bv = g_score[static_cast<int64_t>(b) * C];
    for (int c = 1; c < C; ++c) {
      const float v = g_score[static_cast<int64_t>(b) * C + c];
      if (v > bv) {
        bv = v;
        best = c;
      }
    }
    const bool m = row_mask ? row_mask[b] != 0 : true;
    s_pick = (bv > l_score[b]) && m;
    s_best = best;
  }
  __syncthreads();
  if (!s_pick) return;
  const int64_t o = static_cast<int64_t>(b) * C + s_best;
  const int64_t emit = g_emit[o];
  for (int d = threadIdx.x; d < K; d += blockDim.x)
    draft[static_cast<int64_t>(b) * K + d] =
        d < emit ? g_chain[o * K + d] : -1;
  if (threadIdx.x == 0) num_valid[b] = static_cast<int32_t>(emit);
}

}  // namespace sg

using namespace sg;

extern "C" int sg_gather_tails(const int32_t* token_ids, int64_t row_stride,
                               int32_t seq_len, const int32_t* counts,
                               int32_t batch, int32_t pattern_len,
                               int32_t* tails, int64_t* tail_len,
                               sg_stream_t stream) {
  if (batch < 0 || seq_len < 1 || row_stride < seq_len || pattern_len < 1)
    return SG_ERR_INVALID;
  if (batch == 0) return SG_OK;
  if (!token_ids || !counts || !tails || !tail_len) return SG_ERR_INVALID;
  gather_tails_kernel<<<batch, 64, 0,
                        reinterpret_cast<cudaStream_t>(stream)>>>(
      token_ids, row_stride, seq_len, counts, batch, pattern_len, tails,
      tail_len);
  return check_launch();
}

extern "C" int sg_global_candidates(
    const int64_t* sa_len, const int64_t* sa_start, const int64_t* sa_end,
    const int64_t* d_len, const int64_t* d_pos, const int64_t* d_cnt,
    const int32_t* sa, const int32_t* corpus, int64_t capacity,
    const int32_t* delta, int64_t delta_capacity, const int64_t* delta_len,
    int32_t batch, int32_t num_caps, int32_t max_occ, int32_t k,
    int32_t has_spec_factor, float spec_factor, float spec_offset,
    int64_t* match_len, int32_t* cont, int64_t* occ_count, int64_t* spec_cap,
    sg_stream_t stream) {
  if (batch < 0 || num_caps < 1 || num_caps > kGMaxCaps || max_occ < 1 ||
      k < 1 || capacity < 1 || delta_capacity < 1)
    return SG_ERR_INVALID;
  if (batch == 0) return SG_OK;
  if (!sa_len || !sa_start || !sa_end || !d_len || !d_pos || !d_cnt || !sa ||
      !corpus || !delta || !delta_len || !match_len || !cont || !occ_count)
    return SG_ERR_INVALID;
  GlobalCandArgs a{sa_len, sa_start, sa_end, d_len, d_pos, d_cnt, sa,
                   corpus, capacity, delta, delta_capacity, delta_len,
                   batch, num_caps, max_occ, k, has_spec_factor,
                   spec_factor, spec_offset, match_len, cont, occ_count,
                   spec_cap};
  global_candidates_kernel<<<batch, kGThreads, 0,
                             reinterpret_cast<cudaStream_t>(stream)>>>(a);
  return check_launch();
}

extern "C" int sg_global_combine(int32_t* draft, int32_t* num_valid,
                                 const float* local_score,
                                 const uint8_t* row_mask,
                                 const int32_t* g_chain, const int64_t* g_emit,
                                 const float* g_score, int32_t batch,
                                 int32_t num_caps, int32_t k,
                                 sg_stream_t stream) {
  if (batch < 0 || num_caps < 1 || k < 1) return SG_ERR_INVALID;
  if (batch == 0) return SG_OK;
  if (!draft || !num_valid || !local_score || !g_chain || !g_emit || !g_score)
    return SG_ERR_INVALID;
  global_combine_kernel<<<batch, 32, 0,
                          reinterpret_cast<cudaStream_t>(stream)>>>(
      draft, num_valid, local_score, row_mask, g_chain, g_emit, g_score,
      batch, num_caps, k);
  return check_launch();
}
