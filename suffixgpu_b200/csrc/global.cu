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
// sg_global_draft: the three steps above after the searches, fused per row
//   (proposer.py:246-320): the per-cap plan, the continuation windows of
//   every sampled occurrence staged in shared memory (depths below the
//   candidate's spec cap only), one warp per cap expanding and scoring its
//   chain (sg_vote.cuh), and the selection against the local winner. The
//   [B, C, R, K] continuation block never goes to HBM.
#include <cuda_runtime.h>

#include "sg_common.cuh"
#include "sg_vote.cuh"

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

// Tails of the rows as update_state will leave them (proposer.py:135-184,
// 110-125), read from the buffer before the scatter: positions below the
// row's count come from the buffer, the appended ones from the sampled ids
// where the scatter writes them (j < count, id != -1, inside the row) and
// from the buffer where it does not. The scatter never writes a position
// this reads, so the local step can update the rows concurrently. Also
// the row mask of propose_with_update (count > 0 and new count < limit).
__global__ void gather_tails_update_kernel(
    const int32_t* __restrict__ tok, int64_t stride, int S,
    const int32_t* __restrict__ base_counts,
    const int32_t* __restrict__ sampled, int T,
    const int32_t* __restrict__ valid_count, int64_t limit,
    const uint8_t* __restrict__ mask, int B, int P,
    int32_t* __restrict__ tails, int64_t* __restrict__ tail_len,
    uint8_t* __restrict__ row_mask) {
  const int b = blockIdx.x;
  __shared__ long long s_cnt;
  const int32_t* srow =
      sampled ? sampled + static_cast<int64_t>(b) * T : nullptr;
  const int64_t base = base_counts[b];
  if (threadIdx.x == 0) {
    long long cnt = 0;
    if (srow) {
      if (valid_count) {
        cnt = valid_count[b];
      } else {
        for (int j = 0; j < T; ++j) cnt += srow[j] != -1;
      }
    }
    s_cnt = cnt;
  }
  __syncthreads();
  const int64_t cnt = s_cnt;
  const int64_t q = base + cnt;
  const int64_t tl = q < P ? q : P;
  const int32_t* row = tok + static_cast<int64_t>(b) * stride;
  if (threadIdx.x == 0) {
    tail_len[b] = tl;
    row_mask[b] = srow ? static_cast<uint8_t>(cnt > 0 && q < limit)
                       : static_cast<uint8_t>(mask ? mask[b] != 0 : 1);
  }
  for (int j = threadIdx.x; j < P; j += blockDim.x) {
    int v = 0;
    if (j < tl) {
      int64_t idx = q - tl + j;
      idx = idx < 0 ? 0 : (idx > S - 1 ? S - 1 : idx);
      v = row[idx];
      const int64_t u = idx - base;  // appended id index
      if (srow && u >= 0 && u < cnt && u < T) {
        const int sv = srow[u];
        if (sv != -1) v = sv;  // idx < S: the scatter writes sv there
      }
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
  int64_t sa_entries;  // entries of sa (capacity, or a sample block's size)
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

// Per-cap plan of one row (global_index.py:321-352), run by one thread:
// SA vs delta (ties prefer the SA), adjacent caps resolving to the same
// (length, source) dropped, occurrence count, SA interval, spec cap.
struct CapPlan {
  long long ml[kGMaxCaps];
  int src[kGMaxCaps];  // 1 = SA, 2 = delta, 0 = none
  long long cnt[kGMaxCaps];
  long long start[kGMaxCaps], ilen[kGMaxCaps];
  long long cap[kGMaxCaps];  // spec cap (K without a spec factor)
};

// Step 1 (threads c < C, in parallel): cap c's search results.
__device__ __forceinline__ void plan_load(const GlobalCandArgs& a, int b,
                                          CapPlan& pl) {
  const int c = threadIdx.x;
  if (c < a.C) {
    const int64_t o = static_cast<int64_t>(b) * a.C + c;
    pl.ml[c] = a.sa_len[o];    // SA length until plan_caps resolves it
    pl.cnt[c] = a.d_len[o];    // delta length until plan_caps resolves it
    pl.start[c] = a.sa_start[o];
    pl.ilen[c] = a.sa_end[o] - a.sa_start[o];
    pl.cap[c] = a.d_cnt[o];    // delta count until plan_caps resolves it
  }
}

// Step 2 (one thread, after a barrier): the plan from the loaded values.
__device__ void plan_caps(const GlobalCandArgs& a, int b, CapPlan& pl) {
  const int C = a.C, R = a.R, K = a.K;
  (void)b;
  long long prev_ml = 0;
  int prev_src = 0;
  for (int c = 0; c < C; ++c) {
    const long long sl = pl.ml[c], dl = pl.cnt[c], dcnt = pl.cap[c];
    const bool use_sa = sl >= dl && sl > 0;
    const bool use_delta = dl > sl && dl > 0;
    const long long ml = use_sa ? sl : (use_delta ? dl : 0);
    const int src = use_sa ? 1 : (use_delta ? 2 : 0);
    // adjacent caps with the same (length, source) draft the same chain
    const bool dup = c > 0 && ml == prev_ml && src == prev_src && ml > 0;
    prev_ml = ml;
    prev_src = src;
    pl.ml[c] = dup ? 0 : ml;
    pl.src[c] = dup ? 0 : src;
    long long cnt = 0;
    if (!dup && use_sa) cnt = pl.ilen[c] < R ? pl.ilen[c] : R;
    if (!dup && use_delta) cnt = dcnt;
    pl.cnt[c] = cnt;
    long long cp = K;
    if (a.has_spec_factor) {
      const float v = __fadd_rn(
          __fmul_rn(a.spec_factor, static_cast<float>(pl.ml[c])),
          a.spec_offset);
      cp = static_cast<long long>(floorf(v));
      cp = cp > 0 ? cp : 0;
    }
    pl.cap[c] = cp;
  }
}

// Continuation token j of occurrence r of cap c (_gather_cont,
// global_index.py:443-463): -1 past the source's end, for SEP / PAD and
// any negative token. `key` is the occurrence's start position.
__device__ __forceinline__ int cont_token(const GlobalCandArgs& a, int src,
                                          long long key, long long ml, int j,
                                          int64_t dlen) {
  const long long x = key + ml + j;
  int t = -1;
  if (src == 1) {
    if (x >= 0 && x < a.capacity) t = a.corpus[x];
  } else {
    if (x >= 0 && x < dlen) t = a.delta[x < a.delta_capacity ? x : a.delta_capacity - 1];
  }
  return (t != kPadToken && t >= 0) ? t : -1;
}

// Start position of occurrence r of cap c: the strided SA sample when the
// interval holds more than R suffixes, else its r-th suffix; or the r-th
// delta position.
__device__ __forceinline__ long long occ_key(const GlobalCandArgs& a,
                                             const CapPlan& pl, int c, int r,
                                             int64_t o) {
  if (pl.src[c] == 1) {
    const long long ilen = pl.ilen[c], st = pl.start[c];
    long long idx = ilen > a.R ? st + (static_cast<long long>(r) * ilen) / a.R
                               : st + r;
    idx = idx < 0 ? 0 : (idx > a.sa_entries - 1 ? a.sa_entries - 1 : idx);
    return a.sa[idx];
  }
  return a.d_pos[o * a.R + r];
}

__global__ void __launch_bounds__(kGThreads)
    global_candidates_kernel(const GlobalCandArgs a) {
  __shared__ CapPlan pl;
  __shared__ long long s_key[kGThreads];
  const int b = blockIdx.x, C = a.C, R = a.R, K = a.K;
  plan_load(a, b, pl);
  __syncthreads();
  if (threadIdx.x == 0) {
    plan_caps(a, b, pl);
    for (int c = 0; c < C; ++c) {
      const int64_t o = static_cast<int64_t>(b) * C + c;
      a.match_len[o] = pl.ml[c];
      a.occ_count[o] = pl.cnt[c];
      if (a.spec_cap) a.spec_cap[o] = pl.cap[c];
    }
  }
  __syncthreads();
  const int64_t dlen = *a.delta_len;
  const int total = C * R;
  for (int cr0 = 0; cr0 < total; cr0 += kGThreads) {
    // one occurrence per thread: its start position, then K tokens
    const int cr = cr0 + threadIdx.x;
    const int c = cr / R, r = cr % R;
    const int64_t o = static_cast<int64_t>(b) * C + c;
    const bool live = cr < total && pl.src[c] != 0 && r < pl.cnt[c];
    if (live) s_key[threadIdx.x] = occ_key(a, pl, c, r, o);
    __syncthreads();
    // tokens: consecutive threads write consecutive (occurrence, depth)
    const int span = (total - cr0 < kGThreads ? total - cr0 : kGThreads) * K;
    for (int e = threadIdx.x; e < span; e += kGThreads) {
      const int li = e / K, j = e % K;
      const int cr2 = cr0 + li;
      const int c2 = cr2 / R, r2 = cr2 % R;
      const bool lv = pl.src[c2] != 0 && r2 < pl.cnt[c2];
      a.cont[(static_cast<int64_t>(b) * C * R + cr2) * K + j] =
          lv ? cont_token(a, pl.src[c2], s_key[li], pl.ml[c2], j, dlen) : -1;
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// Fused global draft step
// ---------------------------------------------------------------------------
struct GlobalDraftArgs {
  GlobalCandArgs g;  // its outputs are unused here
  float min_prob, alpha;
  int32_t* draft;            // [B, K] in/out: the local winner
  int32_t* num_valid;        // [B] in/out
  const float* local_score;  // [B]
  const uint8_t* row_mask;   // [B] or null
};

struct GlobalDraftLayout {
  size_t cont, chain, score, emit, warp, warp_bytes, total;
  int H, nw;
  __host__ __device__ GlobalDraftLayout(int C, int R, int K) {
    nw = C < kGThreads / 32 ? C : kGThreads / 32;
    H = static_cast<int>(next_pow2_u32(static_cast<uint32_t>(2 * R > 64 ? 2 * R : 64)));
    size_t o = 0;
    cont = o;  o += 4 * static_cast<size_t>(C) * (R + 1) * K;
    chain = o; o += 4 * static_cast<size_t>(C) * K;
    score = o; o += 4 * static_cast<size_t>(C);
    emit = o;  o += 4 * static_cast<size_t>(C);
    o = (o + 15) & ~size_t(15);
    warp = o;
    warp_bytes = (4 * static_cast<size_t>(R > 64 ? R : 64) + 8 * static_cast<size_t>(H) + 15) & ~size_t(15);
    o += nw * warp_bytes;
    total = o;
  }
};

template <int RJ>
__global__ void __launch_bounds__(kGThreads, 1)
    global_draft_kernel(const GlobalDraftArgs d) {
  extern __shared__ __align__(16) unsigned char gsm[];
  const GlobalCandArgs& a = d.g;
  const int b = blockIdx.x, C = a.C, R = a.R, K = a.K;
  const GlobalDraftLayout L(C, R, K);
  int* cont = reinterpret_cast<int*>(gsm + L.cont);    // [C][K][R + 1]
  int* chain = reinterpret_cast<int*>(gsm + L.chain);  // [C][K]
  float* score = reinterpret_cast<float*>(gsm + L.score);
  int* emit = reinterpret_cast<int*>(gsm + L.emit);
  __shared__ CapPlan pl;
  __shared__ int s_depth[kGMaxCaps];
  const int t = threadIdx.x, warp = warp_id(), lane = lane_id();
  const bool active = d.row_mask ? d.row_mask[b] != 0 : true;
  plan_load(a, b, pl);
  __syncthreads();
  if (t == 0) {
    plan_caps(a, b, pl);
    for (int c = 0; c < C; ++c) {
      const long long cp = pl.cap[c];
      s_depth[c] = cp < K ? static_cast<int>(cp > 0 ? cp : 0) : K;
    }
  }
  __syncthreads();
  const int64_t dlen = *a.delta_len;
  // Stage the continuation windows (depths below each cap's spec cap),
  // depth-major with a padded stride ([C][K][R + 1]: the vote's lanes read
  // consecutive entries and the transposed stores spread over the banks).
  // First every occurrence's start position (the vote scratch holds them
  // until the vote); then, cap by cap (its plan in registers), T lanes per
  // occurrence read T consecutive tokens with asynchronous 4-byte copies
  // straight into shared memory, all in flight at once; after the wait
  // each thread maps the SEP / PAD / negative tokens it copied to -1.
  const int total = C * R;
  const int RS = R + 1;
  int* keys = reinterpret_cast<int*>(gsm + L.warp);
  for (int cr = t; cr < total; cr += kGThreads) {
    const int c = cr / R, r = cr % R;
    const bool live = pl.src[c] != 0 && r < pl.cnt[c];
    keys[cr] = live ? static_cast<int>(occ_key(a, pl, c, r,
                                               static_cast<int64_t>(b) * C + c))
                    : 0;
  }
  __syncthreads();
  {
    const int T = K <= 16 ? 16 : 32;  // lanes per occurrence
    const int G = 32 / T;             // occurrences per warp step
    const int step = (kGThreads / 32) * G;
    const int r0 = warp * G + lane / T;
    for (int pass = 0; pass < 2; ++pass) {
      for (int c = 0; c < C; ++c) {
        const int src = pl.src[c];
        const int depth = s_depth[c];
        if (src == 0 || depth == 0) continue;
        const int cnt = static_cast<int>(pl.cnt[c] < R ? pl.cnt[c] : R);
        const long long ml = pl.ml[c];
        const int* kc = keys + c * R;
        const int32_t* base = src == 1 ? a.corpus : a.delta;
        const long long lim = src == 1 ? a.capacity : dlen;
        for (int j = lane % T; j < depth; j += T) {
          int* row = cont + (c * K + j) * RS;
          if (pass == 0) {
#pragma unroll 4
            for (int r = r0; r < cnt; r += step) {
              const long long x = static_cast<long long>(kc[r]) + ml + j;
              if (x >= 0 && x < lim)
                cp_async_4(row + r, base + (src == 1 || x < a.delta_capacity
                                                ? x : a.delta_capacity - 1));
              else
                row[r] = -1;
            }
          } else {
            for (int r1 = r0; r1 < cnt; r1 += 4 * step) {
              int v[4];
#pragma unroll
              for (int q = 0; q < 4; ++q)
                v[q] = r1 + q * step < cnt ? row[r1 + q * step] : 0;
#pragma unroll
              for (int q = 0; q < 4; ++q)
                if (r1 + q * step < cnt && (v[q] < 0 || v[q] == kPadToken))
                  row[r1 + q * step] = -1;
            }
          }
        }
      }
      if (pass == 0) cp_async_wait_all();
    }
  }
  __syncthreads();
  // one warp per cap: vote + score (the selection only reads the chain
  // below num_emit, the score and num_emit, so the vote stops at the cap)
  VoteScratch vs;
  if (warp < L.nw) {
    vs.act = reinterpret_cast<int*>(gsm + L.warp + warp * L.warp_bytes);
    vs.hkey = vs.act + (R > 64 ? R : 64);
    vs.hcnt = vs.hkey + L.H;
    vs.hmask = L.H - 1;
    vs.hshift = 33 - __ffs(L.H);
    vote_table_clear(vs);
    for (int c = warp; c < C; c += L.nw) {
      int* ch = chain + c * K;
      int n = 0;
      if (active && pl.src[c] != 0)
        n = static_cast<int>(pl.cnt[c] < R ? (pl.cnt[c] > 0 ? pl.cnt[c] : 0) : R);
      const int* cc = cont + static_cast<size_t>(c) * K * (R + 1);
      auto key_of = [](int i) -> int { return i; };
      auto tok = [&](int i, int dd) -> int { return cc[dd * (R + 1) + i]; };
      const ExpandResult er = warp_expand<RJ>(
          key_of, tok, n, K, pl.cap[c], /*stop_at_cap=*/true, d.min_prob,
          d.alpha, vs, ch);
      if (lane == 0) {
        score[c] = er.score;
        emit[c] = er.emit;
      }
    }
  }
  __syncthreads();
  // first-maximum global candidate; it replaces the local winner only on a
  // strictly greater score (proposer.py:305-320)
  if (warp == 0) {
    int best = 0;
    float bv = score[0];
    for (int c = 1; c < C; ++c) {
      if (score[c] > bv) {
        bv = score[c];
        best = c;
      }
    }
    if (active && bv > d.local_score[b]) {
      const int em = emit[best];
      for (int j = lane; j < K; j += 32)
        d.draft[static_cast<int64_t>(b) * K + j] = j < em ? chain[best * K + j] : -1;
      if (lane == 0) d.num_valid[b] = em;
    }
  }
}

template <int RJ>
static int launch_global_draft(const GlobalDraftArgs& d, cudaStream_t st) {
  const GlobalDraftLayout L(d.g.C, d.g.R, d.g.K);
  static int cache[64] = {0};
  const int rc = ensure_dyn_smem(global_draft_kernel<RJ>, L.total, cache);
  if (rc != SG_OK) return rc;
  global_draft_kernel<RJ><<<d.g.B, kGThreads, L.total, st>>>(d);
  return check_launch();
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

extern "C" int sg_gather_tails_update(
    const int32_t* token_ids, int64_t row_stride, int32_t seq_len,
    const int32_t* base_counts, const int32_t* sampled, int32_t sampled_cols,
    const int32_t* valid_count, int64_t limit, const uint8_t* mask,
    int32_t batch, int32_t pattern_len, int32_t* tails, int64_t* tail_len,
    uint8_t* row_mask, sg_stream_t stream) {
  sg::NvtxScope nvtx_range("sg_gather_tails_update");
  if (batch < 0 || seq_len < 1 || row_stride < seq_len || pattern_len < 1 ||
      (sampled && sampled_cols < 1))
    return SG_ERR_INVALID;
  if (batch == 0) return SG_OK;
  if (!token_ids || !base_counts || !tails || !tail_len || !row_mask)
    return SG_ERR_INVALID;
  gather_tails_update_kernel<<<batch, 64, 0,
                               reinterpret_cast<cudaStream_t>(stream)>>>(
      token_ids, row_stride, seq_len, base_counts, sampled, sampled_cols,
      valid_count, limit, mask, batch, pattern_len, tails, tail_len,
      row_mask);
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
  sg::NvtxScope nvtx_range("sg_global_candidates");
  if (batch < 0 || num_caps < 1 || num_caps > kGMaxCaps || max_occ < 1 ||
      k < 1 || capacity < 1 || delta_capacity < 1)
    return SG_ERR_INVALID;
  if (batch == 0) return SG_OK;
  if (!sa_len || !sa_start || !sa_end || !d_len || !d_pos || !d_cnt || !sa ||
      !corpus || !delta || !delta_len || !match_len || !cont || !occ_count)
    return SG_ERR_INVALID;
  GlobalCandArgs a{sa_len, sa_start, sa_end, d_len, d_pos, d_cnt, sa,
                   corpus, capacity, capacity, delta, delta_capacity,
                   delta_len,
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

static int global_draft_impl(
    const int64_t* sa_len, const int64_t* sa_start, const int64_t* sa_end,
    const int64_t* d_len, const int64_t* d_pos, const int64_t* d_cnt,
    const int32_t* sa, int64_t sa_entries, const int32_t* corpus,
    int64_t capacity, const int32_t* delta, int64_t delta_capacity,
    const int64_t* delta_len, int32_t batch, int32_t num_caps,
    int32_t max_occ, int32_t k, int32_t has_spec_factor, float spec_factor,
    float spec_offset, float min_token_prob, float alpha,
    const float* local_score, const uint8_t* row_mask, int32_t* draft,
    int32_t* num_valid, sg_stream_t stream) {
  if (batch < 0 || num_caps < 1 || num_caps > kGMaxCaps || max_occ < 1 ||
      max_occ > 1024 || k < 1 || k > 64 || capacity < 1 || sa_entries < 1 ||
      delta_capacity < 1)
    return SG_ERR_INVALID;
  if (batch == 0) return SG_OK;
  if (!sa_len || !sa_start || !sa_end || !d_len || !d_pos || !d_cnt || !sa ||
      !corpus || !delta || !delta_len || !local_score || !draft || !num_valid)
    return SG_ERR_INVALID;
  // occurrence start positions are staged as int
  if (capacity > INT32_MAX || delta_capacity > INT32_MAX)
    return SG_ERR_UNSUPPORTED;
  GlobalDraftArgs d;
  d.g = GlobalCandArgs{sa_len, sa_start, sa_end, d_len, d_pos, d_cnt, sa,
                       corpus, capacity, sa_entries, delta, delta_capacity,
                       delta_len, batch, num_caps, max_occ, k,
                       has_spec_factor, spec_factor, spec_offset, nullptr,
                       nullptr, nullptr, nullptr};
  d.min_prob = min_token_prob;
  d.alpha = alpha;
  d.draft = draft;
  d.num_valid = num_valid;
  d.local_score = local_score;
  d.row_mask = row_mask;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (max_occ <= 128) return launch_global_draft<4>(d, st);
  if (max_occ <= 256) return launch_global_draft<8>(d, st);
  return launch_global_draft<32>(d, st);
}

extern "C" int sg_global_draft(
    const int64_t* sa_len, const int64_t* sa_start, const int64_t* sa_end,
    const int64_t* d_len, const int64_t* d_pos, const int64_t* d_cnt,
    const int32_t* sa, const int32_t* corpus, int64_t capacity,
    const int32_t* delta, int64_t delta_capacity, const int64_t* delta_len,
    int32_t batch, int32_t num_caps, int32_t max_occ, int32_t k,
    int32_t has_spec_factor, float spec_factor, float spec_offset,
    float min_token_prob, float alpha, const float* local_score,
    const uint8_t* row_mask, int32_t* draft, int32_t* num_valid,
    sg_stream_t stream) {
  sg::NvtxScope nvtx_range("sg_global_draft");
  return global_draft_impl(sa_len, sa_start, sa_end, d_len, d_pos, d_cnt, sa,
                           capacity, corpus, capacity, delta, delta_capacity,
                           delta_len, batch, num_caps, max_occ, k,
                           has_spec_factor, spec_factor, spec_offset,
                           min_token_prob, alpha, local_score, row_mask,
                           draft, num_valid, stream);
}

extern "C" int sg_global_draft_samples(
    const int64_t* sa_len, const int64_t* sample_start,
    const int64_t* sample_end, const int64_t* d_len, const int64_t* d_pos,
    const int64_t* d_cnt, const int32_t* samples, int64_t num_samples,
    const int32_t* corpus, int64_t capacity, const int32_t* delta,
    int64_t delta_capacity, const int64_t* delta_len, int32_t batch,
    int32_t num_caps, int32_t max_occ, int32_t k, int32_t has_spec_factor,
    float spec_factor, float spec_offset, float min_token_prob, float alpha,
    const float* local_score, const uint8_t* row_mask, int32_t* draft,
    int32_t* num_valid, sg_stream_t stream) {
  sg::NvtxScope nvtx_range("sg_global_draft_samples");
  return global_draft_impl(sa_len, sample_start, sample_end, d_len, d_pos,
                           d_cnt, samples, num_samples, corpus, capacity,
                           delta, delta_capacity, delta_len, batch, num_caps,
                           max_occ, k, has_spec_factor, spec_factor,
                           spec_offset, min_token_prob, alpha, local_score,
                           row_mask, draft, num_valid, stream);
}
