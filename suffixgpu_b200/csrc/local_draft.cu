// Fused local draft step for sm_100a: one CTA per request row.
//
// Reproduces SuffixGPUDrafter.propose_with_update / propose with the local
// matcher only (reference suffix_gpu/proposer.py:135-331 and
// LocalMatchKernel, suffix_gpu/local_matcher.py:83-263). The reference runs
// ~40 torch ops or 5 Triton launches per step and materialises match_back
// [B,S], the occurrence lists and the [B,C,R,K] continuation block in HBM;
// here a single kernel keeps everything for a row in shared memory:
//
//   1. TMA bulk copy (cp.async.bulk + mbarrier) of the row's committed
//      tokens into shared memory; the sampled ids are scattered into both
//      the shared copy and the HBM buffer (update_state semantics).
//   2. match_back for every end position i < q, stored as bytes, with a
//      (P+1)-bin histogram of the values (the reference's topk over [B,S]
//      becomes a suffix sum over the histogram: the t-th largest value is
//      the largest L with #{mb >= L} >= t).
//   3. Earliest occurrences of every candidate in one ordered block-wide
//      compaction (two passes over the byte array).
//   4. One warp per candidate expands its continuation chain (sg_vote.cuh),
//      reading continuations straight from the shared row.
//   5. argmax(score + f32(cand) * 1e-6) and the masked draft write.
//
// HBM traffic per row: the committed tokens once, the sampled ids, the
// appended tokens, and the outputs.

#include <cuda_runtime.h>

#include <algorithm>

#include "sg_common.cuh"
#include "sg_vote.cuh"

namespace sg {

constexpr int kLocalThreads = 256;
constexpr int kLocalWarps = kLocalThreads / 32;
constexpr int kMaxCand = 16;  // candidates with threshold 2^c <= S (S < 2^16)

__host__ __device__ inline size_t align16(size_t x) { return (x + 15) & ~size_t(15); }

struct LocalLayout {
  size_t off_tok, off_mb, off_pat, off_hist, off_cand, off_cnt, off_occ;
  size_t off_score, off_emit, off_chain, off_scan, off_warp, warp_bytes;
  size_t total;
  int H;
  __host__ __device__ LocalLayout(int S, int P, int C, int R, int K) {
    const size_t s4 = (static_cast<size_t>(S) + 3) & ~size_t(3);
    H = static_cast<int>(next_pow2_u32(static_cast<uint32_t>(2 * R > 64 ? 2 * R : 64)));
    size_t o = 16;  // mbarrier
    off_tok = o;   o = align16(o + 4 * s4);
    off_mb = o;    o = align16(o + s4);
    off_pat = o;   o = align16(o + 4 * static_cast<size_t>(P));
    off_hist = o;  o = align16(o + 4 * static_cast<size_t>(P + 2));
    off_cand = o;  o = align16(o + 4 * kMaxCand);
    off_cnt = o;   o = align16(o + 4 * kMaxCand);
    off_occ = o;   o = align16(o + 4 * static_cast<size_t>(C) * R);
    off_score = o; o = align16(o + 4 * kMaxCand);
    off_emit = o;  o = align16(o + 4 * kMaxCand);
    off_chain = o; o = align16(o + 4 * static_cast<size_t>(C) * K);
    off_scan = o;  o = align16(o + 4 * static_cast<size_t>(kLocalWarps) * kMaxCand);
    warp_bytes = align16(4 * static_cast<size_t>(R) + 8 * static_cast<size_t>(H));
    off_warp = o;  o += kLocalWarps * warp_bytes;
    total = o;
  }
};

struct LocalArgs {
  sg_draft_params p;
  int n_cand;  // candidates that can be nonzero: 2^c <= S, capped at kMaxCand
  sg_local_inputs in;
  sg_local_outputs out;
};

__device__ __forceinline__ long long spec_cap(const sg_draft_params& p,
                                              int len) {
  if (!p.has_spec_factor) return p.k;
  const float v = __fadd_rn(__fmul_rn(p.spec_factor, static_cast<float>(len)),
                            p.spec_offset);
  const long long c = static_cast<long long>(floorf(v));
  return c > 0 ? c : 0;
}

template <int RJ>
__global__ void __launch_bounds__(kLocalThreads)
    local_draft_kernel(const LocalArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  const sg_draft_params& p = a.p;
  const int S = p.seq_len, P = p.max_pattern_len, R = p.max_occurrences;
  const int K = p.k, C = a.n_cand;
  const LocalLayout L(S, P, C, R, K);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem);
  int* tok_s = reinterpret_cast<int*>(smem + L.off_tok);
  uint8_t* mb_s = smem + L.off_mb;
  int* pat = reinterpret_cast<int*>(smem + L.off_pat);
  int* hist = reinterpret_cast<int*>(smem + L.off_hist);
  int* cand_s = reinterpret_cast<int*>(smem + L.off_cand);
  int* cnt_s = reinterpret_cast<int*>(smem + L.off_cnt);
  int* occ_s = reinterpret_cast<int*>(smem + L.off_occ);
  float* score_s = reinterpret_cast<float*>(smem + L.off_score);
  int* emit_s = reinterpret_cast<int*>(smem + L.off_emit);
  int* chain_s = reinterpret_cast<int*>(smem + L.off_chain);
  int* scan_s = reinterpret_cast<int*>(smem + L.off_scan);

  __shared__ long long s_q, s_base, s_cnt;
  __shared__ int s_mask, s_nload, s_nal, s_bulk;

  const int b = blockIdx.x;
  const int t = threadIdx.x;
  const int lane = lane_id(), warp = warp_id();
  int32_t* row = a.in.token_ids + static_cast<long long>(b) * p.row_stride;

  // ---- 1. row bookkeeping + bulk load -----------------------------------
  if (t == 0) {
    const long long base = a.in.num_tokens[b];
    long long cnt = 0, q = base;
    int m;
    if (a.in.sampled) {
      if (a.in.valid_count) {
        cnt = a.in.valid_count[b];
      } else {
        for (int j = 0; j < a.in.sampled_cols; ++j)
          cnt += a.in.sampled[static_cast<long long>(b) * a.in.sampled_cols + j] != -1;
      }
      q = base + cnt;
      m = (cnt > 0) && (q < a.in.limit);
      a.out.new_counts[b] = static_cast<int32_t>(q);
    } else {
      m = a.in.mask ? (a.in.mask[b] != 0) : 1;
    }
    const long long nl = q < 0 ? 0 : (q < S ? q : S);
    const int nload = m ? static_cast<int>(nl) : 0;
    int nal = nload & ~3;
    const bool aligned = (reinterpret_cast<uintptr_t>(row) & 15) == 0;
    if (!aligned) nal = 0;
    s_q = q; s_base = base; s_cnt = cnt; s_mask = m;
    s_nload = nload; s_nal = nal; s_bulk = nal > 0;
    if (nal > 0) {
      mbar_init(bar, 1);
      const uint32_t bytes = static_cast<uint32_t>(nal) * 4u;
      mbar_arrive_expect_tx(bar, bytes);
      constexpr uint32_t kChunk = 32768;
      for (uint32_t off = 0; off < bytes; off += kChunk) {
        const uint32_t n = bytes - off < kChunk ? bytes - off : kChunk;
        bulk_g2s(reinterpret_cast<unsigned char*>(tok_s) + off,
                 reinterpret_cast<const unsigned char*>(row) + off, n, bar);
      }
    }
  }
  __syncthreads();
  const long long q = s_q;
  const int mask = s_mask, nload = s_nload, nal = s_nal;
  // ragged tail (or the whole row when it is not 16-byte aligned)
  for (int i = nal + t; i < nload; i += kLocalThreads) tok_s[i] = row[i];
  bool timed_out = false;
  if (s_bulk && !mbar_wait(bar, 0)) {
    // A bulk copy of resident memory always lands; should the bound ever
    // run out, wait once more for the copy in flight, then report the row
    // as failed (num_valid = -1) instead of drafting from partial data.
    timed_out = !mbar_wait(bar, 0);
  }
  if (__syncthreads_or(timed_out)) {
    for (int d = t; d < K; d += kLocalThreads)
      a.out.draft[static_cast<long long>(b) * K + d] = -1;
    if (t == 0) a.out.num_valid[b] = -1;
    return;
  }
  // scatter-append the sampled ids (update_state, proposer.py:166-188);
  // the loads above have all landed, so the HBM writes cannot race them
  if (a.in.sampled) {
    for (int j = t; j < a.in.sampled_cols; j += kLocalThreads) {
      const long long pos = s_base + j;
      const int val = a.in.sampled[static_cast<long long>(b) * a.in.sampled_cols + j];
      if (j < s_cnt && val != -1 && pos < S && pos >= 0) {
        row[pos] = val;
        if (pos < nload) tok_s[pos] = val;
      }
    }
  }
  __syncthreads();
  if (t == 0 && s_bulk) mbar_inval(bar);

  if (!mask) {
    for (int d = t; d < K; d += kLocalThreads)
      a.out.draft[static_cast<long long>(b) * K + d] = -1;
    if (t == 0) {
      a.out.num_valid[b] = 0;
      if (a.out.best_score) a.out.best_score[b] = 0.0f;
      if (a.out.best_len) a.out.best_len[b] = 0;
      if (a.out.best_occ) a.out.best_occ[b] = 0;
      if (a.out.row_mask) a.out.row_mask[b] = 0;
    }
    return;
  }

  // ---- 2. pattern + match_back + histogram -------------------------------
  for (int i = t; i < P; i += kLocalThreads) {
    const long long x = q - 1 - i;
    pat[i] = x < 0 ? -2 : tok_s[x < S ? x : S - 1];
  }
  for (int i = t; i < P + 2; i += kLocalThreads) hist[i] = 0;
  __syncthreads();

  const int nw = (nload + 3) >> 2;
  const int pat0 = pat[0];
  for (int w = t; w < nw; w += kLocalThreads) {
    const int i0 = 4 * w;
    const int4 t4 = reinterpret_cast<const int4*>(tok_s)[w];
    const int prev = i0 > 0 ? tok_s[i0 - 1] : -1;
    const int before[4] = {prev, t4.x, t4.y, t4.z};
    uint32_t packed = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int i = i0 + k;
      int m = 0;
      if (i < nload && before[k] == pat0) {
        m = 1;
        for (int tt = 1; tt < P; ++tt) {
          const int y = i - 1 - tt;
          const int v = y >= 0 ? tok_s[y] : -1;
          if (v != pat[tt]) break;
          ++m;
        }
        atomicAdd(&hist[m], 1);
      }
      packed |= static_cast<uint32_t>(m) << (8 * k);
    }
    reinterpret_cast<uint32_t*>(mb_s)[w] = packed;
  }
  __syncthreads();

  // ---- 3. candidates: t-th largest mb for t = 2^c ------------------------
  if (warp == 0) {
    if (lane == 0) {
      int acc = 0;
      for (int l = P; l >= 1; --l) {
        acc += hist[l];
        hist[l] = acc;  // #{mb >= l}
      }
    }
    __syncwarp();
    int cand = 0;
    if (lane < C) {
      const long long thr = 1ll << lane;
      for (int l = P; l >= 1; --l) {
        if (hist[l] >= thr) {
          cand = l;
          break;
        }
      }
      const int mml = p.min_match_len > 1 ? p.min_match_len : 1;
      if (cand < mml) cand = 0;
    }
    const int prev = __shfl_up_sync(SG_FULL_MASK, cand, 1);
    if (lane < C) cand_s[lane] = (lane > 0 && prev == cand) ? 0 : cand;
  }
  __syncthreads();

  // ---- 4. earliest R occurrences of every candidate ----------------------
  {
    int cr[kMaxCand];
#pragma unroll
    for (int c = 0; c < kMaxCand; ++c) cr[c] = c < C ? cand_s[c] : 0;
    const int wpt = (nw + kLocalThreads - 1) / kLocalThreads;
    const int w0 = t * wpt;
    const int w1 = min(w0 + wpt, nw);
    int hits[kMaxCand];
#pragma unroll
    for (int c = 0; c < kMaxCand; ++c) hits[c] = 0;
    for (int w = w0; w < w1; ++w) {
      const uint32_t word = reinterpret_cast<const uint32_t*>(mb_s)[w];
      if (!word) continue;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int m = (word >> (8 * k)) & 0xff;
        if (!m) continue;
#pragma unroll
        for (int c = 0; c < kMaxCand; ++c) hits[c] += (cr[c] > 0 && m >= cr[c]);
      }
    }
    // block exclusive scan of hits[c] in thread order
    int excl[kMaxCand];
#pragma unroll
    for (int c = 0; c < kMaxCand; ++c) {
      if (c >= C) { excl[c] = 0; continue; }
      const int inc = warp_incl_scan(hits[c]);
      if (lane == 31) scan_s[warp * kMaxCand + c] = inc;
      excl[c] = inc - hits[c];
    }
    __syncthreads();
#pragma unroll
    for (int c = 0; c < kMaxCand; ++c) {
      if (c >= C) continue;
      int off = 0, tot = 0;
      for (int w = 0; w < kLocalWarps; ++w) {
        const int v = scan_s[w * kMaxCand + c];
        if (w < warp) off += v;
        tot += v;
      }
      excl[c] += off;
      if (t == 0) cnt_s[c] = tot < R ? tot : R;
    }
    bool any = false;
#pragma unroll
    for (int c = 0; c < kMaxCand; ++c) any |= (cr[c] > 0 && hits[c] > 0 && excl[c] < R);
    if (any) {
      for (int w = w0; w < w1; ++w) {
        const uint32_t word = reinterpret_cast<const uint32_t*>(mb_s)[w];
        if (!word) continue;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int m = (word >> (8 * k)) & 0xff;
          if (!m) continue;
#pragma unroll
          for (int c = 0; c < kMaxCand; ++c) {
            if (cr[c] > 0 && m >= cr[c]) {
              if (excl[c] < R) occ_s[c * R + excl[c]] = 4 * w + k;
              ++excl[c];
            }
          }
        }
      }
    }
  }
  __syncthreads();

  // ---- 5. one warp per candidate: vote + score ---------------------------
  {
    unsigned char* wbase = smem + L.off_warp + warp * L.warp_bytes;
    VoteScratch vs;
    vs.act = reinterpret_cast<int*>(wbase);
    vs.hkey = vs.act + R;
    vs.hcnt = vs.hkey + L.H;
    vs.hmask = L.H - 1;
    for (int c = warp; c < C; c += kLocalWarps) {
      const int cand = cand_s[c];
      int* chain = chain_s + c * K;
      if (cand == 0) {
        for (int d = lane; d < K; d += 32) chain[d] = -1;
        if (lane == 0) {
          score_s[c] = 0.0f;
          emit_s[c] = 0;
        }
        continue;
      }
      const int* occ = occ_s + c * R;
      auto cont = [&](int r, int d) -> int {
        const long long x = static_cast<long long>(occ[r]) + d;
        return x < q ? tok_s[x < S ? x : S - 1] : -1;
      };
      const ExpandResult er = warp_expand<RJ>(
          cont, cnt_s[c], K, spec_cap(p, cand), p.min_token_prob,
          p.vote_alpha, vs, chain);
      if (lane == 0) {
        score_s[c] = er.score;
        emit_s[c] = er.emit;
      }
    }
  }
  __syncthreads();

  // ---- 6. select_local_best (local_matcher.py:245-263) -------------------
  __shared__ int s_best;
  if (t == 0) {
    int best = 0;
    float bv = __fadd_rn(score_s[0], __fmul_rn(static_cast<float>(cand_s[0]), 1e-6f));
    for (int c = 1; c < C; ++c) {
      const float v = __fadd_rn(score_s[c], __fmul_rn(static_cast<float>(cand_s[c]), 1e-6f));
      if (v > bv) {
        bv = v;
        best = c;
      }
    }
    // Candidates c >= n_cand have thresholds above S, hence value 0.0; the
    // first of them is the argmax only when every value above is negative
    // (possible with a negative min_token_prob and alpha).
    if (C < p.num_backoff && 0.0f > bv) best = -1;
    s_best = best;
    a.out.num_valid[b] = best >= 0 ? emit_s[best] : 0;
    if (a.out.best_score) a.out.best_score[b] = best >= 0 ? score_s[best] : 0.0f;
    if (a.out.best_len) a.out.best_len[b] = best >= 0 ? cand_s[best] : 0;
    if (a.out.best_occ) a.out.best_occ[b] = best >= 0 ? cnt_s[best] : 0;
    if (a.out.row_mask) a.out.row_mask[b] = 1;
  }
  __syncthreads();
  const int best = s_best;
  const int emit = best >= 0 ? emit_s[best] : 0;
  for (int d = t; d < K; d += kLocalThreads)
    a.out.draft[static_cast<long long>(b) * K + d] = d < emit ? chain_s[best * K + d] : -1;
}

template <int RJ>
static int launch_local(const LocalArgs& a, size_t smem, cudaStream_t st) {
  static int cache[64] = {0};
  const int rc = ensure_dyn_smem(local_draft_kernel<RJ>, smem, cache);
  if (rc != SG_OK) return rc;
  local_draft_kernel<RJ><<<a.p.batch, kLocalThreads, smem, st>>>(a);
  return check_launch();
}

}  // namespace sg

using namespace sg;

extern "C" int sg_local_draft(const sg_draft_params* params,
                              const sg_local_inputs* in,
                              const sg_local_outputs* out,
                              sg_stream_t stream) {
  if (!params || !in || !out) return SG_ERR_INVALID;
  const sg_draft_params& p = *params;
  if (p.batch < 0 || p.seq_len < 1 || p.row_stride < p.seq_len || p.k < 1 ||
      p.k > 64 || p.max_pattern_len < 1 || p.max_pattern_len > 255 ||
      p.max_occurrences < 1 || p.max_occurrences > 1024 || p.num_backoff < 1)
    return SG_ERR_INVALID;
  if (p.batch == 0) return SG_OK;
  if (!in->num_tokens || !in->token_ids || !out->draft || !out->num_valid)
    return SG_ERR_INVALID;
  if (in->sampled && (!out->new_counts || in->sampled_cols < 0))
    return SG_ERR_INVALID;
  LocalArgs a;
  a.p = p;
  int nc = 0;
  while (nc < p.num_backoff && nc < 31 && (1ll << nc) <= p.seq_len) ++nc;
  if (nc < 1) nc = 1;
  if (nc > kMaxCand) return SG_ERR_UNSUPPORTED;
  a.n_cand = nc;
  a.in = *in;
  a.out = *out;
  const LocalLayout L(p.seq_len, p.max_pattern_len, nc, p.max_occurrences, p.k);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (p.max_occurrences <= 128) return launch_local<4>(a, L.total, st);
  if (p.max_occurrences <= 256) return launch_local<8>(a, L.total, st);
  return launch_local<32>(a, L.total, st);
}
