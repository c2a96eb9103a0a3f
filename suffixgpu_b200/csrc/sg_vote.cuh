// Warp-level majority-vote chain expansion with fused scoring.
//
// Semantics follow suffix_gpu/expand.py:59-147 (torch path) and the
// unweighted branch of _expand_chain_kernel_v2 (triton_kernels.py:140-215):
// at every depth d the occurrences that still agree with the chain so far
// (prefix_ok) and have a token there vote; the winner is the most frequent
// token, ties going to the smallest id; the chain probability is multiplied
// by count / (max(active, 1) + alpha) in correctly rounded fp32; depth d is
// valid while the count is positive and the probability >= min_token_prob;
// the score sums the probabilities of valid depths below the cap.
//
// B200 design: one warp per candidate. Instead of sorting the R values of
// every depth (the Triton kernel) or comparing all pairs (the torch path),
// the warp keeps a compacted list of the surviving occurrences. Up to 32
// survivors vote with __match_any_sync; larger sets count into a per-warp
// open-addressing table in shared memory. After each depth the list is
// compacted to the occurrences that matched the winner (ballot + popc), so
// later depths touch only the survivors.
#pragma once

#include "sg_common.cuh"

namespace sg {

struct ExpandResult {
  int num_valid;  // leading valid depths
  int emit;       // min(num_valid, max(cap, 0))
  float score;
};

// Per-warp shared-memory scratch for the vote.
struct VoteScratch {
  int* act;    // [R] surviving occurrence indices
  int* hkey;   // [H] hash keys (-1 = empty; -1 is never a voting token)
  int* hcnt;   // [H] counts
  int hmask;   // H - 1 (H power of two, >= 2 * R)
};

__device__ __forceinline__ uint32_t hash_tok(int v) {
  uint32_t x = static_cast<uint32_t>(v);
  x *= 0x9E3779B1u;
  return x ^ (x >> 15);
}

// Order key: larger for (higher count, then smaller token).
__device__ __forceinline__ void vote_best(int cnt, int tok, int& best_cnt,
                                          int& best_tok) {
  // warp max of counts, then min token among the lanes holding that count
  const int cmax = __reduce_max_sync(SG_FULL_MASK, cnt);
  const int cand = (cnt == cmax && cnt > 0) ? tok : INT32_MAX;
  // __reduce_min_sync on signed ints orders tokens the way torch's min does
  const int tmin = __reduce_min_sync(SG_FULL_MASK, cand);
  best_cnt = cmax;
  best_tok = tmin;
}

// Expand one candidate with the calling (full) warp.
//   cont(r, d): continuation token of occurrence r at depth d (-1 = none)
//   n_occ: occurrences (rows r < n_occ are active at depth 0)
//   chain_out: K ints written by lane 0..K-1 (warp-strided)
// RJ: max occurrences per lane (R <= 32 * RJ).
template <int RJ, class ContFn>
__device__ ExpandResult warp_expand(ContFn cont, int n_occ, int K,
                                    long long cap, float min_prob,
                                    float alpha, const VoteScratch& vs,
                                    int* chain_out) {
  const int lane = lane_id();
  int n = n_occ;
  for (int i = lane; i < n; i += 32) vs.act[i] = i;
  __syncwarp();

  float prob = 1.0f;
  float score = 0.0f;
  int nv = 0;
  int written = 0;  // depths [0, written) of chain_out are final
  bool alive = n > 0;
  for (int d = 0; d < K && alive; ++d) {
    // gather this depth's tokens for the survivors
    int rr[RJ];
    int vv[RJ];
    int n_act = 0;
#pragma unroll
    for (int j = 0; j < RJ; ++j) {
      const int i = j * 32 + lane;
      rr[j] = -1;
      vv[j] = -1;
      if (i < n) {
        rr[j] = vs.act[i];
        vv[j] = cont(rr[j], d);
      }
      n_act += __popc(__ballot_sync(SG_FULL_MASK, vv[j] != -1));
      if (j * 32 + 32 >= n) break;
    }
    int best_cnt = 0, best_tok = -1;
    if (n_act > 0) {
      if (n <= 32) {
        const int v = vv[0];
        const unsigned act_mask = __ballot_sync(SG_FULL_MASK, v != -1);
        const unsigned peers = __match_any_sync(SG_FULL_MASK, v);
        const int c = (v != -1) ? __popc(peers & act_mask) : 0;
        vote_best(c, v, best_cnt, best_tok);
      } else {
        // clear the table
        for (int h = lane; h <= vs.hmask; h += 32) {
          vs.hkey[h] = -1;
          vs.hcnt[h] = 0;
        }
        __syncwarp();
        int slot[RJ];
#pragma unroll
        for (int j = 0; j < RJ; ++j) {
          slot[j] = -1;
          const int v = vv[j];
          if (v != -1) {
            uint32_t h = hash_tok(v) & vs.hmask;
            for (int probe = 0; probe <= vs.hmask; ++probe) {
              const int old = atomicCAS(&vs.hkey[h], -1, v);
              if (old == -1 || old == v) {
                atomicAdd(&vs.hcnt[h], 1);
                slot[j] = static_cast<int>(h);
                break;
              }
              h = (h + 1) & vs.hmask;
            }
          }
          if (j * 32 + 32 >= n) break;
        }
        __syncwarp();
        int my_cnt = 0, my_tok = INT32_MAX;
#pragma unroll
        for (int j = 0; j < RJ; ++j) {
          if (slot[j] >= 0) {
            const int c = vs.hcnt[slot[j]];
            const int v = vv[j];
            if (c > my_cnt || (c == my_cnt && v < my_tok)) {
              my_cnt = c;
              my_tok = v;
            }
          }
          if (j * 32 + 32 >= n) break;
        }
        vote_best(my_cnt, my_tok, best_cnt, best_tok);
        __syncwarp();
      }
    }
    // fp32 chain probability, correctly rounded, no contraction
    const float denom = __fadd_rn(static_cast<float>(n_act > 1 ? n_act : 1),
                                  alpha);
    prob = __fmul_rn(prob, __fdiv_rn(static_cast<float>(best_cnt), denom));
    const bool valid = best_cnt > 0 && prob >= min_prob;
    if (lane == 0) chain_out[d] = valid ? best_tok : -1;
    written = d + 1;
    if (!valid) {
      alive = false;
      break;
    }
    ++nv;
    if (static_cast<long long>(d) < cap) score = __fadd_rn(score, prob);
    // keep the occurrences that agree with the winner
    int base = 0;
#pragma unroll
    for (int j = 0; j < RJ; ++j) {
      const bool keep = (j * 32 + lane < n) && vv[j] == best_tok;
      const unsigned bal = __ballot_sync(SG_FULL_MASK, keep);
      if (keep) vs.act[base + __popc(bal & ((1u << lane) - 1u))] = rr[j];
      base += __popc(bal);
      if (j * 32 + 32 >= n) break;
    }
    n = base;
    __syncwarp();
  }
  // depths past the first invalid one (or all, with no occurrences)
  for (int dd = written + lane; dd < K; dd += 32) chain_out[dd] = -1;
  __syncwarp();
  ExpandResult res;
  res.num_valid = nv;
  const long long c0 = cap > 0 ? cap : 0;
  res.emit = static_cast<int>(nv < c0 ? nv : c0);
  res.score = score;
  return res;
}

}  // namespace sg
