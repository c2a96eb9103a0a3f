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
// B200 design: one warp per candidate, survivors resident in registers.
// Instead of sorting the R values of every depth (the Triton kernel) or
// comparing all pairs (the torch path), each lane holds up to RJ
// occurrences and an alive bit per slot; a depth reads one token per alive
// slot and votes:
//   * <= 32 survivors (one per lane): each lane counts its token among the
//     32 in a shared buffer (8 vector loads), then two warp reductions;
//   * more: the median voter's token is counted with ballots and wins on a
//     strict majority; otherwise the other tokens go through a per-warp
//     open-addressing table in shared memory, one CAS insert + one atomic
//     add per token, all of a lane's in flight together; every lane then
//     empties the slots it used.
// The winner's non-matching occurrences drop their alive bit; whenever the
// survivors fit fewer slots they are compacted (one per lane at <= 32). While all survivors agree, up
// to 8 depths are committed at once from a shared lookahead.
#pragma once

#include "sg_common.cuh"

namespace sg {

struct ExpandResult {
  int num_valid;  // leading valid depths (computed ones when stopping at cap)
  int emit;       // min(num_valid, max(cap, 0))
  float score;
  bool stopped;   // given up early (the stop rule said it cannot win)
};

// Stop rule of warp_expand that never stops.
struct NeverStop {
  __device__ __forceinline__ bool operator()(float, float, int, int) const {
    return false;
  }
};

// Per-warp shared-memory scratch for the vote.
struct VoteScratch {
  int* act;    // [max(R, 64)] compaction / small-vote buffer
  int* hkey;   // [H] hash keys (-1 = empty; -1 is never a voting token)
  int* hcnt;   // [H] counts
  int hmask;   // H - 1 (H power of two, >= 2 * R)
  int hshift;  // 32 - log2(H)
};

// Empty the table (once per warp; every vote leaves it empty again).
__device__ __forceinline__ void vote_table_clear(const VoteScratch& vs) {
  for (int h = lane_id(); h <= vs.hmask; h += 32) {
    vs.hkey[h] = -1;
    vs.hcnt[h] = 0;
  }
  __syncwarp();
}

// Warp max of counts, then the min token among lanes holding that count.
// (__match_any_sync is avoided throughout: it costs ~380 cycles on sm_100a
// against ~30 for a reduction or a shared-memory load.)
__device__ __forceinline__ void vote_best(int cnt, int tok, int& best_cnt,
                                          int& best_tok) {
  const int cmax = __reduce_max_sync(SG_FULL_MASK, cnt);
  const int cand = (cnt == cmax && cnt > 0) ? tok : INT32_MAX;
  // __reduce_min_sync on signed ints orders tokens the way torch's min does
  best_tok = __reduce_min_sync(SG_FULL_MASK, cand);
  best_cnt = cmax;
}

// Plurality vote over one token per lane (-1 = no vote): every lane counts
// its token among the 32 in a shared buffer. Also returns n_act, the number
// of voting lanes.
__device__ __forceinline__ void vote_small(int v, int* buf, int& best_cnt,
                                           int& best_tok, int& n_act) {
  const int lane = lane_id();
  buf[lane] = v;
  __syncwarp();
  const int4* b4 = reinterpret_cast<const int4*>(buf);
  int c = 0, na = 0;
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const int4 w = b4[q];
    c += (w.x == v) + (w.y == v) + (w.z == v) + (w.w == v);
    na += (w.x != -1) + (w.y != -1) + (w.z != -1) + (w.w != -1);
  }
  __syncwarp();
  vote_best(v != -1 ? c : 0, v, best_cnt, best_tok);
  n_act = na;
}

// Plurality vote over RJ slots per lane (-1 = no vote) with the hash table:
// every token is inserted on its own (all of a lane's inserts in flight
// together) and counted with one shared-memory atomic.
template <int RJ>
__device__ __forceinline__ void vote_hash(const int (&v)[RJ], int nslots,
                                          const VoteScratch& vs,
                                          int& best_cnt, int& best_tok,
                                          int& n_act) {
  int hh[RJ], got[RJ];
  unsigned pend = 0;
  int mine = 0;
#pragma unroll
  for (int j = 0; j < RJ; ++j) {
    got[j] = -1;
    hh[j] = 0;
    if (j < nslots && v[j] != -1) {
      pend |= 1u << j;
      ++mine;
      hh[j] = static_cast<int>((static_cast<uint32_t>(v[j]) * 0x9E3779B1u) >>
                               vs.hshift);
    }
  }
  for (int probe = 0; pend && probe <= vs.hmask; ++probe) {
    int old[RJ];
#pragma unroll
    for (int j = 0; j < RJ; ++j)
      if (pend & (1u << j)) old[j] = atomicCAS(&vs.hkey[hh[j]], -1, v[j]);
#pragma unroll
    for (int j = 0; j < RJ; ++j) {
      if (pend & (1u << j)) {
        if (old[j] == -1 || old[j] == v[j]) {
          got[j] = hh[j];
          pend &= ~(1u << j);
        } else {
          hh[j] = (hh[j] + 1) & vs.hmask;
        }
      }
    }
  }
#pragma unroll
  for (int j = 0; j < RJ; ++j)
    if (got[j] >= 0) atomicAdd(&vs.hcnt[got[j]], 1);
  __syncwarp();
  int my_cnt = 0, my_tok = INT32_MAX;
#pragma unroll
  for (int j = 0; j < RJ; ++j) {
    if (got[j] >= 0) {
      const int c = vs.hcnt[got[j]];
      if (c > my_cnt || (c == my_cnt && v[j] < my_tok)) {
        my_cnt = c;
        my_tok = v[j];
      }
    }
  }
  n_act = __reduce_add_sync(SG_FULL_MASK, mine);
  vote_best(my_cnt, my_tok, best_cnt, best_tok);
  // empty the used slots (duplicates are harmless)
#pragma unroll
  for (int j = 0; j < RJ; ++j) {
    if (got[j] >= 0) {
      vs.hkey[got[j]] = -1;
      vs.hcnt[got[j]] = 0;
    }
  }
  __syncwarp();
}

// Plurality vote over RJ slots per lane. The token of the median voter (in
// occurrence order) is the leader and is counted with ballots; a strict
// majority wins outright. Only otherwise do the remaining tokens go
// through the hash table, with the leader's tokens left out: copies make
// one continuation dominate, and inserting 32 equal keys serialises the
// table's atomics on one slot. The median, not the first voter: suffix-
// array samples come in lexicographic order, so the survivors' tokens at
// a depth are sorted and a majority token always covers the middle.
template <int RJ>
__device__ __forceinline__ void vote_multi(const int (&v)[RJ], int nslots,
                                           const VoteScratch& vs,
                                           int& best_cnt, int& best_tok,
                                           int& n_act) {
  const unsigned lt_mask = (1u << lane_id()) - 1u;
  unsigned bal[RJ];
  int na = 0;
#pragma unroll
  for (int j = 0; j < RJ; ++j) {
    bal[j] = j < nslots ? __ballot_sync(SG_FULL_MASK, v[j] != -1) : 0u;
    na += __popc(bal[j]);
  }
  n_act = na;
  if (na == 0) {
    best_cnt = 0;
    best_tok = INT32_MAX;
    return;
  }
  const int target = na >> 1;  // 0-based rank of the median voter
  int ref = -1, before = 0;
#pragma unroll
  for (int j = 0; j < RJ; ++j) {
    const int cj = __popc(bal[j]);
    if (ref == -1 && before + cj > target) {
      const bool me = ((bal[j] >> lane_id()) & 1u) &&
                      __popc(bal[j] & lt_mask) == target - before;
      const unsigned sel = __ballot_sync(SG_FULL_MASK, me);
      ref = __shfl_sync(SG_FULL_MASK, v[j], __ffs(sel) - 1);
    }
    before += cj;
  }
  int cr = 0;
#pragma unroll
  for (int j = 0; j < RJ; ++j)
    if (j < nslots) cr += __popc(__ballot_sync(SG_FULL_MASK, v[j] == ref));
  if (2 * cr > na) {
    best_cnt = cr;
    best_tok = ref;
    return;
  }
  int w[RJ];
#pragma unroll
  for (int j = 0; j < RJ; ++j) w[j] = v[j] == ref ? -1 : v[j];
  int hc, ht, hn;
  vote_hash<RJ>(w, nslots, vs, hc, ht, hn);
  if (hc > cr || (hc == cr && ht < ref)) {
    best_cnt = hc;
    best_tok = ht;
  } else {
    best_cnt = cr;
    best_tok = ref;
  }
}

// Expand one candidate with the calling (full) warp.
//   key_of(i): key of the i-th occurrence, i < n_occ (read once)
//   cont(key, d): continuation token of that occurrence at depth d (-1 =
//                 none)
//   stop_at_cap: stop expanding at depth cap. Depths >= cap change neither
//                num_emit nor the score nor chain[:num_emit], so the
//                drafter (which only uses those) sets it; the expand_chain
//                operator, which also returns num_valid, does not.
//   chain_out: K ints; entries past the last computed depth are -1.
// RJ: max occurrences per lane (R <= 32 * RJ).
//   stop(score, prob, d, rem): checked before depth d with the score and
//                 chain probability so far and rem = the scored depths left
//                 (warp-uniform); true gives the candidate up (the result
//                 then has stopped set and is not a valid expansion).
template <int RJ, class KeyFn, class ContFn, class StopFn = NeverStop>
__device__ ExpandResult warp_expand(KeyFn key_of, ContFn cont, int n_occ,
                                    int K, long long cap, bool stop_at_cap,
                                    float min_prob, float alpha,
                                    const VoteScratch& vs, int* chain_out,
                                    StopFn stop = StopFn()) {
  const int lane = lane_id();
  const unsigned lt_mask = (1u << lane) - 1u;
  int depth_end = K;
  if (stop_at_cap)
    depth_end = cap < K ? static_cast<int>(cap > 0 ? cap : 0) : K;

  int e[RJ];
  unsigned amask = 0;  // alive slots of this lane
#pragma unroll
  for (int j = 0; j < RJ; ++j) {
    const int i = j * 32 + lane;
    e[j] = 0;
    if (i < n_occ) {
      e[j] = key_of(i);
      amask |= 1u << j;
    }
  }
  int n = n_occ;               // survivors (warp-uniform)
  int nslots = (n + 31) >> 5;  // slots that may hold survivors
  const bool unit_alpha = alpha == 0.0f;
  int* ref = vs.act + 32;      // lookahead tokens of the first survivor

  float prob = 1.0f;
  float score = 0.0f;
  int nv = 0;
  int written = 0;  // depths [0, written) of chain_out are final
  int first = 0;    // lowest alive lane when nslots == 1
  bool unanimous = false;  // the last multi-slot vote had every survivor agree
  const int scored_end = cap < depth_end ? static_cast<int>(cap > 0 ? cap : 0)
                                         : depth_end;
  bool stopped = false;
  for (int d = 0; d < depth_end && n > 0; ++d) {
    if (stop(score, prob, d, scored_end > d ? scored_end - d : 0)) {
      stopped = true;
      break;
    }
    if (nslots == 1 || (unanimous && depth_end - d >= 4)) {
      // Unanimous lookahead: while every survivor has the same token, the
      // vote is that token with count = active = survivors, so the depths
      // can be committed without voting (same fp32 steps). With one slot
      // per lane it is tried at every depth; with more, only after a
      // unanimous vote and with at least 4 depths to go (it reads 8 depths
      // of every survivor: measured at 2-4 single-depth votes' cost), and
      // the first survivor (lowest slot, then lowest lane) publishes its
      // tokens before the others compare.
      const int ahead = min(8, depth_end - d);
      int r[8];
      int agree = ahead;
      if (nslots == 1) {
        const bool alive = amask & 1u;
        int tk[8];
#pragma unroll
        for (int u = 0; u < 8; ++u)
          tk[u] = (u < ahead && alive) ? cont(e[0], d + u) : -1;
        if (lane == first) {
#pragma unroll
          for (int u = 0; u < 8; ++u) ref[u] = tk[u];
        }
        __syncwarp();
#pragma unroll
        for (int u = 7; u >= 0; --u) {
          r[u] = ref[u];
          if (u < ahead && (r[u] == -1 || (alive && tk[u] != r[u]))) agree = u;
        }
      } else {
        int l0 = -1, ej = 0;
#pragma unroll
        for (int j = 0; j < RJ; ++j) {
          if (j < nslots) {
            const unsigned bal = __ballot_sync(SG_FULL_MASK, (amask >> j) & 1u);
            if (l0 < 0 && bal) {
              l0 = __ffs(bal) - 1;
              ej = e[j];
            }
          }
        }
        if (lane == l0) {
#pragma unroll
          for (int u = 0; u < 8; ++u) ref[u] = u < ahead ? cont(ej, d + u) : -1;
        }
        __syncwarp();
#pragma unroll
        for (int u = 7; u >= 0; --u) {
          r[u] = ref[u];
          if (u < ahead && r[u] == -1) agree = u;
        }
#pragma unroll
        for (int j = 0; j < RJ; ++j) {
          if (j < nslots && ((amask >> j) & 1u)) {
            int aj = agree;
#pragma unroll
            for (int u = 7; u >= 0; --u)
              if (u < agree && cont(e[j], d + u) != r[u]) aj = u;
            agree = aj < agree ? aj : agree;
          }
        }
      }
      const int run = __reduce_min_sync(SG_FULL_MASK, agree);
      if (run > 0) {
        const float ratio = unit_alpha
            ? 1.0f
            : __fdiv_rn(static_cast<float>(n),
                        __fadd_rn(static_cast<float>(n), alpha));
        bool stop = false;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          if (u < run && !stop) {
            prob = __fmul_rn(prob, ratio);
            const bool valid = prob >= min_prob;
            if (lane == 0) chain_out[d + u] = valid ? r[u] : -1;
            written = d + u + 1;
            if (!valid) {
              stop = true;
            } else {
              ++nv;
              if (static_cast<long long>(d + u) < cap)
                score = __fadd_rn(score, prob);
            }
          }
        }
        __syncwarp();
        if (stop) break;
        if (run < ahead) unanimous = false;  // depth d + run disagrees
        d += run - 1;  // the loop's ++d moves to the first undecided depth
        continue;
      }
      __syncwarp();
    }
    int v[RJ];
#pragma unroll
    for (int j = 0; j < RJ; ++j) {
      v[j] = -1;
      if (j < nslots && (amask & (1u << j))) v[j] = cont(e[j], d);
    }
    int best_cnt = 0, best_tok = -1, n_act = 0;
    if (nslots == 1) {
      vote_small(v[0], vs.act, best_cnt, best_tok, n_act);
    } else {
      vote_multi<RJ>(v, nslots, vs, best_cnt, best_tok, n_act);
      unanimous = best_cnt == n && n_act == n;
    }
    // fp32 chain probability, correctly rounded, no contraction; a
    // unanimous vote with alpha 0 divides a count by itself: exactly 1
    float ratio;
    if (unit_alpha && best_cnt == n_act && n_act > 0) {
      ratio = 1.0f;
    } else {
      const float denom =
          __fadd_rn(static_cast<float>(n_act > 1 ? n_act : 1), alpha);
      ratio = __fdiv_rn(static_cast<float>(best_cnt), denom);
    }
    prob = __fmul_rn(prob, ratio);
    const bool valid = best_cnt > 0 && prob >= min_prob;
    if (lane == 0) chain_out[d] = valid ? best_tok : -1;
    written = d + 1;
    if (!valid) break;
    ++nv;
    if (static_cast<long long>(d) < cap) score = __fadd_rn(score, prob);
    // keep the occurrences that agree with the winner: exactly best_cnt
#pragma unroll
    for (int j = 0; j < RJ; ++j)
      if (j < nslots && v[j] != best_tok) amask &= ~(1u << j);
    n = best_cnt;
    if (nslots > 1 && n <= 32 * (nslots - 1)) {
      // compact the survivors into the fewest slots (occurrence order)
      int base = 0;
#pragma unroll
      for (int j = 0; j < RJ; ++j) {
        if (j < nslots) {
          const bool alive = (amask >> j) & 1u;
          const unsigned bal = __ballot_sync(SG_FULL_MASK, alive);
          if (alive) vs.act[base + __popc(bal & lt_mask)] = e[j];
          base += __popc(bal);
        }
      }
      __syncwarp();
      const int ns = (n + 31) >> 5;
      amask = 0;
#pragma unroll
      for (int j = 0; j < RJ; ++j) {
        const int i = 32 * j + lane;
        if (j < ns) {
          e[j] = i < n ? vs.act[i] : 0;
          if (i < n) amask |= 1u << j;
        }
      }
      nslots = ns;
      __syncwarp();
    }
    if (nslots == 1)
      first = __ffs(__ballot_sync(SG_FULL_MASK, amask & 1u)) - 1;
  }
  // depths past the last computed one
  for (int dd = written + lane; dd < K; dd += 32) chain_out[dd] = -1;
  __syncwarp();
  ExpandResult res;
  res.num_valid = nv;
  const long long c0 = cap > 0 ? cap : 0;
  res.emit = static_cast<int>(nv < c0 ? nv : c0);
  res.score = score;
  res.stopped = stopped;
  return res;
}

}  // namespace sg
