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
// B200 design: one warp per candidate, survivors resident in registers
// (each lane holds up to RJ occurrences and an alive bit per slot). The
// cost of a depth is its chain of dependent warp operations, so the
// expansion works in passes of up to LA depths:
//   * every survivor reads its next LA tokens at once; one packed warp sum
//     gives the median survivor's (the leader's) count and the voters at
//     depth d, and when the leader holds a strict majority there, the
//     survivors' agreement lengths with the leader and two packed warp
//     sums per two further depths give the same for the rest of the pass:
//     every leading depth where the leader's token holds a strict majority
//     is decided without counting any other token;
//   * a depth without one gets a full vote: <= 32 survivors (one per lane)
//     count their tokens among the 32 in a shared buffer; more survivors
//     count the first and the last pending voter's tokens with ballots (one
//     round, which ends the vote when the uncounted votes cannot reach the
//     best count), and only the remainder goes through a per-warp
//     open-addressing table in shared memory (one CAS insert + one atomic
//     add per token).
// The winner's non-matching occurrences drop their alive bit; whenever the
// survivors fit fewer slots they are compacted (one per lane at <= 32).
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
// every token is inserted on its own and counted with one shared-memory
// atomic. The probe loop is warp-uniform and every slot issues its atomics
// unconditionally (an atomic under a lane condition waits for the one
// before it): a slot with nothing to insert compares -1 against -1, or
// adds 0, at an address of its own, which changes nothing in any order.
template <int RJ>
__device__ __forceinline__ void vote_hash(const int (&v)[RJ], int nslots,
                                          const VoteScratch& vs,
                                          int& best_cnt, int& best_tok,
                                          int& n_act) {
  const int lane = lane_id();
  int hh[RJ], got[RJ];
  unsigned pend = 0;
  int mine = 0;
#pragma unroll
  for (int j = 0; j < RJ; ++j) {
    const bool act = j < nslots && v[j] != -1;
    got[j] = -1;
    hh[j] = act ? static_cast<int>((static_cast<uint32_t>(v[j]) * 0x9E3779B1u) >>
                                   vs.hshift)
                : ((lane * RJ + j) & vs.hmask);
    if (act) {
      pend |= 1u << j;
      ++mine;
    }
  }
  for (int probe = 0; probe <= vs.hmask; ++probe) {
    if (!__any_sync(SG_FULL_MASK, pend != 0u)) break;
    int old[RJ];
#pragma unroll
    for (int j = 0; j < RJ; ++j) {
      const bool p = (pend >> j) & 1u;
      old[j] = atomicCAS(&vs.hkey[hh[j]], -1, p ? v[j] : -1);
    }
#pragma unroll
    for (int j = 0; j < RJ; ++j) {
      if ((pend >> j) & 1u) {
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
    atomicAdd(&vs.hcnt[got[j] >= 0 ? got[j] : hh[j]], got[j] >= 0 ? 1 : 0);
  __syncwarp();
  int my_cnt = 0, my_tok = INT32_MAX;
#pragma unroll
  for (int j = 0; j < RJ; ++j) {
    const int c = vs.hcnt[got[j] >= 0 ? got[j] : hh[j]];
    if (got[j] >= 0 && (c > my_cnt || (c == my_cnt && v[j] < my_tok))) {
      my_cnt = c;
      my_tok = v[j];
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

// The median alive survivor (occurrence order): its slot and lane. n is the
// number of alive survivors. Suffix-array samples come in lexicographic
// order, so a majority continuation always covers the median.
template <int RJ>
__device__ __forceinline__ void median_alive(unsigned amask, int n, int& slot,
                                             int& src) {
  const unsigned lt_mask = (1u << lane_id()) - 1u;
  const int target = n >> 1;  // 0-based rank
  // (ballots of slots past the survivors are 0: no alive bit there)
  int before = 0, sb = 0;
  unsigned bs = 0u;
  slot = 0;
#pragma unroll
  for (int j = 0; j < RJ; ++j) {
    const unsigned bal = __ballot_sync(SG_FULL_MASK, (amask >> j) & 1u);
    const int cj = __popc(bal);
    const bool pick = before <= target && target < before + cj;
    slot = pick ? j : slot;
    bs = pick ? bal : bs;
    sb = pick ? before : sb;
    before += cj;
  }
  const bool me =
      ((bs >> lane_id()) & 1u) && __popc(bs & lt_mask) == target - sb;
  src = __ffs(__ballot_sync(SG_FULL_MASK, me)) - 1;
}

// Plurality over RJ slots per lane when the leader's token ref (count cr,
// na voters in all) has no strict majority. One round counts the tokens
// of the first and the last pending voter with ballots; the vote is over
// once the uncounted votes cannot reach the best count. Copies make a few
// continuations dominate, so this often decides it; otherwise the hash
// table sees the rest, without the dominant keys (inserting many equal
// keys would serialise its atomics on one slot).
template <int RJ>
__device__ __forceinline__ void vote_rest(const int (&v)[RJ], int nslots,
                                          const VoteScratch& vs, int ref,
                                          int cr, int na, int& best_cnt,
                                          int& best_tok) {
  best_cnt = ref != -1 ? cr : 0;
  best_tok = best_cnt > 0 ? ref : INT32_MAX;
  int rem = na - best_cnt;  // votes not yet counted
  unsigned pend = 0u;
#pragma unroll
  for (int j = 0; j < RJ; ++j)
    if (j < nslots && v[j] != -1 && v[j] != ref) pend |= 1u << j;
  {  // one round
    if (rem < best_cnt || rem == 0) return;
    unsigned bal[RJ];  // (pending bits are never past nslots)
#pragma unroll
    for (int j = 0; j < RJ; ++j)
      bal[j] = __ballot_sync(SG_FULL_MASK, (pend >> j) & 1u);
    int j1 = -1, l1 = 0, j2 = -1, l2 = 0;
#pragma unroll
    for (int j = 0; j < RJ; ++j) {
      if (j1 < 0 && bal[j]) {
        j1 = j;
        l1 = __ffs(bal[j]) - 1;
      }
      const int jj = RJ - 1 - j;
      if (j2 < 0 && bal[jj]) {
        j2 = jj;
        l2 = 31 - __clz(bal[jj]);
      }
    }
    int x1 = v[0], x2 = v[0];
#pragma unroll
    for (int j = 1; j < RJ; ++j) {
      if (j == j1) x1 = v[j];
      if (j == j2) x2 = v[j];
    }
    const int t1 = __shfl_sync(SG_FULL_MASK, x1, l1);
    const int t2 = __shfl_sync(SG_FULL_MASK, x2, l2);
    int c1 = 0, c2 = 0;
#pragma unroll
    for (int j = 0; j < RJ; ++j) {
      const bool p = (pend >> j) & 1u;
      c1 += __popc(__ballot_sync(SG_FULL_MASK, p && v[j] == t1));
      c2 += __popc(__ballot_sync(SG_FULL_MASK, p && v[j] == t2 && t2 != t1));
    }
    if (c1 > best_cnt || (c1 == best_cnt && t1 < best_tok)) {
      best_cnt = c1;
      best_tok = t1;
    }
    if (c2 > best_cnt || (c2 == best_cnt && c2 > 0 && t2 < best_tok)) {
      best_cnt = c2;
      best_tok = t2;
    }
#pragma unroll
    for (int j = 0; j < RJ; ++j)
      if (v[j] == t1 || v[j] == t2) pend &= ~(1u << j);
    rem -= c1 + c2;
  }
  if (rem < best_cnt || rem == 0) return;
  int w[RJ];
#pragma unroll
  for (int j = 0; j < RJ; ++j) w[j] = ((pend >> j) & 1u) ? v[j] : -1;
  int hc, ht, hn;
  vote_hash<RJ>(w, nslots, vs, hc, ht, hn);
  if (hc > best_cnt || (hc == best_cnt && hc > 0 && ht < best_tok)) {
    best_cnt = hc;
    best_tok = ht;
  }
}

// Running state of one chain expansion.
struct ChainState {
  float prob;   // chain probability so far
  float score;  // sum of the valid depths' probabilities below the cap
  int nv;       // valid depths
  int written;  // depths [0, written) of the chain are final
};

// The fp32 ratio count / (max(voters, 1) + alpha) of a depth, correctly
// rounded, without contraction (with alpha 0 a count divided by itself is
// exactly 1, as the reference's division gives).
__device__ __forceinline__ float depth_ratio(int cnt, int act, float alpha) {
  const float denom = __fadd_rn(static_cast<float>(act > 1 ? act : 1), alpha);
  return __fdiv_rn(static_cast<float>(cnt), denom);
}

// Commit depth d with its count, ratio and token. False ends the chain.
__device__ __forceinline__ bool commit_ratio(ChainState& cs, int d, int cnt,
                                             float ratio, int tok,
                                             float min_prob, long long cap,
                                             int* chain_out) {
  cs.prob = __fmul_rn(cs.prob, ratio);
  const bool valid = cnt > 0 && cs.prob >= min_prob;
  if (lane_id() == 0) chain_out[d] = valid ? tok : -1;
  cs.written = d + 1;
  if (!valid) return false;
  ++cs.nv;
  if (static_cast<long long>(d) < cap) cs.score = __fadd_rn(cs.score, cs.prob);
  return true;
}

// Survivors into the fewest slots (occurrence order) once n fits in fewer.
template <int RJ>
__device__ __forceinline__ void compact_survivors(int (&e)[RJ], unsigned& amask,
                                                  int& nslots, int n,
                                                  const VoteScratch& vs) {
  if (!(nslots > 1 && n <= 32 * (nslots - 1))) return;
  const int lane = lane_id();
  const unsigned lt_mask = (1u << lane) - 1u;
  int base = 0;
#pragma unroll
  for (int j = 0; j < RJ; ++j) {
    const bool alive = (amask >> j) & 1u;  // never past nslots
    const unsigned bal = __ballot_sync(SG_FULL_MASK, alive);
    if (alive) vs.act[base + __popc(bal & lt_mask)] = e[j];
    base += __popc(bal);
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
//   stop(score, prob, d, rem): checked before a pass of depths starting at
//                 d with the score and chain probability so far and rem =
//                 the scored depths left (warp-uniform); true gives the
//                 candidate up (the result then has stopped set and is not
//                 a valid expansion).
//
// A pass reads the next LA depths of every survivor at once and compares
// them with the median survivor's (the leader's). One packed warp sum gives
// the leader's count c_0 and the voters a_0 at depth d; only when 2 c_0 >
// a_0 does the pass go on: a survivor's agreement length lcp says at which
// depths it still votes for the leader's token, so two packed warp sums per
// two depths give c_k and a_k (survivors that agreed up to k and have a
// token there) for the rest of the pass. Every leading depth with a strict
// majority (2 c_k > a_k) is the vote's result without counting any other
// token; the first depth without one gets a full vote (vote_small, or
// vote_rest knowing c_k).
template <int RJ, class KeyFn, class ContFn, class StopFn = NeverStop>
__device__ ExpandResult warp_expand(KeyFn key_of, ContFn cont, int n_occ,
                                    int K, long long cap, bool stop_at_cap,
                                    float min_prob, float alpha,
                                    const VoteScratch& vs, int* chain_out,
                                    StopFn stop = StopFn()) {
  constexpr int LA = RJ <= 4 ? 4 : 1;  // depths per pass (registers)
  const int lane = lane_id();
  int depth_end = K;
  if (stop_at_cap)
    depth_end = cap < K ? static_cast<int>(cap > 0 ? cap : 0) : K;

  int e[RJ];
  unsigned amask = 0;  // alive slots of this lane
#pragma unroll
  for (int j = 0; j < RJ; ++j) {
    const int i = j * 32 + lane;
    // the first key stands in past n_occ (read unconditionally, unused)
    e[j] = key_of(i < n_occ ? i : 0);
    if (i < n_occ) amask |= 1u << j;
    else e[j] = 0;
  }
  int n = n_occ;               // survivors (warp-uniform)
  int nslots = (n + 31) >> 5;  // slots that may hold survivors

  ChainState cs{1.0f, 0.0f, 0, 0};
  const int scored_end = cap < depth_end ? static_cast<int>(cap > 0 ? cap : 0)
                                         : depth_end;
  bool stopped = false;
  bool ended = false;  // a depth failed: the chain ends there

  int d = 0;
  while (d < depth_end && n > 0) {
    if (stop(cs.score, cs.prob, d, scored_end > d ? scored_end - d : 0)) {
      stopped = true;
      break;
    }
    // ---- pass: the leader's tokens at depths d .. d + la - 1
    int ls, ll;
    median_alive<RJ>(amask, n, ls, ll);
    const int la = depth_end - d < LA ? depth_end - d : LA;
    // Every slot's LA tokens are read unconditionally (keys are always
    // valid, the depth is clamped below depth_end) and masked afterwards: a
    // load under a condition waits for the one before it.
    int tk[RJ][LA];
#pragma unroll
    for (int j = 0; j < RJ; ++j)
#pragma unroll
      for (int u = 0; u < LA; ++u)
        tk[j][u] = cont(e[j], u < la ? d + u : d);
#pragma unroll
    for (int j = 0; j < RJ; ++j) {
      const bool alive = j < nslots && ((amask >> j) & 1u);
#pragma unroll
      for (int u = 0; u < LA; ++u)
        if (!alive || u >= la) tk[j][u] = -1;
    }
    // the leader's token at depth d and its count there (one packed warp
    // sum): the rest of the pass only runs when it holds a strict majority
    int x0 = tk[0][0];
#pragma unroll
    for (int j = 1; j < RJ; ++j)
      if (j == ls) x0 = tk[j][0];
    const int r0 = __shfl_sync(SG_FULL_MASK, x0, ll);
    unsigned pk = 0u;
#pragma unroll
    for (int j = 0; j < RJ; ++j)
      pk += (tk[j][0] != -1 ? 0x10000u : 0u) +
            (r0 != -1 && tk[j][0] == r0 ? 1u : 0u);
    pk = __reduce_add_sync(SG_FULL_MASK, pk);
    int ref = r0, cr = static_cast<int>(pk & 0xffffu),
        na = static_cast<int>(pk >> 16);
    int v[RJ];  // the survivors' tokens at the depth that gets a full vote
#pragma unroll
    for (int j = 0; j < RJ; ++j) v[j] = tk[j][0];
    if (2 * cr > na) {
      int r[LA];
      r[0] = r0;
#pragma unroll
      for (int u = 1; u < LA; ++u) {
        int x = tk[0][u];
#pragma unroll
        for (int j = 1; j < RJ; ++j)
          if (j == ls) x = tk[j][u];
        r[u] = __shfl_sync(SG_FULL_MASK, x, ll);
      }
      // agreement length with the leader (lcp), and whether the survivor
      // has a token at its first disagreeing depth (it votes there): bit
      // masks over the pass's depths, no branches
      int lcp[RJ];
      bool has[RJ];
#pragma unroll
      for (int j = 0; j < RJ; ++j) {
        unsigned eqm = 0u, tkm = 0u;
#pragma unroll
        for (int u = 0; u < LA; ++u) {
          eqm |= static_cast<unsigned>(tk[j][u] == r[u] && r[u] != -1) << u;
          tkm |= static_cast<unsigned>(tk[j][u] != -1) << u;
        }
        const int m = __ffs(~eqm) - 1;  // leading agreeing depths (<= LA)
        const bool alive = (amask >> j) & 1u;
        lcp[j] = alive ? m : -1;
        has[j] = alive && ((tkm >> m) & 1u);
      }
      // c_k = #{lcp > k}; a_k = c_k + #{lcp == k, has}: two depths per sum
      int cnt[LA], act[LA];
      cnt[0] = cr;
      act[0] = na;
#pragma unroll
      for (int k = 1; k < LA; k += 2) {
        unsigned pc = 0u, pa = 0u;
#pragma unroll
        for (int j = 0; j < RJ; ++j) {
          const unsigned g0 = lcp[j] > k;
          const unsigned a0 =
              g0 | static_cast<unsigned>(lcp[j] == k && has[j]);
          pc += g0;
          pa += a0;
          if (k + 1 < LA) {
            const unsigned g1 = lcp[j] > k + 1;
            const unsigned a1 =
                g1 | static_cast<unsigned>(lcp[j] == k + 1 && has[j]);
            pc += g1 << 16;
            pa += a1 << 16;
          }
        }
        pc = __reduce_add_sync(SG_FULL_MASK, pc);
        pa = __reduce_add_sync(SG_FULL_MASK, pa);
        cnt[k] = static_cast<int>(pc & 0xffffu);
        act[k] = static_cast<int>(pa & 0xffffu);
        if (k + 1 < LA) {
          cnt[k + 1] = static_cast<int>(pc >> 16);
          act[k + 1] = static_cast<int>(pa >> 16);
        }
      }
      // Commit the leading depths the leader's token wins by majority, with
      // the ratios of all depths computed first (the divisions overlap); at
      // the first depth without one, keep the leader's figures and the
      // survivors' tokens there (inside the unrolled loop: a selection by
      // run after it would index the arrays dynamically, through local
      // memory).
      float ratio[LA];
#pragma unroll
      for (int k = 0; k < LA; ++k)
        ratio[k] = depth_ratio(cnt[k], act[k], alpha);
      int run = 0, nn = n;
      bool open = true;
#pragma unroll
      for (int k = 0; k < LA; ++k) {
        const bool here = open && k < la;
        const bool maj = here && 2 * cnt[k] > act[k];
        const float np = __fmul_rn(cs.prob, ratio[k]);
        const bool valid = np >= min_prob;
        if (maj) {
          cs.prob = np;
          if (lane == 0) chain_out[d + k] = valid ? r[k] : -1;
          cs.written = d + k + 1;
          const float ns = __fadd_rn(cs.score, np);
          if (valid) {
            ++cs.nv;
            if (static_cast<long long>(d + k) < cap) cs.score = ns;
          }
          ended = !valid;
          ++run;
          nn = cnt[k];
        }
        if (here && !maj) {
          ref = r[k];
          cr = cnt[k];
          na = act[k];
#pragma unroll
          for (int j = 0; j < RJ; ++j) v[j] = lcp[j] >= k ? tk[j][k] : -1;
        }
        open = maj && valid;
      }
      if (ended) break;
      d += run;
      n = nn;
#pragma unroll
      for (int j = 0; j < RJ; ++j)
        if (lcp[j] < run) amask &= ~(1u << j);
      if (run == la) {
        compact_survivors<RJ>(e, amask, nslots, n, vs);
        continue;
      }
    }
    // ---- full vote at depth d (the leader has no strict majority), on the
    // pass's tokens (the slots are compacted only after it)
    int best_cnt = 0, best_tok = -1, n_act = na;
    if (nslots == 1) {
      vote_small(v[0], vs.act, best_cnt, best_tok, n_act);
    } else {
      vote_rest<RJ>(v, nslots, vs, ref, cr, na, best_cnt, best_tok);
    }
    if (!commit_ratio(cs, d, best_cnt, depth_ratio(best_cnt, n_act, alpha),
                      best_tok, min_prob, cap, chain_out)) {
      ended = true;
      break;
    }
    // keep the occurrences that agree with the winner: exactly best_cnt
#pragma unroll
    for (int j = 0; j < RJ; ++j)
      if (v[j] != best_tok) amask &= ~(1u << j);
    n = best_cnt;
    ++d;
    compact_survivors<RJ>(e, amask, nslots, n, vs);
  }
  // depths past the last computed one
  for (int dd = cs.written + lane; dd < K; dd += 32) chain_out[dd] = -1;
  __syncwarp();
  ExpandResult res;
  res.num_valid = cs.nv;
  const long long c0 = cap > 0 ? cap : 0;
  res.emit = static_cast<int>(cs.nv < c0 ? cs.nv : c0);
  res.score = cs.score;
  res.stopped = stopped;
  return res;
}

}  // namespace sg
