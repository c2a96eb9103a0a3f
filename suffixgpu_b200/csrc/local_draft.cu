// Fused local draft step for sm_100a: one CTA per request row.
//
// Reproduces SuffixGPUDrafter.propose_with_update / propose with the local
// matcher only (reference suffix_gpu/proposer.py:135-331 and
// LocalMatchKernel, suffix_gpu/local_matcher.py:83-263). The reference runs
// ~40 torch ops or 5 Triton launches per step and materialises match_back
// [B,S], the occurrence lists and the [B,C,R,K] continuation block in HBM;
// here a single kernel keeps everything for a row in shared memory:
//
//   1. Warp 0 reads the row's count and sampled ids; as soon as the count
//      is in, one thread issues a TMA bulk copy (cp.async.bulk + mbarrier)
//      of the tokens the update can leave committed (count + T) into
//      shared memory. The sampled ids are scattered into the shared copy,
//      and into the HBM buffer once the match scan has started
//      (update_state semantics).
//   2. match_back for every end position i < q. Each warp owns a contiguous
//      segment of positions and appends the nonzero ones, in position order,
//      to its own hit list (one prefix sum per 1024-token chunk, no
//      block-wide scan), then turns its histogram of the values into
//      #{mb >= L} per length. The reference's topk over [B,S] becomes a
//      count over these: the t-th largest value is the largest L with
//      #{mb >= L} >= t.
//   3. The earliest R occurrences of each candidate: every warp writes its
//      qualifying hits at the offset the per-warp counts give. One warp per
//      candidate then expands its
//      continuation chain (sg_vote.cuh) reading continuations straight from
//      the shared row, stopping at the candidate's spec cap.
//   4. argmax(score + f32(cand) * 1e-6) and the masked draft write.
//
// HBM traffic per row: the committed tokens once, the sampled ids, the
// appended tokens, and the outputs.

#include <cuda_runtime.h>

#include <atomic>

#include "sg_common.cuh"
#include "sg_vote.cuh"

namespace sg {

constexpr int kLocalThreads = 256;
constexpr int kLocalWarps = kLocalThreads / 32;
constexpr int kMaxCand = 16;  // candidates with threshold 2^c <= S (S < 2^16)

__host__ __device__ inline size_t align16(size_t x) { return (x + 15) & ~size_t(15); }

struct LocalLayout {
  size_t off_tok, off_hits, off_pat, off_whist, off_cge, off_cand, off_score;
  size_t off_emit, off_chain, off_wlen, off_occ, off_warp, warp_bytes;
  size_t total;
  int H;
  __host__ __device__ LocalLayout(int S, int P, int C, int R, int K) {
    const size_t s4 = (static_cast<size_t>(S) + 3) & ~size_t(3);
    H = static_cast<int>(next_pow2_u32(static_cast<uint32_t>(2 * R > 64 ? 2 * R : 64)));
    size_t o = 16;  // mbarrier
    off_tok = o;   o = align16(o + 4 * s4);
    // per-warp hit lists: segments are rounded up to 128 positions each
    off_hits = o;  o = align16(o + 4 * s4 + 4 * 128 * kLocalWarps);
    off_pat = o;   o = align16(o + 4 * static_cast<size_t>(P));
    // per warp: #{hits with mb >= L} for L = 0..P+1 (a histogram until the
    // warp's suffix sum turns it into counts)
    off_whist = o; o = align16(o + 4 * static_cast<size_t>(P + 2) * kLocalWarps);
    off_cge = o;   o = align16(o + 4 * static_cast<size_t>(P + 2));
    off_cand = o;  o = align16(o + 4 * kMaxCand);
    off_score = o; o = align16(o + 4 * kMaxCand);
    off_emit = o;  o = align16(o + 4 * kMaxCand);
    off_chain = o; o = align16(o + 4 * static_cast<size_t>(C) * K);
    off_wlen = o;  o = align16(o + 4 * kLocalWarps);
    off_occ = o;   o = align16(o + 4 * static_cast<size_t>(C) * R);
    warp_bytes = align16(4 * static_cast<size_t>(R > 64 ? R : 64) +
                         8 * static_cast<size_t>(H));
    off_warp = o;  o += kLocalWarps * warp_bytes;
    total = o;
  }
};

struct LocalArgs {
  sg_draft_params p;
  int n_cand;  // candidates that can be nonzero: 2^c <= S, capped at kMaxCand
  int wait_polls;  // bound of the row-load wait (sg_set_wait_polls)
  sg_local_inputs in;
  sg_local_outputs out;
};

// Device error word of this library's draft kernels (one per device that
// loads the library): bits OR-ed in by kernels, read and cleared by
// sg_device_error. Set only on failures, so it costs nothing otherwise.
static __device__ unsigned int g_device_error;

// Bound of the first wait for a row's bulk load, in polls. Lowered only by
// tests (sg_set_wait_polls) to make that wait run out on purpose.
static std::atomic<int> g_wait_polls{kWaitPolls};

__device__ __forceinline__ long long spec_cap(const sg_draft_params& p,
                                              int len) {
  if (!p.has_spec_factor) return p.k;
  const float v = __fadd_rn(__fmul_rn(p.spec_factor, static_cast<float>(len)),
                            p.spec_offset);
  const long long c = static_cast<long long>(floorf(v));
  return c > 0 ? c : 0;
}

// Candidate lengths for support thresholds 2^0..2^(C-1)
// (local_matcher.py:134-157): cand_t is the t-th largest match_back value,
// i.e. the largest L with #{mb >= L} >= t (0 if none), zeroed below
// min_match_len and when equal to the previous candidate. ge[w * (P + 2) +
// L] holds warp w's #{mb >= L}; the block totals go to cge when given.
// Executed by a full warp; lane c < C returns candidate c.
__device__ __forceinline__ int warp_candidates(const int* ge, int P, int C,
                                               int min_match, int* cge) {
  const int lane = lane_id();
  const int stride = P + 2;
  int cand = 0;
  for (int L0 = 1; L0 <= P; L0 += 32) {
    const int L = L0 + lane;
    // (loads from a clamped length, masked after: no load under a branch)
    const int Lc = L <= P ? L : P;
    int v = 0;
#pragma unroll
    for (int w = 0; w < kLocalWarps; ++w) v += ge[w * stride + Lc];
    if (L > P) v = 0;
    if (cge && L <= P) cge[L] = v;
    // cand_c = #{L : cnt_ge[L] >= 2^c}: cnt_ge is non-increasing in L
    for (int c = 0; c < C; ++c) {
      const unsigned m = __ballot_sync(SG_FULL_MASK, L <= P && v >= (1 << c));
      if (lane == c) cand += __popc(m);
    }
  }
  const int mml = min_match > 1 ? min_match : 1;
  if (cand < mml) cand = 0;
  const int prev = __shfl_up_sync(SG_FULL_MASK, cand, 1);
  return (lane > 0 && prev == cand) ? 0 : cand;
}

// update_state's writes for one row (proposer.py:166-188), by one warp:
// row[base + j] = sampled[j] for j < cnt with sampled[j] != -1 and the
// position inside the row; the new count goes to *new_count.
__device__ __forceinline__ void scatter_to_row(int32_t* row, int lane, int T,
                                               const int32_t* srow,
                                               int my_samp, long long base,
                                               long long cnt, int S,
                                               long long q,
                                               int32_t* new_count) {
  for (int j = lane; j < T; j += 32) {
    const int val = j < 32 ? my_samp : srow[j];
    const long long pos = base + j;
    if (j < cnt && val != -1 && pos < S && pos >= 0) row[pos] = val;
  }
  if (lane == 0) *new_count = static_cast<int32_t>(q);
}

template <int RJ, int NC>
__global__ void __launch_bounds__(kLocalThreads, RJ > 8 ? 1 : 2)
    local_draft_kernel(const LocalArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  const sg_draft_params& p = a.p;
  const int S = p.seq_len, P = p.max_pattern_len, R = p.max_occurrences;
  const int K = p.k, C = a.n_cand;
  const LocalLayout L(S, P, C, R, K);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem);
  int* tok_s = reinterpret_cast<int*>(smem + L.off_tok);
  int* hits = reinterpret_cast<int*>(smem + L.off_hits);
  int* pat = reinterpret_cast<int*>(smem + L.off_pat);
  int* whist = reinterpret_cast<int*>(smem + L.off_whist);  // [warps][P+2]
  int* cge = reinterpret_cast<int*>(smem + L.off_cge);      // [P+2]
  float* score_s = reinterpret_cast<float*>(smem + L.off_score);
  int* emit_s = reinterpret_cast<int*>(smem + L.off_emit);
  int* cand_s = reinterpret_cast<int*>(smem + L.off_cand);
  int* chain_s = reinterpret_cast<int*>(smem + L.off_chain);
  int* wlen = reinterpret_cast<int*>(smem + L.off_wlen);
  int* occ_s = reinterpret_cast<int*>(smem + L.off_occ);  // [cands][R]

  __shared__ long long s_q, s_base, s_cnt;
  __shared__ int s_mask, s_nload, s_nal;
  // the best selection value among the candidates finished so far, as an
  // order-preserving key (0 = none yet)
  __shared__ unsigned s_best_key;

  const int b = blockIdx.x;
  const int t = threadIdx.x;
  // Programmatic dependent launch: the next kernel on the stream may be
  // scheduled as soon as every CTA of this one has started, and this one
  // waits until the kernel before it has completed and its writes are
  // visible (both are no-ops for an ordinary launch). Every global access
  // comes after the wait, except the sampled ids / valid counts the CPU
  // wrote to page-locked host memory (host_ids): their host-link round
  // trip overlaps the wait.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  int my_samp = -1;  // warp 0, lane j < T: sampled[b, j]
  int host_vc = 0;   // warp 0: valid_count[b] read early
  if (a.in.host_ids && threadIdx.x < 32 && a.in.sampled) {
    const int T0 = a.in.sampled_cols;
    if (static_cast<int>(threadIdx.x) < T0)
      my_samp = a.in.sampled[static_cast<long long>(b) * T0 + threadIdx.x];
    if (a.in.valid_count) host_vc = a.in.valid_count[b];
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int lane = lane_id(), warp = warp_id();
  const unsigned lt_mask = (1u << lane) - 1u;
  int32_t* row = a.in.token_ids + static_cast<long long>(b) * p.row_stride;
  const int T = a.in.sampled_cols;
  const int32_t* srow =
      a.in.sampled ? a.in.sampled + static_cast<long long>(b) * T : nullptr;

  VoteScratch vs;
  vs.act = reinterpret_cast<int*>(smem + L.off_warp + warp * L.warp_bytes);
  vs.hkey = vs.act + (R > 64 ? R : 64);
  vs.hcnt = vs.hkey + L.H;
  vs.hmask = L.H - 1;
  vs.hshift = 33 - __ffs(L.H);

  // ---- 1. row bookkeeping (warp 0) + bulk load ----------------------------
  if (warp == 0) {
    // the ids may live in host memory: their load goes out first and the
    // bulk copy does not wait for it (below)
    if (srow && lane < T && !a.in.host_ids) my_samp = srow[lane];
    const long long base = a.in.num_tokens[b];
    // Tokens to bulk-copy (whole 16-byte words; a last partial word is
    // copied whole when it lies inside the row's S tokens, and positions
    // past the count are never read as tokens). Without valid counts the
    // update adds at most T ids, so base + T tokens cover the row and the
    // copy starts before the ids arrive; if the row turns out not to
    // draft, the copy is waited for and unused. A remaining ragged tail,
    // or a row that is not 16-byte aligned, is read with plain loads after
    // the barrier, while the bulk copy is in flight.
    auto start_copy = [&](long long upto) -> int {
      const int n = static_cast<int>(upto < 0 ? 0 : (upto < S ? upto : S));
      int nal = n & ~3;
      if (nal < n && nal + 4 <= S) nal += 4;
      if ((reinterpret_cast<uintptr_t>(row) & 15) != 0) nal = 0;
      if (lane == 0 && nal > 0) {
        mbar_init(bar, 1);
        const uint32_t bytes = static_cast<uint32_t>(nal) * 4u;
        mbar_arrive_expect_tx(bar, bytes);
        constexpr uint32_t kChunk = 32768;
        for (uint32_t off = 0; off < bytes; off += kChunk) {
          const uint32_t nb = bytes - off < kChunk ? bytes - off : kChunk;
          bulk_g2s(reinterpret_cast<unsigned char*>(tok_s) + off,
                   reinterpret_cast<const unsigned char*>(row) + off, nb, bar);
        }
      }
      return nal;
    };
    const bool early = !(srow && a.in.valid_count);
    int nal = early ? start_copy(srow ? base + T : base) : 0;
    long long cnt = 0, q = base;
    int m;
    if (srow) {
      if (a.in.valid_count) {
        cnt = a.in.host_ids ? host_vc : a.in.valid_count[b];
      } else {
        cnt = __popc(__ballot_sync(SG_FULL_MASK, lane < T && my_samp != -1));
        for (int j0 = 32; j0 < T; j0 += 32)  // T > 32 (rare)
          cnt += __popc(__ballot_sync(
              SG_FULL_MASK, j0 + lane < T && srow[j0 + lane] != -1));
      }
      q = base + cnt;
      m = (cnt > 0) && (q < a.in.limit);
    } else {
      m = a.in.mask ? (a.in.mask[b] != 0) : 1;
    }
    const long long nl = q < 0 ? 0 : (q < S ? q : S);
    const int nload = m ? static_cast<int>(nl) : 0;
    if (!early) nal = start_copy(nload);
    if (lane == 0) {
      s_q = q; s_base = base; s_cnt = cnt; s_mask = m;
      s_nload = nload; s_nal = nal;
      s_best_key = 0u;
    }
  } else {
    // other warps: empty the vote tables (warp 1 also warp 0's) and the
    // per-warp histograms while the loads are in flight
    vote_table_clear(vs);
    if (warp == 1) {
      VoteScratch v0 = vs;
      const ptrdiff_t back = static_cast<ptrdiff_t>(L.warp_bytes / 4);
      v0.act -= back;
      v0.hkey -= back;
      v0.hcnt -= back;
      vote_table_clear(v0);
    }
    for (int i = t - 32; i < (P + 2) * kLocalWarps; i += kLocalThreads - 32)
      whist[i] = 0;
  }
  __syncthreads();
  const long long q = s_q;
  // q clamped into int range: positions are < S < 2^23
  const int q32 = q > INT32_MAX ? INT32_MAX : (q < INT32_MIN ? INT32_MIN : static_cast<int>(q));
  const int mask = s_mask, nload = s_nload, nal = s_nal;
  // the ragged tail, or the whole row when it is not 16-byte aligned
  // (disjoint from the bulk copy's shared-memory range)
  for (int i = nal + t; i < nload; i += kLocalThreads) tok_s[i] = row[i];
  bool timed_out = false;
  if (nal > 0 && !mbar_wait(bar, 0, a.wait_polls)) {
    // A bulk copy of resident memory always lands; should the bound ever
    // run out, the row drafts nothing (zero drafts, not partial data) and
    // the device error word says so. The copy in flight is waited for
    // (with the full bound) before the block's shared memory is given up.
    timed_out = true;
    atomicOr(&g_device_error, kDevErrWait);
    mbar_wait(bar, 0);
  }
  if (__syncthreads_or(timed_out)) {
    for (int d = t; d < K; d += kLocalThreads)
      a.out.draft[static_cast<long long>(b) * K + d] = -1;
    if (t == 0) {
      a.out.num_valid[b] = 0;
      if (a.out.best_score) a.out.best_score[b] = 0.0f;
      if (a.out.best_len) a.out.best_len[b] = 0;
      if (a.out.best_occ) a.out.best_occ[b] = 0;
      if (a.out.row_mask) a.out.row_mask[b] = 0;
    }
    // the update does not depend on the load: it still happens
    if (warp == 0 && srow)
      scatter_to_row(row, lane, T, srow, my_samp, s_base, s_cnt, S, q,
                     a.out.new_counts + b);
    return;
  }
  if (warp == 0 && mask) {
    // scatter-append the sampled ids into the shared copy (update_state,
    // proposer.py:166-188); the HBM row gets them once the match scan has
    // started (no global store ahead of the next barrier)
    if (srow) {
      const long long base = s_base, cnt = s_cnt;
      for (int j = lane; j < T; j += 32) {
        const int val = j < 32 ? my_samp : srow[j];
        const long long pos = base + j;
        if (j < cnt && val != -1 && pos < nload && pos >= 0) tok_s[pos] = val;
      }
    }
    __syncwarp();  // this warp's scatter into tok_s is visible below
    // pattern, newest-first: pat[t] = tok[q-1-t] or -2 before the start
    // (local_matcher.py:103-112); reads clamp to the buffer like gather
    for (int i = lane; i < P; i += 32) {
      const long long x = q - 1 - i;
      pat[i] = x < 0 ? -2 : tok_s[x < S ? x : S - 1];
    }
  }
  __syncthreads();

  // the update's HBM writes: all loads of the row have landed (a drafting
  // row issues them once its match scan has started)
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
    if (warp == 0 && srow)
      scatter_to_row(row, lane, T, srow, my_samp, s_base, s_cnt, S, q,
                     a.out.new_counts + b);
    return;
  }
  if (warp == 0 && srow)
    scatter_to_row(row, lane, T, srow, my_samp, s_base, s_cnt, S, q,
                   a.out.new_counts + b);

  // ---- 2. match_back: ordered hit lists per warp segment -----------------
  // Each warp owns an equal contiguous segment (a multiple of 32 tokens),
  // walked in 1024-token chunks. In a chunk, lane l examines the 32 tokens
  // [32 l, 32 l + 32) as one bit mask; its 8 vector loads go in a
  // lane-rotated order, so each load instruction of the warp is free of bank
  // conflicts. One prefix sum of the per-lane hit counts then places the
  // positions in order.
  const int nw = (nload + 3) >> 2;  // 4-token words
  // equal segments (whole 8-word lane groups) so that every warp scans a
  // share of the row: 1024-token segments left warps idle on shorter rows
  const int seg = ((nw + kLocalWarps - 1) / kLocalWarps + 7) & ~7;
  const int hstride = P + 2;
  int* my_ge = whist + warp * hstride;
  int* my_hits;
  int nh = 0;
  {
    const int w_begin = warp * seg;
    const int w_end = min(w_begin + seg, nw);
    my_hits = hits + static_cast<size_t>(w_begin) * 4;  // 4*seg slots
    const int4* tok4 = reinterpret_cast<const int4*>(tok_s);
    const int pt0 = pat[0];
    // 2a. positions i with tok[i-1] == pat[0], in order; positions before
    // the buffer start read -1
    uint32_t carry = 0;  // token before the chunk == pat[0]
    if (w_begin < nw) {
      const int tb = tok_s[w_begin > 0 ? 4 * w_begin - 1 : 0];
      carry = (w_begin > 0 ? tb : -1) == pt0;
    }
    for (int c0 = w_begin; c0 < w_end; c0 += 256) {
      const int wl = c0 + 8 * lane;  // this lane's first word
      // The 8 loads are issued together and compared afterwards (a load
      // under a branch waits for the compare before it); a word past the
      // segment reads the segment's first word and is masked out.
      int4 v[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int w = wl + ((k + lane) & 7);
        v[k] = tok4[w < w_end ? w : w_begin];
      }
      uint32_t eq = 0;  // bit q: token 4 wl + q == pat[0]
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int j = (k + lane) & 7;
        const uint32_t bits = static_cast<uint32_t>(v[k].x == pt0) |
                              (static_cast<uint32_t>(v[k].y == pt0) << 1) |
                              (static_cast<uint32_t>(v[k].z == pt0) << 2) |
                              (static_cast<uint32_t>(v[k].w == pt0) << 3);
        eq |= wl + j < w_end ? bits << (4 * j) : 0u;
      }
      // end position 4 wl + p is a hit iff token 4 wl + p - 1 matches: bit
      // p - 1 of eq, or bit 31 of the previous lane's mask for p = 0
      const uint32_t up = __shfl_up_sync(SG_FULL_MASK, eq, 1);
      uint32_t hm = (eq << 1) | (lane == 0 ? carry : (up >> 31));
      carry = __shfl_sync(SG_FULL_MASK, eq, 31) >> 31;
      const int p0 = 4 * wl;
      // ends at or past nload are no positions; ends at or past the
      // segment's end belong to the next warp, which counts them by carry
      const int nvalid = min(nload, 4 * w_end) - p0;
      if (nvalid < 32) hm &= nvalid <= 0 ? 0u : ((1u << nvalid) - 1u);
      if (__ballot_sync(SG_FULL_MASK, hm != 0) == 0) continue;
      const int c = __popc(hm);
      int inc = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int x = __shfl_up_sync(SG_FULL_MASK, inc, o);
        if (lane >= o) inc += x;
      }
      // the lane's hits in order: a walk over the 32 bits with predicated
      // stores (full-rate integer operations only; finding set bits one by
      // one costs a slow-unit __ffs per hit)
      int pos = nh + inc - c;
#pragma unroll
      for (int q = 0; q < 32; ++q) {
        const unsigned bit = (hm >> q) & 1u;
        if (bit) my_hits[pos] = p0 + q;
        pos += bit;
      }
      nh += __shfl_sync(SG_FULL_MASK, inc, 31);
    }
    __syncwarp();
    // 2b. extend every hit; consecutive lanes take consecutive hits, four
    // per lane in flight (their loads go out together)
    const int pr1 = pat[P > 1 ? 1 : 0], pr2 = pat[P > 2 ? 2 : 0],
              pr3 = pat[P > 3 ? 3 : 0];
    const int pt1 = P > 1 ? pr1 : INT32_MIN;
    const int pt2 = P > 2 ? pr2 : INT32_MIN;
    const int pt3 = P > 3 ? pr3 : INT32_MIN;
    int h1 = 0, h2 = 0, h3 = 0, h4 = 0, hp = 0;
    for (int i0 = lane; i0 < nh; i0 += 128) {
      int e[4], t1[4], t2[4], t3[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = i0 + 32 * u;
        // (a slot past nh still lies in the hits buffer: unused)
        const int x = my_hits[i];
        e[u] = i < nh ? x : 0;  // 0: no tokens before it
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int a1 = tok_s[e[u] >= 2 ? e[u] - 2 : 0];
        const int a2 = tok_s[e[u] >= 3 ? e[u] - 3 : 0];
        const int a3 = tok_s[e[u] >= 4 ? e[u] - 4 : 0];
        t1[u] = e[u] >= 2 ? a1 : -1;
        t2[u] = e[u] >= 3 ? a2 : -1;
        t3[u] = e[u] >= 4 ? a3 : -1;
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = i0 + 32 * u;
        if (i >= nh) break;
        int m = 1;
        if (t1[u] == pt1) {
          m = 2;
          if (t2[u] == pt2) {
            m = 3;
            if (t3[u] == pt3) {
              m = 4;
              // four tokens (and pattern entries) per round trip
              for (int tt = 4; tt < P; tt += 4) {
                int run = 0;
                bool go = true;
#pragma unroll
                for (int z = 0; z < 4; ++z) {
                  const int y = e[u] - 1 - tt - z;
                  const int xv = tok_s[y >= 0 ? y : 0];
                  const int x = y >= 0 ? xv : -1;
                  const int pv = pat[min(tt + z, P - 1)];
                  go = go && tt + z < P && x == pv;
                  run += go;
                }
                m += run;
                if (run < 4) break;
              }
            }
          }
        }
        if (m > P) m = P;
        h1 += m == 1;
        h2 += m == 2;
        h3 += m == 3;
        h4 += m == 4;
        hp += m == P && P > 4;  // full-length matches: no atomic per hit
        if (m > 4 && m < P) atomicAdd(&my_ge[m], 1);
        my_hits[i] = (e[u] << 8) | m;
      }
    }
    h1 = warp_sum(h1);
    h2 = warp_sum(h2);
    h3 = warp_sum(h3);
    h4 = warp_sum(h4);
    hp = warp_sum(hp);
    __syncwarp();  // this warp's atomics on my_ge have landed
    // histogram -> #{hits with mb >= L}, suffix sums from the top chunk
    int above = 0;  // #{hits with mb above this chunk of lengths}
    for (int L0 = ((P - 1) & ~31) + 1; L0 >= 1; L0 -= 32) {
      const int Lx = L0 + lane;
      int v = Lx <= P ? my_ge[Lx] : 0;
      v += Lx == 1 ? h1 : Lx == 2 ? h2 : Lx == 3 ? h3 : Lx == 4 ? h4 : 0;
      if (Lx == P && P > 4) v += hp;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_down_sync(SG_FULL_MASK, v, o);
        if (lane + o < 32) v += u;
      }
      v += above;
      above = __shfl_sync(SG_FULL_MASK, v, 0);
      if (Lx <= P) my_ge[Lx] = v;
    }
    if (lane == 0) {
      my_ge[P + 1] = 0;
      wlen[warp] = nh;
    }
  }
  __syncthreads();

  // ---- 3. candidates and their earliest R occurrences -------------------
  const int cand_lane =
      warp_candidates(whist, P, C, p.min_match_len, warp == 0 ? cge : nullptr);
  if (warp == 0 && lane < C) cand_s[lane] = cand_lane;
  // Every warp writes its qualifying hits for each candidate at the offset
  // given by the per-warp counts of the warps before it (a candidate's warp
  // walking all the lists itself measured 4-4.5 k cycles on light rows,
  // more than this pass and its barrier).
  {
    // earliest R end positions per candidate (local_matcher.py:160-184)
    for (int c = 0; c < C; ++c) {
      const int cand = __shfl_sync(SG_FULL_MASK, cand_lane, c);
      if (cand == 0) continue;
      const int k = my_ge[cand];
      if (k == 0) continue;
      int off = 0;
      for (int w = 0; w < warp; ++w) off += whist[w * hstride + cand];
      if (off >= R) continue;
      int* oc = occ_s + c * R + off;
      const int room = R - off;
      if (k == nh) {
        // every hit of this list qualifies: a straight copy
        const int lim = nh < room ? nh : room;
        for (int i = lane; i < lim; i += 32) oc[i] = my_hits[i] >> 8;
      } else {
        // four chunks of 32 hits per round: their loads and ballots go
        // out together (a slot past nh is in the buffer and unused)
        int got = 0;
        for (int i0 = 0; i0 < nh && got < k && got < room; i0 += 128) {
          int ev[4];
          unsigned bv[4];
#pragma unroll
          for (int qd = 0; qd < 4; ++qd) {
            const int i = i0 + 32 * qd + lane;
            const int ex = my_hits[i];
            ev[qd] = i < nh ? ex : 0;
          }
#pragma unroll
          for (int qd = 0; qd < 4; ++qd)
            bv[qd] = __ballot_sync(SG_FULL_MASK, (ev[qd] & 0xff) >= cand);
#pragma unroll
          for (int qd = 0; qd < 4; ++qd) {
            const int r = got + __popc(bv[qd] & lt_mask);
            if (((bv[qd] >> lane) & 1u) && r < room) oc[r] = ev[qd] >> 8;
            got += __popc(bv[qd]);
          }
        }
      }
    }
  }
  __syncthreads();

  // ---- 3b. one warp per candidate: vote + score --------------------------
  for (int c = warp; c < C; c += kLocalWarps) {
    const int cand = __shfl_sync(SG_FULL_MASK, cand_lane, c);
    int* chain = chain_s + c * K;
    if (cand == 0) {
      for (int d = lane; d < K; d += 32) chain[d] = -1;
      if (lane == 0) {
        score_s[c] = 0.0f;
        emit_s[c] = 0;
      }
      continue;
    }
    const int* oc = occ_s + c * R;
    int n = 0;
    for (int w = 0; w < kLocalWarps; ++w) n += whist[w * hstride + cand];
    if (n > R) n = R;
    // continuation tokens (local_matcher.py:186-195): tok[e + d] if e+d < q
    auto key_of = [&](int i) -> int { return oc[i]; };
    auto cont = [&](int e, int d) -> int {
      const int x = e + d;  // e < S < 2^23, d < 64
      // the load is unconditional (an address in the row), the mask after
      const int v = tok_s[x < S ? x : S - 1];
      return x < q32 ? v : -1;
    };
    // The selection (step 4) takes the first maximum of score + f32(cand)
    // * 1e-6. With alpha >= 0 a depth's ratio count / (active + alpha) is
    // at most 1, so the chain probability never grows and the final score
    // is at most score + rem * prob (rem = scored depths left). A
    // candidate whose bound, with a margin above fp32 rounding, is below
    // the value a finished candidate already reached cannot be selected
    // and stops voting; its outputs are never read.
    const float tie = __fmul_rn(static_cast<float>(cand), 1e-6f);
    const bool may_stop = p.vote_alpha >= 0.0f;
    auto stop = [&](float score, float prob, int d, int rem) -> bool {
      (void)d;
      const unsigned kb = *reinterpret_cast<volatile unsigned*>(&s_best_key);
      if (!may_stop || kb == 0u) return false;
      const uint32_t bits = (kb & 0x80000000u) ? (kb & 0x7fffffffu) : ~kb;
      const float best = __uint_as_float(bits);
      // rounded up at every step: above the exact score + rem * prob +
      // tie, and the 1e-5 covers the fp32 rounding of the real sums
      float ub = __fadd_ru(__fadd_ru(score, __fmul_ru(static_cast<float>(rem),
                                                      prob)), tie);
      ub = __fadd_ru(__fmul_ru(ub, 1.00001f), 1e-30f);
      return ub < best;
    };
    const ExpandResult er = warp_expand<RJ>(
        key_of, cont, n, K, spec_cap(p, cand), /*stop_at_cap=*/true,
        p.min_token_prob, p.vote_alpha, vs, chain, stop);
    if (lane == 0) {
      if (er.stopped) {
        score_s[c] = -INFINITY;  // never the maximum (see the rule above)
        emit_s[c] = 0;
      } else {
        score_s[c] = er.score;
        emit_s[c] = er.emit;
        const float v = __fadd_rn(__fadd_rn(er.score, tie), 0.0f);
        const uint32_t vb = __float_as_uint(v);
        atomicMax(&s_best_key, (vb & 0x80000000u) ? ~vb : (vb | 0x80000000u));
      }
    }
  }
  __syncthreads();

  // ---- 4. select_local_best (local_matcher.py:245-263) -------------------
  if (warp == 0) {
    // value = score + f32(cand) * 1e-6; the first maximum wins. Floats map
    // to unsigned keys with the same order (-0 folded into +0).
    float v = -INFINITY;
    if (lane < C)
      v = __fadd_rn(__fadd_rn(score_s[lane],
                              __fmul_rn(static_cast<float>(cand_s[lane]), 1e-6f)),
                    0.0f);
    const uint32_t bits = __float_as_uint(v);
    const uint32_t key = (bits & 0x80000000u) ? ~bits : (bits | 0x80000000u);
    const uint32_t kmax = __reduce_max_sync(SG_FULL_MASK, key);
    const int idx = __reduce_min_sync(SG_FULL_MASK, key == kmax ? lane : 32);
    const uint32_t kb = (kmax & 0x80000000u) ? (kmax & 0x7fffffffu) : ~kmax;
    const float bvf = __uint_as_float(kb);
    int best = idx;
    const float bv = bvf;
    // Candidates c >= n_cand have thresholds above S, hence value 0.0; the
    // first of them is the argmax only when every value above is negative
    // (possible with a negative min_token_prob and alpha).
    if (C < p.num_backoff && 0.0f > bv) best = -1;
    const int emit = best >= 0 ? emit_s[best] : 0;
    for (int d = lane; d < K; d += 32)
      a.out.draft[static_cast<long long>(b) * K + d] =
          d < emit ? chain_s[best * K + d] : -1;
    if (lane == 0) {
      a.out.num_valid[b] = emit;
      if (a.out.best_score)
        a.out.best_score[b] = best >= 0 ? score_s[best] : 0.0f;
      if (a.out.best_len) a.out.best_len[b] = best >= 0 ? cand_s[best] : 0;
      if (a.out.best_occ) {
        // occurrence count of the chosen candidate: min(#{mb >= cand}, R)
        int occ = 0;
        if (best >= 0 && cand_s[best] > 0) {
          const int ge = cge[cand_s[best]];
          occ = ge < R ? ge : R;
        }
        a.out.best_occ[b] = occ;
      }
      if (a.out.row_mask) a.out.row_mask[b] = 1;
    }
  }
}

template <int RJ, int NC>
static int launch_local_nc(const LocalArgs& a, size_t smem, cudaStream_t st) {
  static int cache[64] = {0};
  const int rc = ensure_dyn_smem(local_draft_kernel<RJ, NC>, smem, cache);
  if (rc != SG_OK) return rc;
  // launched with programmatic stream serialization: the kernel's CTAs
  // can be resident while the previous kernel on the stream finishes
  // (griddepcontrol in the kernel keeps the data dependency)
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(a.p.batch));
  cfg.blockDim = dim3(kLocalThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, local_draft_kernel<RJ, NC>, a);
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return SG_ERR_CUDA;
  }
  return check_launch();
}

template <int RJ>
static int launch_local(const LocalArgs& a, size_t smem, cudaStream_t st) {
  return a.n_cand <= 8 ? launch_local_nc<RJ, 8>(a, smem, st)
                       : launch_local_nc<RJ, kMaxCand>(a, smem, st);
}

}  // namespace sg

using namespace sg;

extern "C" int sg_local_draft(const sg_draft_params* params,
                              const sg_local_inputs* in,
                              const sg_local_outputs* out,
                              sg_stream_t stream) {
  sg::NvtxScope nvtx_range("sg_local_draft");
  if (!params || !in || !out) return SG_ERR_INVALID;
  const sg_draft_params& p = *params;
  if (p.batch < 0 || p.seq_len < 1 || p.row_stride < p.seq_len || p.k < 1 ||
      p.k > 64 || p.max_pattern_len < 1 || p.max_pattern_len > 255 ||
      p.max_occurrences < 1 || p.max_occurrences > 1024 || p.num_backoff < 1)
    return SG_ERR_INVALID;
  if (p.seq_len >= (1 << 23)) return SG_ERR_UNSUPPORTED;
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
  a.wait_polls = g_wait_polls.load(std::memory_order_relaxed);
  a.in = *in;
  a.out = *out;
  const LocalLayout L(p.seq_len, p.max_pattern_len, nc, p.max_occurrences, p.k);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (p.max_occurrences <= 128) return launch_local<4>(a, L.total, st);
  if (p.max_occurrences <= 256) return launch_local<8>(a, L.total, st);
  return launch_local<32>(a, L.total, st);
}

extern "C" int sg_set_wait_polls(int polls) {
  return sg::g_wait_polls.exchange(polls < 0 ? sg::kWaitPolls : polls);
}

extern "C" int sg_device_error(uint32_t* bits, int clear, sg_stream_t stream) {
  if (!bits) return SG_ERR_INVALID;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  unsigned int v = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&v, sg::g_device_error,
                                            sizeof(v), 0,
                                            cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e == cudaSuccess && clear && v) {
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbolAsync(sg::g_device_error, &zero, sizeof(zero), 0,
                                cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  }
  if (e != cudaSuccess) {
    sg::set_cuda_error(e);
    return SG_ERR_CUDA;
  }
  *bits = v;
  return SG_OK;
}
