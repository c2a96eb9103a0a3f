/*
 * suffixgpu.h -- C ABI of the B200 (sm_100a) SuffixGPU drafter kernels.
 *
 * Every entry point takes raw device pointers, sizes and scalars plus a
 * cudaStream_t, enqueues work on that stream and returns a status code.
 * None of them allocates device memory or synchronises the host, so they
 * can be captured into CUDA graphs. Scratch memory, where a kernel needs
 * some, is passed in by the caller as a workspace pointer + byte size; the
 * matching *_workspace_size() query says how much.
 *
 * Integer conventions: token ids are int32. Where the reference's Python
 * operator returns int64 tensors (counts, positions, SA intervals), the
 * corresponding pointer here is int64_t so the host can hand the buffer
 * back without a conversion.
 *
 * Reference = zip95297/SuffixGPU (Python/Triton). Each declaration names the
 * reference function whose results it reproduces.
 */
#ifndef SUFFIXGPU_H_
#define SUFFIXGPU_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* sg_stream_t; /* == cudaStream_t */

/* ---- status codes ------------------------------------------------------ */
#define SG_OK 0
#define SG_ERR_INVALID 1     /* bad shape, pointer or parameter */
#define SG_ERR_WORKSPACE 2   /* workspace missing or too small */
#define SG_ERR_CUDA 3        /* launch / runtime error (see sg_last_cuda_error) */
#define SG_ERR_UNSUPPORTED 4 /* shape beyond this build's limits */

/* Human-readable text for a status code (static storage). */
const char* sg_status_string(int status);
/* Last CUDA error code seen by an entry point on this thread (0 if none). */
int sg_last_cuda_error(void);
/* ABI version: (major << 16) | minor. */
int sg_abi_version(void);
/* Device address of page-locked ("pinned") host memory: SG_OK and
 * *device_ptr set when host_ptr lies in a cudaHostAlloc / cudaHostRegister
 * allocation the current device can reach; SG_ERR_INVALID for pageable or
 * device memory. With unified addressing the two addresses are equal. The
 * local draft step accepts such addresses for its sampled ids and its
 * draft / num_valid outputs (see sg_local_inputs). No reference counterpart:
 * the reference takes device tensors only; this lets a host-side caller
 * skip the separate copies of the step's small inputs and outputs. */
int sg_mapped_host_ptr(const void* host_ptr, void** device_ptr);

/* ---- local drafter ------------------------------------------------------
 * Drafter parameters shared by the local and global paths
 * (reference: suffix_gpu/proposer.py:37-112, local_matcher.py:52-74).
 */
typedef struct sg_draft_params {
  int32_t batch;            /* B: rows */
  int32_t seq_len;          /* S: row capacity of token_ids */
  int64_t row_stride;       /* elements between consecutive rows (>= S) */
  int32_t k;                /* draft length K (<= 64) */
  int32_t max_pattern_len;  /* P (<= 255) */
  int32_t max_occurrences;  /* R (<= 1024) */
  int32_t num_backoff;      /* C: support thresholds 2^0..2^(C-1) (<= 32) */
  int32_t min_match_len;    /* clamped to >= 1 like the reference */
  int32_t has_spec_factor;  /* 0: cap = K; 1: floor(f*L + o) */
  float spec_factor;        /* max_spec_factor (rounded to fp32) */
  float spec_offset;        /* max_spec_offset (rounded to fp32) */
  float min_token_prob;     /* rounded to fp32 */
  float vote_alpha;         /* vote_smoothing_alpha (rounded to fp32) */
} sg_draft_params;

/* Inputs of one local draft step. `sampled`, `valid_count` and the
 * outputs `draft` / `num_valid` may also point into page-locked host memory
 * (the address sg_mapped_host_ptr returns): the kernel then reads the ids
 * and writes the drafts over the host link itself, so a host-driven decode
 * loop needs no separate host<->device copies for them. The caller must not
 * touch those host buffers until the stream has passed the call. */
typedef struct sg_local_inputs {
  const int32_t* num_tokens; /* [B] counts before the update (propose mode:
                                the current counts) */
  int32_t* token_ids;        /* [B, row_stride] resident buffer; updated in
                                place in update mode */
  const int32_t* sampled;    /* [B, sampled_cols] ids, -1 padded; NULL =
                                propose mode (no update) */
  int32_t sampled_cols;      /* T */
  int32_t host_ids;          /* 0, or nonzero when sampled (and valid_count)
                                are page-locked host memory that the CPU
                                wrote before the call: the kernel then reads
                                them before waiting for the previous kernel
                                on the stream, hiding the host-link latency.
                                Must stay 0 if GPU work still in flight
                                writes them. */
  const int32_t* valid_count; /* [B] or NULL: #(sampled[b, :] != -1) */
  const uint8_t* mask;       /* propose mode: [B] rows allowed to draft, or
                                NULL = all rows */
  int64_t limit;             /* update mode: rows draft only while
                                new_count < limit (min(max_model_len, S)) */
} sg_local_inputs;

/* Outputs of one local draft step (optional ones may be NULL). */
typedef struct sg_local_outputs {
  int32_t* draft;       /* [B, K] int32, -1 past num_valid */
  int32_t* num_valid;   /* [B] int32 */
  int32_t* new_counts;  /* [B] int32, update mode only */
  float* best_score;    /* [B] score of the selected local candidate */
  int32_t* best_len;    /* [B] its match length */
  int32_t* best_occ;    /* [B] its occurrence count */
  uint8_t* row_mask;    /* [B] 1 where the row was allowed to draft */
} sg_local_outputs;

/*
 * Fused local draft step: optional scatter-append of the sampled ids,
 * eligibility mask, local suffix match with backoff candidates, earliest
 * occurrences, continuation vote/score and best-candidate select.
 *
 * Replaces SuffixGPUDrafter.propose_with_update / propose for the
 * local-only drafter (suffix_gpu/proposer.py:135-218, :220-331 with
 * global_index None), i.e. LocalMatchKernel.forward
 * (suffix_gpu/local_matcher.py:83-242) and the Triton kernels
 * _scatter_append_kernel / _match_back_kernel / _first_occ_kernel /
 * _expand_chain_kernel_v2 (suffix_gpu/triton_kernels.py:39-256).
 *
 * Update mode (sampled != NULL): token_ids rows are updated in place,
 * new_counts[b] = num_tokens[b] + cnt[b] with cnt = valid_count[b] or the
 * number of sampled[b, :] entries != -1, and a row drafts only when
 * cnt > 0 and new_count < limit (proposer.py:186-218).
 * Propose mode (sampled == NULL): counts are num_tokens and rows draft
 * where mask[b] != 0.
 * Rows must fit in shared memory: S <= ~40k tokens on B200.
 * Failure: a row whose bulk load into shared memory does not land within
 * the kernel's bounded wait drafts nothing (draft all -1, num_valid 0,
 * row_mask 0; the update still happens) and sets SG_DEVERR_WAIT in the
 * device error word (sg_device_error). Never expected on a healthy GPU.
 */
int sg_local_draft(const sg_draft_params* params, const sg_local_inputs* in,
                   const sg_local_outputs* out, sg_stream_t stream);

/* ---- device-side failures (no reference counterpart: the reference has
 * no bounded waits) ------------------------------------------------------- */
#define SG_DEVERR_WAIT 1u /* a bounded wait of sg_local_draft ran out */

/* Reads the current device's error word (bits SG_DEVERR_*, 0 when no
 * kernel has failed since the last clear) into *bits; clear != 0 resets it.
 * Synchronises `stream`: call it off the hot path (a health check, a test).
 * The word is process-wide per device. */
int sg_device_error(uint32_t* bits, int clear, sg_stream_t stream);

/* Test hook: the number of polls of sg_local_draft's first wait for a
 * row's bulk load; 0 makes that wait give up at once, a negative value
 * restores the default (2^22). A small bound lets a test make the wait run
 * out on purpose; the kernel still waits for the copy in flight with the
 * default bound before it exits. Applies to the launches that follow,
 * process-wide. Returns the previous bound. */
int sg_set_wait_polls(int polls);

/* ---- reference operator layer (suffix_gpu/triton_kernels.py) ----------- */

/* scatter_append (triton_kernels.py:392-402 / proposer.py:166-188):
 * token_ids[b, base[b] + j] = sampled[b, j] for j < min(T, cnt[b]) when
 * sampled != -1 and the position is < S. new_counts = base + cnt.
 * valid_count NULL: cnt = #(sampled[b, :] != -1). */
int sg_scatter_append(int32_t* token_ids, int64_t row_stride, int32_t batch,
                      int32_t seq_len, const int32_t* base,
                      const int32_t* valid_count, const int32_t* sampled,
                      int32_t sampled_cols, int32_t* new_counts,
                      sg_stream_t stream);

/* match_back (triton_kernels.py:259-281): out[b, i] = longest L <= P with
 * src[.., i-L:i] == the newest-first pattern pat[b, :L]; positions before
 * the buffer start read -1. row_stride 0 = one shared src of n_src
 * elements; otherwise src is [B, row_stride]. out is [B, n_out] int32. */
int sg_match_back(const int32_t* src, int64_t row_stride, int64_t n_src,
                  const int32_t* pat, int32_t batch, int32_t pat_len,
                  int64_t n_out, int32_t* out, sg_stream_t stream);

/* first_occurrences (triton_kernels.py:362-389): for each row of B*C
 * (row / C selects the mb row), the earliest R positions with
 * mb >= thr (thr <= 0: none), zero-padded, count clamped to R. */
int sg_first_occurrences(const int32_t* mb, int64_t n_cols,
                         const int64_t* thr, int32_t rows, int32_t cands,
                         int32_t max_occ, int64_t* out_pos,
                         int64_t* out_cnt, sg_stream_t stream);

/* expand_chain (suffix_gpu/expand.py:59-147, triton_kernels.py:305-338),
 * unweighted votes: cont [N, R, K] int32 (-1 = no token), num_occ [N],
 * cap [N] (NULL = K). Outputs chain [N, K] int32, num_valid [N] int64,
 * num_emit [N] int64, score [N] fp32. */
int sg_expand_chain(const int32_t* cont, int32_t rows, int32_t max_occ,
                    int32_t k, const int64_t* num_occ, const int64_t* cap,
                    float min_token_prob, float alpha, int32_t* chain,
                    int64_t* num_valid, int64_t* num_emit, float* score,
                    sg_stream_t stream);

/* ---- vLLM glue ----------------------------------------------------------- */

/* The per-step preparation of vLLM's GPU n-gram proposer
 * (vllm/v1/spec_decode/ngram_proposer_gpu.py, update_token_ids_ngram) in
 * one launch; no reference counterpart (the reference ships no vLLM
 * adapter). For each request row b < batch:
 *   valid_sampled[b, :] = sampled[b, :cols], or -1s when discard[b] != 0
 *   valid_count[b] = #(valid_sampled[b, j] != -1 and < vocab_size)
 *   next_ids[b] = valid_sampled[b, valid_count[b] - 1] if valid_count[b] > 0
 *                 else token_ids[b, clamp(num_tokens[b] - 1, 0, seq_len - 1)]
 * sampled is [batch, sampled_stride] (cols used), valid_sampled is
 * [batch, cols] contiguous, discard may be NULL (no discards). */
int sg_vllm_prepare(const int32_t* sampled, int64_t sampled_stride,
                    int32_t batch, int32_t cols, const uint8_t* discard,
                    const int32_t* token_ids, int64_t row_stride,
                    int32_t seq_len, const int32_t* num_tokens,
                    int64_t vocab_size, int32_t* next_ids,
                    int32_t* valid_count, int32_t* valid_sampled,
                    sg_stream_t stream);

/* ---- suffix array (suffix_gpu/suffix_array.py) -------------------------- */

/* Workspace bytes sg_build_suffix_array needs for n tokens (about 54 n:
 * two 8-byte key and two 4-byte value buffers, ranks, two active lists,
 * the large-group key / value / position lists and flags, plus per-tile
 * digit counts). */
size_t sg_suffix_array_workspace_size(int64_t n);

/* build_suffix_array (suffix_array.py:15-63): sa_out[0..n) = start
 * positions of the suffixes of tokens[0..n) in lexicographic order (signed
 * token order, end of string first). Identical to the reference's result
 * (the suffix array is unique). Prefix doubling over still-tied suffixes
 * with a device radix sort; the call reads the active count back once per
 * doubling round, so it synchronises `stream` (run it from its own host
 * thread / stream for a background rebuild). rounds_out (host pointer,
 * may be NULL) receives the number of doubling rounds after the initial
 * token sort. n < 2^31 - 1. */
int sg_build_suffix_array(const int32_t* tokens, int64_t n, int32_t* sa_out,
                          void* workspace, size_t workspace_bytes,
                          int32_t* rounds_out, sg_stream_t stream);

/* sg_build_suffix_array without any device allocation, for callers that
 * cannot allocate (an engine that has reserved all GPU memory up front, a
 * plugin host that only passes input and output buffers). No counterpart in
 * the reference. The workspace is an 8 MiB static __device__ array inside
 * this library (held by every GPU that loads it), so n is limited to the
 * largest n with sg_suffix_array_workspace_size(n) <= 8 MiB (about 155
 * thousand tokens); larger n returns SG_ERR_UNSUPPORTED without launching
 * anything. The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress); make that first call before any stream capture
 * begins. All calls share the array, which keeps the last call's contents:
 * calls whose work overlaps on the GPU (other streams, other host threads)
 * race and must be serialised by the caller. Synchronises `stream` like
 * sg_build_suffix_array. Nothing is allocated, on the device or the host:
 * the per-round count read-backs land in a small array on the calling
 * thread's stack. */
int sg_build_suffix_array_noalloc(const int32_t* tokens, int64_t n,
                                  int32_t* sa_out, int32_t* rounds_out,
                                  sg_stream_t stream);

/* Workspace bytes sg_suffix_array_append needs for n tokens (~48 n). */
size_t sg_suffix_array_append_workspace_size(int64_t n);

/* Incremental rebuild (the staging build of GlobalIndex._launch_rebuild,
 * global_index.py:147-223, without re-sorting the kept corpus; the
 * reference rebuilds from scratch). sa_out[0..n) = the suffix array of
 * tokens[0..n), identical to sg_build_suffix_array's, given:
 *   tokens[0..kept) == the previous snapshot's tokens[evicted..evicted+kept)
 *   prev_sa[0..prev_n) = the suffix array of the previous snapshot (length
 *     prev_n, evicted + kept <= prev_n),
 *   prev_rounds = the rounds its build reported (its longest common prefix
 *     of two suffixes is below 2^prev_rounds).
 * The suffixes with more than 2^prev_rounds kept tokens left keep their
 * previous order; the rest are sorted by the full builder and merged in.
 * rounds_out (host, may be NULL) receives the new snapshot's bound, to be
 * passed as prev_rounds to the next call. Synchronises `stream` like
 * sg_build_suffix_array; prev_sa and sa_out must not overlap. */
int sg_suffix_array_append(const int32_t* tokens, int64_t n,
                           const int32_t* prev_sa, int64_t prev_n,
                           int64_t evicted, int64_t kept,
                           int32_t prev_rounds, int32_t* sa_out,
                           void* workspace, size_t workspace_bytes,
                           int32_t* rounds_out, sg_stream_t stream);

/* ---- suffix-array search (suffix_gpu/sa_search.py) ---------------------- */

/* search_interval (sa_search.py:66-107, triton_kernels.py:284-302): SA
 * interval [start, end) of suffixes starting with each pattern row
 * pattern[b, :width] of length pattern_len[b], by the reference's fixed
 * ceil(log2(n+1))-iteration merged lower/upper bound search. */
int sg_sa_search(const int32_t* sa, const int32_t* corpus, int64_t n,
                 const int32_t* pattern, int32_t batch, int32_t width,
                 const int64_t* pattern_len, int64_t* out_start,
                 int64_t* out_end, sg_stream_t stream);

/* suffix_match_backoff (sa_search.py:110-163): for every row, searches the
 * suffixes of length 1..max_len of query[b, :query_len[b]] and, per cap c,
 * returns the longest found length <= caps[c] with its SA interval (0s when
 * none). Outputs [B, num_caps] int64. row_mask (may be NULL) skips rows. */
int sg_suffix_match_backoff(const int32_t* sa, const int32_t* corpus,
                            int64_t n, const int32_t* query, int32_t batch,
                            int32_t query_width, const int64_t* query_len,
                            int32_t max_len, const int64_t* caps,
                            int32_t num_caps, const uint8_t* row_mask,
                            int64_t* out_len, int64_t* out_start,
                            int64_t* out_end, sg_stream_t stream);

/* ---- global index (suffix_gpu/global_index.py) --------------------------- */

/* GlobalIndex.append_documents' device writes (global_index.py:86-108: per
 * document a slice copy, a SEP write and a length fill), batched: document
 * i (docs[i], lens[i] int32 tokens, device memory) is written to
 * buf[pos_i .. pos_i + lens[i]) followed by SEP = -2, with pos_0 = start and
 * pos_{i+1} = pos_i + lens[i] + 1; then *len_out (device int64, may be
 * NULL) = the end of the last document's SEP. One launch per 32 documents;
 * docs and lens are host arrays read during the call. Requires the end
 * <= capacity (else SG_ERR_INVALID, nothing launched). */
int sg_append_documents(int32_t* buf, int64_t capacity, int64_t start,
                        const int32_t* const* docs, const int64_t* lens,
                        int32_t n_docs, int64_t* len_out, sg_stream_t stream);

/* The delta's compaction (global_index.py:127-131, 191-199: the documents
 * before `from` left it): buf[0 .. count) = buf[from .. from + count)
 * (overlapping move, exact), then *len_out (device int64, may be NULL) =
 * count. One launch. */
int sg_delta_compact(int32_t* buf, int64_t capacity, int64_t from,
                     int64_t count, int64_t* len_out, sg_stream_t stream);

/* GlobalIndex._delta_match_backoff (global_index.py:465-546) over the delta
 * buffer; delta_len is a device int64 scalar. Outputs: out_len [B, C]
 * (min(longest match, cap)), out_pos [B, C, R] earliest start positions
 * (zero-padded), out_cnt [B, C] (clamped to R). num_caps <= 16. */
int sg_delta_match_backoff(const int32_t* delta, int64_t delta_capacity,
                           const int64_t* delta_len, const int32_t* query,
                           int32_t batch, int32_t query_width,
                           const int64_t* query_len, int32_t max_len,
                           const int64_t* caps, int32_t num_caps,
                           int32_t max_occ, const uint8_t* row_mask,
                           int64_t* out_len, int64_t* out_pos,
                           int64_t* out_cnt, sg_stream_t stream);

/* SuffixGPUDrafter._gather_tails (proposer.py:110-125): last
 * min(count, P) tokens of each row, oldest first, zero-padded to P. */
int sg_gather_tails(const int32_t* token_ids, int64_t row_stride,
                    int32_t seq_len, const int32_t* counts, int32_t batch,
                    int32_t pattern_len, int32_t* tails, int64_t* tail_len,
                    sg_stream_t stream);

/* The tails sg_gather_tails would return after update_state
 * (proposer.py:135-184) of these rows with these sampled ids (NULL: no
 * update, counts = base_counts), read from the buffer before the scatter
 * (it only reads positions the scatter leaves alone, so the local step may
 * update the rows concurrently on another stream); row_mask[b] receives
 * the drafting mask (propose_with_update: count > 0 and new count < limit;
 * propose: mask[b], or 1 when mask is NULL). No reference counterpart:
 * the reference gathers after the update (proposer.py:243-320). */
int sg_gather_tails_update(const int32_t* token_ids, int64_t row_stride,
                           int32_t seq_len, const int32_t* base_counts,
                           const int32_t* sampled, int32_t sampled_cols,
                           const int32_t* valid_count, int64_t limit,
                           const uint8_t* mask, int32_t batch,
                           int32_t pattern_len, int32_t* tails,
                           int64_t* tail_len, uint8_t* row_mask,
                           sg_stream_t stream);

/* Tail of GlobalIndex._query_backoff (global_index.py:321-370) and
 * _gather_cont (:443-463): SA-vs-delta choice per cap, adjacent-duplicate
 * removal, strided SA interval sampling, continuation block cont
 * [B, C, R, K] int32 (-1 padded), match_len / occ_count [B, C] int64, and
 * (spec_cap non-NULL) the spec cap of each candidate
 * (local_matcher.py:76-81). num_caps <= 16. */
int sg_global_candidates(const int64_t* sa_len, const int64_t* sa_start,
                         const int64_t* sa_end, const int64_t* d_len,
                         const int64_t* d_pos, const int64_t* d_cnt,
                         const int32_t* sa, const int32_t* corpus,
                         int64_t capacity, const int32_t* delta,
                         int64_t delta_capacity, const int64_t* delta_len,
                         int32_t batch, int32_t num_caps, int32_t max_occ,
                         int32_t k, int32_t has_spec_factor,
                         float spec_factor, float spec_offset,
                         int64_t* match_len, int32_t* cont,
                         int64_t* occ_count, int64_t* spec_cap,
                         sg_stream_t stream);

/* Final selection of SuffixGPUDrafter.propose (proposer.py:305-331): per
 * row, the first-maximum global candidate replaces the local draft (already
 * in draft / num_valid, as written by sg_local_draft) when its score is
 * strictly greater than local_score and the row may draft. */
int sg_global_combine(int32_t* draft, int32_t* num_valid,
                      const float* local_score, const uint8_t* row_mask,
                      const int32_t* g_chain, const int64_t* g_emit,
                      const float* g_score, int32_t batch, int32_t num_caps,
                      int32_t k, sg_stream_t stream);

/* The global half of SuffixGPUDrafter.propose after the two searches
 * (proposer.py:246-320), fused per row: sg_global_candidates' plan and
 * continuations (kept on chip, never written out), expand_chain with the
 * drafter's min_token_prob / alpha stopped at each candidate's spec cap,
 * and sg_global_combine's selection against the local winner in draft /
 * num_valid / local_score. Inputs are sg_suffix_match_backoff's and
 * sg_delta_match_backoff's outputs. max_occ <= 1024, k <= 64; returns
 * SG_ERR_UNSUPPORTED when the row's continuation block
 * (num_caps * max_occ * k int32 plus vote scratch) exceeds shared memory,
 * in which case the three separate calls apply. */
int sg_global_draft(const int64_t* sa_len, const int64_t* sa_start,
                    const int64_t* sa_end, const int64_t* d_len,
                    const int64_t* d_pos, const int64_t* d_cnt,
                    const int32_t* sa, const int32_t* corpus,
                    int64_t capacity, const int32_t* delta,
                    int64_t delta_capacity, const int64_t* delta_len,
                    int32_t batch, int32_t num_caps, int32_t max_occ,
                    int32_t k, int32_t has_spec_factor, float spec_factor,
                    float spec_offset, float min_token_prob, float alpha,
                    const float* local_score, const uint8_t* row_mask,
                    int32_t* draft, int32_t* num_valid, sg_stream_t stream);

/* ---- suffix-array shards (multi-GPU global drafter, benchmark config 5) ---
 * No reference counterpart: the reference has one suffix array on one
 * device. These calls split its query across GPUs without changing its
 * result: each GPU keeps the suffixes that start in its share of the corpus
 * (in suffix-array order, each with its global rank), searches every row
 * of the job on them, and the per-GPU results are summed by collectives
 * (see suffixgpu_b200/distributed.py). The reference behaviour reproduced
 * is suffix_match_backoff (sa_search.py:110-163) and the strided sample of
 * _query_backoff (global_index.py:339-352). */

/* Workspace bytes of sg_shard_extract for an n-entry suffix array. */
size_t sg_shard_extract_workspace_size(int64_t n);

/* The shard [lo, hi) of a whole-corpus suffix array sa[0..n): shard_pos[k]
 * = the k-th entry of sa whose position lies in [lo, hi) (sa order, so the
 * shard's own suffix array) and shard_rank[k] = its index in sa (its global
 * rank). Both outputs hold hi - lo entries (every position occurs once). */
int sg_shard_extract(const int32_t* sa, int64_t n, int64_t lo, int64_t hi,
                     int32_t* shard_pos, int32_t* shard_rank, void* workspace,
                     size_t workspace_bytes, sg_stream_t stream);

/* Packed query rows [batch, max_len + 2] int32: the tail (max_len tokens,
 * oldest first, sg_gather_tails' layout), the tail length and the drafting
 * flag (row_mask[b] != 0; all rows when row_mask is NULL). */
int sg_shard_pack_rows(const int32_t* tails, const int64_t* tail_len,
                       const uint8_t* row_mask, int32_t batch,
                       int32_t max_len, int32_t* rows, sg_stream_t stream);

/* Per packed row: out_len[b] = the longest l <= the tail length whose
 * last-l-token pattern starts some suffix of this shard (0: none, or the
 * row does not draft), or max_len + 1 when the tail holds a -1 token (a
 * pattern can then match past the corpus end, where tokens read -1, and
 * the found lengths need not be 1..L). The MAX over all shards is the
 * whole corpus's longest match: since a match of l tokens leaves one of
 * l - 1 tokens, the lengths found over the whole corpus are 1..that MAX,
 * and suffix_match_backoff's best length for cap c (sa_search.py:150-163)
 * is min(cap_c, MAX). One warp per row, binary search over l. */
int sg_shard_longest(const int32_t* shard_sa, int64_t shard_n,
                     const int32_t* corpus, int64_t corpus_n,
                     const int32_t* rows, int32_t batch, int32_t max_len,
                     int32_t* out_len, sg_stream_t stream);

/* Per packed row b and length l = 1..max_len: out_bounds[b, l-1, 0..1] =
 * (lower, upper) of the tail's last l tokens over the shard's suffix array
 * shard_sa[0..shard_n) (positions into corpus[0..corpus_n)): the number of
 * shard suffixes below the pattern and the number not above it, i.e. the
 * search_interval bounds on that array (sa_search.py:66-107, comparator
 * :25-63 with the whole corpus's end). Zeros for rows that do not draft and
 * lengths beyond the tail. Summed over all shards of a corpus they equal
 * search_interval on the whole suffix array. With `longest` (the MAX of
 * sg_shard_longest over the shards, [batch]) only the lengths
 * min(caps[c], longest[b]) are searched (every length when longest[b] >
 * max_len) and the others are zeros: enough for the per-cap selection.
 * max_len <= 128. */
int sg_shard_bounds(const int32_t* shard_sa, int64_t shard_n,
                    const int32_t* corpus, int64_t corpus_n,
                    const int32_t* rows, int32_t batch, int32_t max_len,
                    const int32_t* longest, const int64_t* caps,
                    int32_t num_caps, int32_t* out_bounds,
                    sg_stream_t stream);

/* From the summed bounds (bounds_sum, every shard's sg_shard_bounds added)
 * and this shard's own (bounds_local), per row and cap: the best length
 * (the longest <= cap and <= the tail length with a non-empty interval),
 * and samples[b, c, j] for j < R = the corpus position of sample j of that
 * interval (start + floor(j * ilen / R) when ilen > R, else start + j,
 * global ranks) when this shard holds it, else 0. Caps whose best length
 * equals the previous cap's get zeros (they share its samples). For rows
 * own_lo .. own_lo + own_n - 1, sa_len / sa_start / sa_end [own_n, C]
 * int64 receive sg_global_draft_samples' per-cap inputs: the best length
 * and the [start, end) slice of the samples array ([own_n, C, R] laid out
 * like samples' rows own_lo..) holding its min(ilen, R) samples in order.
 * num_caps <= 16. */
int sg_shard_resolve(const int32_t* bounds_sum, const int32_t* bounds_local,
                     const int32_t* rows, int32_t batch, int32_t max_len,
                     const int64_t* caps, int32_t num_caps, int32_t max_occ,
                     const int32_t* shard_pos, const int32_t* shard_rank,
                     int32_t* samples, int32_t own_lo, int32_t own_n,
                     int64_t* sa_len, int64_t* sa_start, int64_t* sa_end,
                     sg_stream_t stream);

/* sg_global_draft with the suffix array replaced by a block of resolved
 * samples (num_samples int32 corpus positions, indexed by sample_start /
 * sample_end from sg_shard_resolve). Same outputs and limits. */
int sg_global_draft_samples(
    const int64_t* sa_len, const int64_t* sample_start,
    const int64_t* sample_end, const int64_t* d_len, const int64_t* d_pos,
    const int64_t* d_cnt, const int32_t* samples, int64_t num_samples,
    const int32_t* corpus, int64_t capacity, const int32_t* delta,
    int64_t delta_capacity, const int64_t* delta_len, int32_t batch,
    int32_t num_caps, int32_t max_occ, int32_t k, int32_t has_spec_factor,
    float spec_factor, float spec_offset, float min_token_prob, float alpha,
    const float* local_score, const uint8_t* row_mask, int32_t* draft,
    int32_t* num_valid, sg_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* SUFFIXGPU_H_ */
