"""CPU oracle for the SuffixGPU draft path -- TEST INFRASTRUCTURE ONLY.

This module is a numpy restatement of the reference project's pure-PyTorch
CPU path (zip95297/SuffixGPU, ``suffix_gpu/*.py``). Every function cites the
reference file:line it follows. It exists to check the CUDA product path:
only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import it. The product package (``suffixgpu_b200``) never imports
it and has no CPU fallback.

Pinning: the restatement is checked bit-for-bit against golden vectors that
``tests/golden/make_golden.py`` produced by running the reference's own
torch CPU path in the build container (``tests/test_oracle_golden.py``).

Numerics follow torch's CPU semantics, verified in the build container:
a Python float scalar combined with a float32 tensor is first rounded to
float32 and the operation runs in float32 (mul, add, compare); float32
division is correctly rounded. numpy float32 arithmetic does the same.
"""

from __future__ import annotations

import math
from collections import deque

import numpy as np

PAD_TOKEN = np.iinfo(np.int32).max      # global_index.py:34
SEP_TOKEN = -2                           # global_index.py:38
_I64_MAX = np.iinfo(np.int64).max

f32 = np.float32


# ---------------------------------------------------------------------------
# expand.py
# ---------------------------------------------------------------------------
def majority_token(values: np.ndarray, active: np.ndarray, sentinel: int,
                   weights: np.ndarray | None = None,
                   chunk: int = 256) -> tuple[np.ndarray, np.ndarray]:
    """Pairwise-equality plurality vote per row (expand.py:16-56).

    Ties resolve to the smallest token id. Rows with no active entry get
    (sentinel, 0). Unweighted counts are int64; weighted counts float32.
    Rows are processed in chunks to bound the [N, R, R] temporary.
    """
    n, r = values.shape
    tok = np.empty(n, dtype=values.dtype)
    if weights is None:
        cnt = np.empty(n, dtype=np.int64)
    else:
        cnt = np.empty(n, dtype=np.float32)
    for s in range(0, n, chunk):
        v = values[s:s + chunk].astype(np.int64)
        a = active[s:s + chunk]
        eq = v[:, :, None] == v[:, None, :]
        if weights is None:
            votes = (eq & a[:, None, :]).sum(axis=2)
            votes = np.where(a, votes, 0)
        else:
            w = np.where(a, weights[s:s + chunk].astype(np.float32), f32(0))
            votes = (eq.astype(np.float32) * w[:, None, :]).sum(
                axis=2, dtype=np.float32)
            votes = np.where(a, votes, f32(0))
        max_cnt = votes.max(axis=1, keepdims=True)
        winner = a & (votes == max_cnt) & (max_cnt > 0)
        cand = np.where(winner, v, _I64_MAX)
        t = cand.min(axis=1)
        any_a = a.any(axis=1)
        tok[s:s + chunk] = np.where(any_a, t, sentinel).astype(values.dtype)
        mc = max_cnt[:, 0]
        cnt[s:s + chunk] = np.where(any_a, mc, np.zeros_like(mc))
    return tok, cnt


def expand_chain(cont: np.ndarray, num_occ: np.ndarray, k: int,
                 sentinel: int = -1, min_token_prob: float = 0.0,
                 cap: np.ndarray | None = None,
                 weights: np.ndarray | None = None,
                 alpha: float = 0.0):
    """Majority-vote chain expansion with fused scoring (expand.py:59-147).

    Returns (chain [N,k] int32, num_valid [N] i64, num_emit [N] i64,
    score [N] f32).
    """
    b, r, _ = cont.shape
    cont = cont.astype(np.int32)
    if cap is None:
        cap = np.full(b, k, dtype=np.int64)
    cap = np.asarray(cap).astype(np.int64)
    num_occ = np.asarray(num_occ).astype(np.int64)
    active = np.arange(r)[None, :] < num_occ[:, None]
    chain = np.full((b, k), sentinel, dtype=np.int32)
    prefix_ok = active.copy()
    cum_prob = np.ones(b, dtype=np.float32)
    score = np.zeros(b, dtype=np.float32)
    minp = f32(min_token_prob)
    al = f32(alpha)
    for d in range(k):
        col = cont[:, :, d]
        active_d = prefix_ok & (col != sentinel)
        tok, cnt = majority_token(col, active_d, sentinel, weights=weights)
        if weights is None:
            denom = np.maximum(active_d.sum(axis=1), 1).astype(np.float32)
        else:
            denom = np.where(active_d, weights.astype(np.float32),
                             f32(0)).sum(axis=1, dtype=np.float32)
        ratio = (cnt.astype(np.float32) / (denom + al)).astype(np.float32)
        cum_prob = (cum_prob * ratio).astype(np.float32)
        valid = (tok != sentinel) & (cnt > 0) & (cum_prob >= minp)
        chain[:, d] = np.where(valid, tok, chain[:, d])
        score = (score + np.where(valid & (cap > d), cum_prob,
                                  f32(0))).astype(np.float32)
        prefix_ok = prefix_ok & (col == tok[:, None]) & valid[:, None]
    filled = (chain != sentinel).astype(np.int64)
    num_valid = np.cumprod(filled, axis=1).sum(axis=1)
    num_emit = np.minimum(num_valid, np.maximum(cap, 0))
    return chain, num_valid, num_emit, score


# ---------------------------------------------------------------------------
# local_matcher.py
# ---------------------------------------------------------------------------
def spec_cap(match_len: np.ndarray, k: int, max_spec_factor: float | None,
             max_spec_offset: float) -> np.ndarray:
    """floor(f32(factor) * f32(L) + f32(offset)) clamped >= 0
    (local_matcher.py:76-81)."""
    match_len = np.asarray(match_len)
    if max_spec_factor is None:
        return np.full(match_len.shape, k, dtype=np.int64)
    prod = (f32(max_spec_factor) * match_len.astype(np.float32)).astype(
        np.float32)
    s = (prod + f32(max_spec_offset)).astype(np.float32)
    return np.maximum(np.floor(s).astype(np.int64), 0)


def match_back(src: np.ndarray, pat: np.ndarray, n_out: int) -> np.ndarray:
    """Rolling-AND longest common suffix (local_matcher.py:119-126,
    global_index.py:506-515).

    src is [B, S] (per-row buffer) or [N] (shared buffer); positions before
    the buffer start read -1. Returns [B, n_out] int32.
    """
    b, p = pat.shape
    shared = src.ndim == 1
    src = src.astype(np.int64)
    n_src = src.shape[-1]
    if shared:
        lp = np.concatenate([np.full(p, -1, np.int64), src])
    else:
        lp = np.concatenate([np.full((b, p), -1, np.int64), src], axis=1)
    need = p - 1 + n_out
    if lp.shape[-1] < need:  # n_out > n_src cannot occur on the hot path
        raise ValueError("n_out exceeds buffer")
    acc = np.ones((b, n_out), dtype=bool)
    mb = np.zeros((b, n_out), dtype=np.int32)
    pat = pat.astype(np.int64)
    for t in range(p):
        if shared:
            seg = lp[p - 1 - t:p - 1 - t + n_out][None, :]
        else:
            seg = lp[:, p - 1 - t:p - 1 - t + n_out]
        acc &= seg == pat[:, t:t + 1]
        mb += acc
    del n_src
    return mb


def first_occurrences_masked(mask: np.ndarray, r: int) -> tuple[np.ndarray,
                                                                 np.ndarray]:
    """Earliest r positions of each mask row, zero-padded; count clamped
    to r. Same result as the reference's smallest-k topk over position keys
    (local_matcher.py:170-184) and its early-exit scan kernel
    (triton_kernels.py:217-243).

    mask: [..., N] bool. Returns (pos [..., r] i64, count [..., ] i64).
    """
    lead = mask.shape[:-1]
    m2 = mask.reshape(-1, mask.shape[-1])
    rank = np.cumsum(m2, axis=1) - 1
    sel = m2 & (rank < r)
    rows, cols = np.nonzero(sel)
    out = np.zeros((m2.shape[0], r), dtype=np.int64)
    out[rows, rank[rows, cols]] = cols
    cnt = np.minimum(m2.sum(axis=1), r).astype(np.int64)
    return out.reshape(*lead, r), cnt.reshape(lead)


class LocalMatcher:
    """Restatement of LocalMatchKernel (local_matcher.py:49-242)."""

    def __init__(self, k: int, max_pattern_len: int = 32,
                 min_match_len: int = 1, max_occurrences: int = 32,
                 min_token_prob: float = 0.0,
                 max_spec_factor: float | None = None,
                 max_spec_offset: float = 0.0,
                 support_thresholds=(1, 2, 4, 8),
                 vote_smoothing_alpha: float = 0.0):
        self.k = k
        self.max_pattern_len = max_pattern_len
        self.min_match_len = max(1, min_match_len)
        self.max_occurrences = max_occurrences
        self.min_token_prob = min_token_prob
        self.max_spec_factor = max_spec_factor
        self.max_spec_offset = max_spec_offset
        self.vote_smoothing_alpha = vote_smoothing_alpha
        self.support_thresholds = tuple(int(t) for t in support_thresholds)
        if not self.support_thresholds:
            raise ValueError("support_thresholds must be non-empty")
        self._thresholds = np.array(self.support_thresholds, dtype=np.int64)

    def spec_cap(self, match_len):
        return spec_cap(match_len, self.k, self.max_spec_factor,
                        self.max_spec_offset)

    def gather_candidates(self, num_tokens, token_ids, combined_mask):
        """local_matcher.py:83-196 -> (cand [B,C] i64, cont [B,C,R,K] i32,
        occ_count [B,C] i64)."""
        token_ids = np.asarray(token_ids)
        b, s = token_ids.shape
        k, r, p = self.k, self.max_occurrences, self.max_pattern_len
        q = np.asarray(num_tokens).astype(np.int64)
        combined_mask = np.asarray(combined_mask).astype(bool)
        rows = np.arange(b)[:, None]
        # pattern, newest-first (local_matcher.py:107-112)
        pat_idx = q[:, None] - 1 - np.arange(p)[None, :]
        pat = np.where(pat_idx >= 0,
                       token_ids[rows, np.clip(pat_idx, 0, s - 1)], -2)
        mb = match_back(token_ids, pat, s)                    # :114-126
        pos = np.arange(s)
        valid_i = pos[None, :] < q[:, None]                   # :127-132
        mb = np.where(valid_i, mb, 0).astype(np.int32)
        # candidate per support threshold = t-th largest mb (:134-157)
        w_thr = min(max(self.support_thresholds), s)
        top_mb = -np.sort(-mb.astype(np.int64), axis=1)[:, :w_thr]
        tidx = np.clip(self._thresholds - 1, 0, w_thr - 1)
        cand = top_mb[:, tidx].astype(np.int64)
        cand = np.where(self._thresholds[None, :] > w_thr, 0, cand)
        cand = np.where((cand >= self.min_match_len)
                        & combined_mask[:, None], cand, 0)
        if cand.shape[1] > 1:
            dup = np.zeros_like(cand, dtype=bool)
            dup[:, 1:] = cand[:, 1:] == cand[:, :-1]
            cand = np.where(dup, 0, cand)
        # earliest occurrences (:160-184)
        mask = (valid_i[:, None, :] & (mb[:, None, :] >= cand[:, :, None])
                & (cand > 0)[:, :, None])
        occ_end, occ_count = first_occurrences_masked(mask, r)
        # continuation gather (:186-195)
        idx = occ_end[..., None] + np.arange(k)[None, None, None, :]
        row_active = (np.arange(r)[None, None, :]
                      < occ_count[:, :, None])[..., None]
        valid_idx = (idx < q[:, None, None, None]) & row_active
        vals = token_ids[np.arange(b)[:, None, None, None],
                         np.clip(idx, 0, s - 1)]
        cont = np.where(valid_idx, vals, -1).astype(np.int32)
        return cand, cont, occ_count

    def forward(self, num_tokens, token_ids, combined_mask):
        """local_matcher.py:198-242 -> (draft [B,K] i32, num_valid [B] i32,
        match_len [B] i64, occ [B] i64, score [B] f32)."""
        b = np.asarray(token_ids).shape[0]
        k, r = self.k, self.max_occurrences
        cand, cont, occ_count = self.gather_candidates(
            num_tokens, token_ids, combined_mask)
        c = cand.shape[1]
        cap = self.spec_cap(cand.reshape(b * c))
        chain, _, num_emit, score = expand_chain(
            cont.reshape(b * c, r, k), occ_count.reshape(b * c), k,
            min_token_prob=self.min_token_prob, cap=cap,
            alpha=self.vote_smoothing_alpha)
        sel = select_local_best(cand, chain.reshape(b, c, k),
                                num_emit.reshape(b, c),
                                occ_count.reshape(b, c), score.reshape(b, c))
        sel_chain, sel_emit, sel_len, sel_occ, sel_score = sel
        slot = np.arange(k)[None, :]
        sel_chain = np.where(slot < sel_emit[:, None], sel_chain, -1)
        return (sel_chain.astype(np.int32), sel_emit.astype(np.int32),
                sel_len, sel_occ, sel_score)


def select_local_best(cand, chain, num_emit, occ, score):
    """argmax(score + f32(cand) * 1e-6), first max (local_matcher.py:
    245-263)."""
    b = cand.shape[0]
    tie = (cand.astype(np.float32) * f32(1e-6)).astype(np.float32)
    best = (score + tie).astype(np.float32).argmax(axis=1)
    bi = np.arange(b)
    return (chain[bi, best], num_emit[bi, best], cand[bi, best],
            occ[bi, best], score[bi, best])


# ---------------------------------------------------------------------------
# suffix_array.py
# ---------------------------------------------------------------------------
def build_suffix_array(tokens: np.ndarray, early_exit: bool = True
                       ) -> np.ndarray:
    """Prefix doubling with packed int64 keys (suffix_array.py:15-63).

    ``early_exit`` stops once every rank is distinct; later rounds are a
    fixpoint (argsort of distinct ranks reproduces the same order), so the
    result equals the reference's fixed ``ceil(log2 n)`` rounds.
    """
    tokens = np.asarray(tokens).reshape(-1)
    n = tokens.shape[0]
    if n == 0:
        return np.empty(0, dtype=np.int64)
    if n == 1:
        return np.zeros(1, dtype=np.int64)
    rank = np.unique(tokens.astype(np.int64), return_inverse=True)[1]
    rank = rank.reshape(-1).astype(np.int64)
    base = n + 1
    sa = np.argsort(rank, kind="stable")
    k = 1
    rounds = max(1, math.ceil(math.log2(n)))
    for _ in range(rounds):
        second = np.zeros(n, dtype=np.int64)
        if k < n:
            second[:-k] = rank[k:] + 1
        key = rank * base + second
        sa = np.argsort(key, kind="stable")
        sorted_key = key[sa]
        distinct = np.ones(n, dtype=np.int64)
        distinct[1:] = (sorted_key[1:] != sorted_key[:-1])
        new_rank_sorted = np.cumsum(distinct) - 1
        new_rank = np.empty_like(rank)
        new_rank[sa] = new_rank_sorted
        rank = new_rank
        k *= 2
        if early_exit and new_rank_sorted[-1] == n - 1:
            break
    return sa.astype(np.int64)


# ---------------------------------------------------------------------------
# sa_search.py
# ---------------------------------------------------------------------------
def cmp_pattern(sa, corpus, mid, pattern, pattern_len):
    """-1 / 0 / 1 comparison of SA suffixes vs padded patterns
    (sa_search.py:25-63)."""
    n = sa.shape[0]
    m = pattern.shape[1]
    pos = sa[mid].astype(np.int64)
    offs = np.arange(m)
    idx = pos[:, None] + offs[None, :]
    valid_pos = idx < n
    tok = np.where(valid_pos, corpus[np.clip(idx, 0, n - 1)], -1).astype(
        np.int64)
    pat_valid = offs[None, :] < pattern_len[:, None]
    eq_ok = (tok == pattern) | ~pat_valid
    lcp_raw = np.cumprod(eq_ok.astype(np.int64), axis=1).sum(axis=1)
    lcp = np.minimum(lcp_raw, pattern_len)
    full = lcp >= pattern_len
    spos = np.clip(pos + lcp, 0, n - 1)
    schar = np.where(pos + lcp < n, corpus[spos], -1).astype(np.int64)
    pchar = pattern[np.arange(pattern.shape[0]), np.minimum(lcp, m - 1)]
    cmp_ = np.where(schar < pchar, -1, np.where(schar > pchar, 1, 0))
    return np.where(full, 0, cmp_)


def search_interval(sa, corpus, pattern, pattern_len):
    """Merged fixed-iteration lower/upper bound search (sa_search.py:
    66-107). Returns (start [B] i64, end [B] i64)."""
    sa = np.asarray(sa)
    corpus = np.asarray(corpus).astype(np.int64)
    pattern = np.asarray(pattern).astype(np.int64)
    pattern_len = np.asarray(pattern_len).astype(np.int64)
    n = sa.shape[0]
    iters = max(1, math.ceil(math.log2(n + 1)))
    b = pattern.shape[0]
    pat2 = np.concatenate([pattern, pattern], axis=0)
    plen2 = np.concatenate([pattern_len, pattern_len], axis=0)
    is_upper = np.zeros(2 * b, dtype=bool)
    is_upper[b:] = True
    lo = np.zeros(2 * b, dtype=np.int64)
    hi = np.full(2 * b, n, dtype=np.int64)
    for _ in range(iters):
        mid = np.minimum((lo + hi) // 2, n - 1)
        c = cmp_pattern(sa, corpus, mid, pat2, plen2)
        go_right = (c < 0) | (is_upper & (c == 0))
        lo = np.where(go_right, mid + 1, lo)
        hi = np.where(go_right, hi, mid)
    return lo[:b], lo[b:]


def suffix_match_backoff(sa, corpus, query, query_len, max_len, caps):
    """Per-cap longest suffix match from one SA walk over lengths
    1..max_len (sa_search.py:110-163). Returns (match_len [B,C] i64,
    start [B,C] i64, end [B,C] i64)."""
    query = np.asarray(query).astype(np.int64)
    query_len = np.asarray(query_len).astype(np.int64)
    caps = np.asarray(caps).astype(np.int64)
    b, q = query.shape
    m = max_len
    lengths = np.arange(1, m + 1, dtype=np.int64)
    offs = np.arange(m, dtype=np.int64)
    idx = (query_len[:, None, None] - lengths[None, :, None]
           + offs[None, None, :])
    valid = (offs[None, None, :] < lengths[None, :, None]) & (idx >= 0)
    tok = query[np.arange(b)[:, None, None], np.clip(idx, 0, q - 1)]
    pat = np.where(valid, tok, 0)
    start, end = search_interval(sa, corpus, pat.reshape(b * m, m),
                                 np.broadcast_to(lengths, (b, m)).reshape(-1))
    start = start.reshape(b, m)
    end = end.reshape(b, m)
    found = (end > start) & (lengths[None, :] <= query_len[:, None])
    found_len = found.astype(np.int64) * lengths[None, :]
    within = lengths[None, None, :] <= caps[None, :, None]
    best = (found_len[:, None, :] * within).max(axis=2)
    pick = np.maximum(best - 1, 0)
    s_best = np.take_along_axis(start, pick, axis=1)
    e_best = np.take_along_axis(end, pick, axis=1)
    return best, np.where(best > 0, s_best, 0), np.where(best > 0, e_best, 0)


def longest_suffix_match(sa, corpus, query, query_len, max_len):
    """Single-cap special case (sa_search.py:166-185)."""
    caps = np.array([max_len], dtype=np.int64)
    best, s, e = suffix_match_backoff(sa, corpus, query, query_len, max_len,
                                      caps)
    return best[:, 0], s[:, 0], e[:, 0]


# ---------------------------------------------------------------------------
# global_index.py
# ---------------------------------------------------------------------------
class NeverDoneEvent:
    """Host-side fake of an in-flight rebuild event."""

    def query(self) -> bool:
        return False


class GlobalIndex:
    """Restatement of GlobalIndex (global_index.py:41-553). Device tensors
    become numpy arrays; rebuilds are synchronous (the reference's CPU
    behaviour, global_index.py:204-215)."""

    def __init__(self, capacity, delta_capacity, k, max_occurrences=32,
                 rebuild_threshold=None):
        self.capacity = capacity
        self.delta_capacity = delta_capacity
        self.k = k
        self.max_occurrences = max_occurrences
        self.rebuild_threshold = rebuild_threshold or max(
            1, delta_capacity // 2)
        self.corpus = np.full(capacity, PAD_TOKEN, dtype=np.int32)
        self.staging_corpus = self.corpus.copy()
        self.sa = np.arange(capacity, dtype=np.int32)
        self.staging_sa = self.sa.copy()
        self.delta = np.zeros(delta_capacity, dtype=np.int32)
        self.delta_len_t = 0
        self.active_len = 0
        self.delta_len = 0
        self.active_doc_lens: deque[int] = deque()
        self.delta_doc_lens: list[int] = []
        self._rebuild_event = None
        self._pending = None
        self.rebuilds = 0

    # writes (global_index.py:86-133)
    def append_documents(self, docs) -> None:
        for doc in docs:
            doc = np.asarray(doc).astype(np.int32).reshape(-1)
            n = doc.shape[0]
            if n == 0:
                continue
            if n + 1 > self.delta_capacity:
                doc = doc[-(self.delta_capacity - 1):]
                n = doc.shape[0]
            if self.delta_len + n + 1 > self.delta_capacity:
                self._make_room(n + 1)
            self.delta[self.delta_len:self.delta_len + n] = doc
            self.delta[self.delta_len + n] = SEP_TOKEN
            self.delta_len += n + 1
            self.delta_len_t = self.delta_len
            self.delta_doc_lens.append(n + 1)
        self.maybe_rebuild()

    def _make_room(self, needed: int) -> None:
        self.poll_rebuild()
        if self._rebuild_event is None:
            self._launch_rebuild()
        if self.delta_len + needed <= self.delta_capacity:
            return
        self._drop_oldest_docs(self.delta_len + needed - self.delta_capacity)

    def _drop_oldest_docs(self, drop: int) -> None:
        acc = 0
        docs_dropped = 0
        for ln in self.delta_doc_lens:
            if acc >= drop:
                break
            acc += ln
            docs_dropped += 1
        remaining = self.delta_len - acc
        if remaining > 0:
            self.delta[:remaining] = self.delta[acc:self.delta_len].copy()
        self.delta_len = remaining
        self.delta_len_t = remaining
        self.delta_doc_lens = self.delta_doc_lens[docs_dropped:]

    # rebuild (global_index.py:138-253)
    def maybe_rebuild(self) -> None:
        self.poll_rebuild()
        if self._rebuild_event is not None or self.delta_len == 0:
            return
        if self.delta_len < self.rebuild_threshold:
            return
        self._launch_rebuild()

    def _launch_rebuild(self) -> None:
        if self._rebuild_event is not None:
            return
        keep_start = 0
        for ln in self.active_doc_lens:
            if self.active_len - keep_start + self.delta_len \
                    <= self.capacity:
                break
            keep_start += ln
        n_active_keep = self.active_len - keep_start
        snap = min(self.delta_len, self.capacity - n_active_keep)
        acc = 0
        for ln in self.delta_doc_lens:
            if acc + ln <= snap:
                acc += ln
            else:
                break
        snap = acc
        n_new = n_active_keep + snap
        if n_new == 0:
            return
        dst = self.staging_corpus
        dst[:] = PAD_TOKEN
        if n_active_keep > 0:
            dst[:n_active_keep] = self.corpus[keep_start:self.active_len]
        if snap > 0:
            dst[n_active_keep:n_new] = self.delta[:snap]
        new_doc_lens: deque[int] = deque()
        acc = 0
        for ln in self.active_doc_lens:
            acc += ln
            if acc > keep_start:
                new_doc_lens.append(ln)
        acc = 0
        for ln in self.delta_doc_lens:
            acc += ln
            if acc <= snap:
                new_doc_lens.append(ln)
        docs_absorbed = self._count_docs_within(snap)
        remaining = self.delta_len - snap
        if remaining > 0:
            self.delta[:remaining] = self.delta[snap:self.delta_len].copy()
        self.delta_len = remaining
        self.delta_len_t = remaining
        self.delta_doc_lens = self.delta_doc_lens[docs_absorbed:]
        m = min(n_new + 1, self.capacity)
        self._build_staging_sa(dst, m)
        self._finish_swap(n_new, new_doc_lens)

    def _build_staging_sa(self, dst, m) -> None:
        self.staging_sa[:m] = build_suffix_array(dst[:m]).astype(np.int32)
        if m < self.capacity:
            self.staging_sa[m:] = np.arange(m, self.capacity, dtype=np.int32)

    def _count_docs_within(self, tokens: int) -> int:
        acc = 0
        count = 0
        for ln in self.delta_doc_lens:
            acc += ln
            if acc > tokens:
                break
            count += 1
        return count

    def _finish_swap(self, n_new, new_doc_lens) -> None:
        self.corpus[:] = self.staging_corpus
        self.sa[:] = self.staging_sa
        self.active_len = n_new
        self.active_doc_lens = new_doc_lens
        self._rebuild_event = None
        self._pending = None
        self.rebuilds += 1

    def poll_rebuild(self) -> None:
        if self._rebuild_event is None:
            return
        if self._rebuild_event.query():
            n_new, new_doc_lens = self._pending
            self._finish_swap(n_new, new_doc_lens)

    def load_documents(self, docs) -> None:
        """Bulk form of harvesting (the product's GlobalIndex.load_documents;
        no reference counterpart), stated literally: the documents (each
        trimmed to its last capacity - 1 tokens so that it fits with its SEP)
        go to an otherwise empty, unbounded delta, and the reference's
        rebuild (global_index.py:147-223) runs until the delta is empty."""
        if self.delta_len:
            raise ValueError("load_documents needs an empty delta")
        docs = [np.asarray(d).astype(np.int32).reshape(-1) for d in docs]
        docs = [d[-(self.capacity - 1):] for d in docs if d.size > 0]
        saved_cap = self.delta_capacity
        total = sum(d.size + 1 for d in docs)
        self.delta = np.zeros(max(total, 1), dtype=np.int32)
        self.delta_capacity = self.delta.size
        for d in docs:
            n = d.size
            self.delta[self.delta_len:self.delta_len + n] = d
            self.delta[self.delta_len + n] = SEP_TOKEN
            self.delta_len += n + 1
            self.delta_doc_lens.append(n + 1)
        self.delta_len_t = self.delta_len
        while self.delta_len > 0:
            before = self.delta_len
            self._launch_rebuild()
            if self.delta_len == before:
                break
        self.delta = np.zeros(saved_cap, dtype=np.int32)
        self.delta_capacity = saved_cap
        self.delta_len = 0
        self.delta_len_t = 0
        self.delta_doc_lens = []

    # queries (global_index.py:257-370, 443-553)
    def query(self, query, query_len, max_len):
        caps = np.array([max_len], dtype=np.int64)
        ml, cont, occ = self._query_backoff(query, query_len, max_len, caps)
        return ml[:, 0], cont[:, 0], occ[:, 0]

    def _query_backoff(self, query, query_len, max_len, caps):
        query = np.asarray(query)
        query_len = np.asarray(query_len).astype(np.int64)
        caps = np.asarray(caps).astype(np.int64)
        b = query.shape[0]
        cnum = caps.shape[0]
        r = self.max_occurrences
        sa_len, sa_start, sa_end = suffix_match_backoff(
            self.sa, self.corpus, query, query_len, max_len, caps)
        d_len, d_pos, d_cnt = self._delta_match_backoff(
            query, query_len, max_len, caps)
        use_sa = (sa_len >= d_len) & (sa_len > 0)
        use_delta = (d_len > sa_len) & (d_len > 0)
        zero = np.zeros((b, cnum), dtype=np.int64)
        match_len = np.where(use_sa, sa_len,
                             np.where(use_delta, d_len, zero))
        if cnum > 1:
            src = use_sa.astype(np.int8) + 2 * use_delta.astype(np.int8)
            dup = np.zeros_like(use_sa)
            dup[:, 1:] = ((match_len[:, 1:] == match_len[:, :-1])
                          & (src[:, 1:] == src[:, :-1])
                          & (match_len[:, 1:] > 0))
            use_sa = use_sa & ~dup
            use_delta = use_delta & ~dup
            match_len = np.where(dup, zero, match_len)
        offs = np.arange(r, dtype=np.int64)
        ilen = sa_end - sa_start
        strided = sa_start[:, :, None] + (offs[None, None, :]
                                          * ilen[:, :, None]) // r
        seq = sa_start[:, :, None] + offs[None, None, :]
        sa_idx = np.clip(np.where((ilen > r)[:, :, None], strided, seq), 0,
                         self.capacity - 1)
        sa_cnt = np.minimum(ilen, r)
        take = offs[None, None, :] < sa_cnt[:, :, None]
        pos = self.sa[sa_idx.reshape(-1)].reshape(b, cnum, r).astype(
            np.int64)
        sa_occ = np.where(take, pos, 0)
        flat_len = match_len.reshape(b * cnum)
        sa_cont = self._gather_cont(
            self.corpus, self.capacity, sa_occ.reshape(b * cnum, r),
            sa_cnt.reshape(b * cnum), flat_len, use_sa.reshape(b * cnum))
        d_cont = self._gather_cont(
            self.delta, self.delta_len_t, d_pos.reshape(b * cnum, r),
            d_cnt.reshape(b * cnum), flat_len, use_delta.reshape(b * cnum))
        cont = np.full((b * cnum, r, self.k), -1, dtype=np.int32)
        sel_sa = use_sa.reshape(b * cnum, 1, 1)
        sel_delta = use_delta.reshape(b * cnum, 1, 1)
        cont = np.where(sel_sa, sa_cont, cont)
        cont = np.where(sel_delta, d_cont, cont)
        occ_count = np.where(use_sa, sa_cnt,
                             np.where(use_delta, d_cnt, zero))
        return match_len, cont.reshape(b, cnum, r, self.k), occ_count

    def _gather_cont(self, src, src_len, occ_pos, occ_cnt, match_len, sel):
        b, r = occ_pos.shape
        n = src.shape[0]
        row = np.arange(r)[None, :]
        row_active = (row < occ_cnt[:, None]) & sel[:, None]
        idx = (occ_pos[:, :, None] + match_len[:, None, None]
               + np.arange(self.k)[None, None, :])
        valid = row_active[:, :, None] & (idx < src_len) & (idx >= 0)
        vals = src[np.clip(idx, 0, n - 1)].astype(np.int64)
        ok = valid & (vals != PAD_TOKEN) & (vals >= 0)
        return np.where(ok, vals, -1).astype(np.int32)

    def _delta_match_backoff(self, query, query_len, max_len, caps):
        query = np.asarray(query).astype(np.int64)
        query_len = np.asarray(query_len).astype(np.int64)
        caps = np.asarray(caps).astype(np.int64)
        b = query.shape[0]
        cnum = caps.shape[0]
        r = self.max_occurrences
        cap = self.delta_capacity
        q = query.shape[1]
        n_i = cap + 1
        offs = np.arange(max_len)
        pat_idx = query_len[:, None] - 1 - offs[None, :]
        pat = np.where(pat_idx >= 0,
                       query[np.arange(b)[:, None],
                             np.clip(pat_idx, 0, q - 1)], -3)
        mb = match_back(self.delta, pat, n_i)
        pos_i = np.arange(n_i)
        valid_i = pos_i[None, :] <= self.delta_len_t
        mb = np.where(valid_i, mb, 0)
        lo_full = mb.max(axis=1).astype(np.int64)
        lo = np.minimum(lo_full[:, None], caps[None, :])
        mask = (valid_i[:, None, :] & (mb[:, None, :] >= lo[:, :, None])
                & (lo > 0)[:, :, None])
        occ_end, cnt = first_occurrences_masked(mask, r)
        occ = np.maximum(occ_end - lo[:, :, None], 0)
        return lo, occ, cnt

    def expand(self, cont, occ_count, min_token_prob=0.0):
        chain, num_valid, _, _ = expand_chain(
            cont, occ_count, self.k, min_token_prob=min_token_prob)
        return chain, num_valid


# ---------------------------------------------------------------------------
# proposer.py
# ---------------------------------------------------------------------------
def global_caps(max_pattern_len: int, num_backoff: int) -> list[int]:
    """Descending global length caps (proposer.py:78-87)."""
    nb = max(1, int(num_backoff))
    if nb == 1:
        caps = [max_pattern_len]
    else:
        caps = [max(2, max_pattern_len >> i) for i in range(nb - 1)] + [2]
    return sorted(set(caps), reverse=True)


class SuffixDrafter:
    """Restatement of SuffixGPUDrafter (proposer.py:26-393) on CPU."""

    def __init__(self, k, max_pattern_len=32, min_match_len=1,
                 max_occurrences=128, enable_global=False,
                 global_capacity=1 << 22, delta_capacity=1 << 16,
                 rebuild_threshold=None, max_spec_factor=None,
                 max_spec_offset=0.0, min_token_prob=0.0, num_backoff=8,
                 vote_smoothing_alpha=0.0):
        self.k = k
        self.max_pattern_len = max_pattern_len
        self.max_spec_factor = max_spec_factor
        self.max_spec_offset = max_spec_offset
        self.min_token_prob = min_token_prob
        self.num_backoff = max(1, int(num_backoff))
        self.vote_smoothing_alpha = float(vote_smoothing_alpha)
        thresholds = tuple(2 ** i for i in range(self.num_backoff))
        self._global_caps = np.array(
            global_caps(max_pattern_len, self.num_backoff), dtype=np.int64)
        self.local = LocalMatcher(
            k=k, max_pattern_len=max_pattern_len,
            min_match_len=min_match_len, max_occurrences=max_occurrences,
            min_token_prob=min_token_prob, max_spec_factor=max_spec_factor,
            max_spec_offset=max_spec_offset, support_thresholds=thresholds,
            vote_smoothing_alpha=self.vote_smoothing_alpha)
        self.global_index = None
        self._ingested: dict = {}
        if enable_global:
            self.global_index = GlobalIndex(
                global_capacity, delta_capacity, k,
                max_occurrences=max_occurrences,
                rebuild_threshold=rebuild_threshold)

    def _gather_tails(self, num_tokens, token_ids):
        """proposer.py:110-125."""
        b, s = token_ids.shape
        p = self.max_pattern_len
        q_len = np.asarray(num_tokens).astype(np.int64)
        tail_len = np.minimum(q_len, p)
        offs = np.arange(p)
        idx = q_len[:, None] - tail_len[:, None] + offs[None, :]
        valid = offs[None, :] < tail_len[:, None]
        tails = np.where(valid, token_ids[np.arange(b)[:, None],
                                          np.clip(idx, 0, s - 1)], 0)
        return tails.astype(np.int32), tail_len

    def poll(self) -> None:
        if self.global_index is not None:
            self.global_index.poll_rebuild()

    def update_state(self, num_tokens, token_ids, sampled,
                     valid_sampled_tokens_count=None):
        """In-place scatter of sampled ids (proposer.py:135-184)."""
        b, s = token_ids.shape
        t = sampled.shape[1]
        base = np.asarray(num_tokens).astype(np.int64)
        if valid_sampled_tokens_count is None:
            valid_sampled_tokens_count = (sampled != -1).sum(axis=1)
        cnt = np.asarray(valid_sampled_tokens_count).astype(np.int64)
        rows = np.arange(b)
        for j in range(t):
            pos_j = np.minimum(base + j, s - 1)
            ok_j = (j < cnt) & (sampled[:, j] != -1) & (base + j < s)
            old_j = token_ids[rows, pos_j]
            val_j = np.where(ok_j, sampled[:, j].astype(token_ids.dtype),
                             old_j)
            token_ids[rows, pos_j] = val_j
        return (base + cnt).astype(np.int32)

    def propose_with_update(self, num_tokens, token_ids, sampled,
                            valid_sampled_tokens_count=None,
                            max_model_len=None):
        """proposer.py:186-214."""
        if valid_sampled_tokens_count is None:
            valid_sampled_tokens_count = (sampled != -1).sum(axis=1)
        new_counts = self.update_state(num_tokens, token_ids, sampled,
                                       valid_sampled_tokens_count)
        mask = np.asarray(valid_sampled_tokens_count).astype(np.int64) > 0
        s = token_ids.shape[1]
        limit = s if max_model_len is None else min(max_model_len, s)
        mask &= new_counts.astype(np.int64) < limit
        draft, num_valid = self.propose(new_counts, token_ids, mask)
        return draft, num_valid, new_counts

    def propose(self, num_tokens, token_ids, combined_mask=None):
        """proposer.py:216-327."""
        num_tokens = np.asarray(num_tokens)
        b = num_tokens.shape[0]
        k = self.k
        if combined_mask is None:
            combined_mask = np.ones(b, dtype=bool)
        combined_mask = np.asarray(combined_mask).astype(bool)
        if self.global_index is None:
            draft, num_valid, _, _, _ = self.local.forward(
                num_tokens, token_ids, combined_mask)
        else:
            r = self.local.max_occurrences
            tails, tail_len = self._gather_tails(num_tokens, token_ids)
            cand_l, cont_l, occ_l = self.local.gather_candidates(
                num_tokens, token_ids, combined_mask)
            g_len, g_cont, g_occ = self.global_index._query_backoff(
                tails, tail_len, self.max_pattern_len, self._global_caps)
            cl = cand_l.shape[1]
            cg = g_len.shape[1]
            len_all = np.concatenate([cand_l, g_len], axis=1)
            cont_all = np.concatenate([cont_l, g_cont], axis=1)
            occ_all = np.concatenate([occ_l, g_occ], axis=1)
            cap_all = self.local.spec_cap(len_all.reshape(-1))
            chain, _, emit, score = expand_chain(
                cont_all.reshape(b * (cl + cg), r, k), occ_all.reshape(-1),
                k, min_token_prob=self.min_token_prob, cap=cap_all,
                alpha=self.vote_smoothing_alpha)
            chain = chain.reshape(b, cl + cg, k)
            emit = emit.reshape(b, cl + cg)
            score = score.reshape(b, cl + cg)
            l_chain, l_emit, _, _, l_score = select_local_best(
                cand_l, chain[:, :cl], emit[:, :cl], occ_all[:, :cl],
                score[:, :cl])
            g_score_all = score[:, cl:]
            best_g = g_score_all.argmax(axis=1)
            bi = np.arange(b)
            g_chain = chain[:, cl:][bi, best_g]
            g_emit = emit[:, cl:][bi, best_g]
            g_score = g_score_all[bi, best_g]
            pick_global = (g_score > l_score) & combined_mask
            draft = np.where(pick_global[:, None], g_chain, l_chain)
            num_valid = np.where(pick_global, g_emit,
                                 l_emit.astype(np.int64))
        num_valid = np.where(combined_mask, num_valid.astype(np.int64), 0)
        slot = np.arange(k)[None, :]
        draft = np.where(slot < num_valid[:, None], draft, -1)
        return draft.astype(np.int32), num_valid.astype(np.int32)

    def harvest_finished(self, row_indices, lengths, token_ids):
        rows = [token_ids[r] for r in row_indices]
        self.harvest_rows(rows, lengths)

    def harvest_rows(self, rows, lengths):
        if self.global_index is None or not rows:
            return
        docs = [row[:ln] for row, ln in zip(rows, lengths) if ln > 0]
        if docs:
            self.global_index.append_documents(docs)

    def ingest_active(self, keys, rows, lengths, final=False, chunk=64):
        """proposer.py:354-390."""
        if self.global_index is None:
            return
        overlap = self.max_pattern_len + self.k
        docs = []
        for key, row, ln in zip(keys, rows, lengths):
            done = self._ingested.get(key, 0)
            if ln - done >= chunk or (final and ln > done):
                start = max(0, done - overlap)
                docs.append(row[start:ln])
                self._ingested[key] = ln
            if final:
                self._ingested.pop(key, None)
        if docs:
            self.global_index.append_documents(docs)
