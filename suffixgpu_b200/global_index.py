"""GlobalIndex: cross-request memory (suffix array over finished responses
plus an append-only delta buffer), the reference's GlobalIndex
(suffix_gpu/global_index.py:41-553) on the sm_100a kernels.

State and rules are the reference's (what a caller can observe: corpus,
suffix array, delta, document lengths, when rebuilds happen and what they
evict or absorb); the implementation is this package's. Document lengths
live in two ``DocLedger`` queues of running totals (doc_ledger.py), so a
rebuild's eviction and absorption come from binary searches, and the
device writes of a harvest are one C-ABI call (sg_append_documents: all
documents and their SEPs in one launch, the device length included), as
is the delta's compaction (sg_delta_compact). Queries go through
sg_suffix_match_backoff + sg_delta_match_backoff + the fused global step.
The active corpus / SA keep their storage across swaps (in-place copies),
so captured CUDA graphs stay valid.

Rebuilds run synchronously without a rebuild stream (the reference's
behaviour on CPU and without one). With ``rebuild_stream`` set, the
staging build runs on that stream from a background host thread and the
swap happens at the first ``poll_rebuild`` after it has finished, as in the
reference.
"""

from __future__ import annotations

import ctypes
import queue
import threading
import time
import weakref
from collections import deque

import torch

from suffixgpu_b200 import ops
from suffixgpu_b200._lib import call, check, lib, ptr, stream_of, torch_ops
from suffixgpu_b200.doc_ledger import DocLedger, plan_bulk_load, plan_snapshot

PAD_TOKEN = torch.iinfo(torch.int32).max
SEP_TOKEN = -2
_UNSUPPORTED = 4  # SG_ERR_UNSUPPORTED
# Incremental rebuilds only while the active SA's common prefixes are below
# 2^12 tokens: the merge re-sorts the last 2^rounds kept tokens and its
# comparisons can run that deep (on a corpus of exactly repeated 256K-token
# stretches the merge took 12 ms against 4.2 ms for a full build).
_APPEND_MAX_ROUNDS = 12


class _ThreadEvent:
    """Completion flag of a background build (query() like a CUDA event)."""

    def __init__(self):
        self._done = threading.Event()
        self.error: BaseException | None = None

    def set(self):
        self._done.set()

    def query(self) -> bool:
        return self._done.is_set()

    def wait(self):
        self._done.wait()


def _serve_builds(jobs: queue.SimpleQueue) -> None:
    """Body of an index's build thread: runs queued builds until None."""
    while True:
        job = jobs.get()
        if job is None:
            return
        job()
        del job  # the job holds the index; do not keep it while idle


def _stream_handles(streams):
    """Raw handles (s0, s1, ev0..ev3) for the global-step operators, or None
    when they cannot be used: everything on the current stream (no side
    streams; 0 handles) is fine, side streams need events that exist
    already (a torch event gets its CUDA event at its first record)."""
    if streams is None:
        return (0, 0, 0, 0, 0, 0)
    s0, s1, ev = streams
    hs = [e.cuda_event for e in ev]
    if not all(hs):
        return None
    return (s0.cuda_stream, s1.cuda_stream, *hs)


class GlobalIndex:
    """GPU-resident global suffix index with periodic rebuilds."""

    def __init__(self, capacity: int, delta_capacity: int, k: int,
                 max_occurrences: int = 32,
                 rebuild_threshold: int | None = None,
                 device: torch.device | str = "cuda",
                 rebuild_stream: torch.cuda.Stream | None = None):
        self.capacity = capacity
        self.delta_capacity = delta_capacity
        self.k = k
        self.max_occurrences = max_occurrences
        self.rebuild_threshold = rebuild_threshold or max(
            1, delta_capacity // 2)
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("GlobalIndex (suffixgpu_b200) needs a CUDA "
                             "device")
        self.rebuild_stream = rebuild_stream
        dev = self.device
        self.corpus = torch.full((capacity,), PAD_TOKEN, dtype=torch.int32,
                                 device=dev)
        self.staging_corpus = self.corpus.clone()
        self.sa = torch.arange(capacity, dtype=torch.int32, device=dev)
        self.staging_sa = self.sa.clone()
        self._arange = self.sa.clone()
        self.delta = torch.zeros(delta_capacity, dtype=torch.int32,
                                 device=dev)
        self.delta_len_t = torch.zeros((), dtype=torch.int64, device=dev)
        self.active_len = 0
        self.delta_len = 0
        # document lengths (each counting its SEP), oldest first
        self.active_doc_lens = DocLedger()
        self.delta_doc_lens = DocLedger()
        # a background rebuild in flight: its completion flag, and what the
        # swap applies (corpus length, evicted documents, absorbed lengths)
        self._rebuild_event = None
        self._pending = None
        # one long-lived build thread per index (started on first use): a
        # queue hand-off per rebuild instead of a thread start
        self._worker: threading.Thread | None = None
        self._jobs: queue.SimpleQueue | None = None
        self.rebuilds = 0
        self.last_rounds = 0
        self._step_bufs: dict = {}
        self._sa_ws: torch.Tensor | None = None
        # Incremental rebuilds (sg_suffix_array_append): the staging SA is
        # merged from the active one when at most half of the snapshot has
        # to be sorted afresh. _sa_rounds bounds the active SA's longest
        # common prefix (< 2^_sa_rounds; None when unknown, e.g. after
        # load_state_dict of an old state); the empty index's SA is exact.
        self.incremental_rebuild = True
        self._sa_rounds: int | None = 0
        self._staging_rounds: int | None = None
        self.last_build = None  # "full" or "append"
        # (kind, host seconds, snapshot tokens) of the latest builds
        self.build_log: deque = deque(maxlen=1024)
        # Multi-GPU: maps "my rebuild has finished" to "every rank's has",
        # so that replicas of the index swap at the same call.
        self.rebuild_agree = None
        # callables run after a new suffix array became the active one
        # (suffix-array shards re-extract theirs)
        self.on_swap: list = []

    # ------------------------------------------------------------------
    # writes (global_index.py:86-133)
    # ------------------------------------------------------------------
    def append_documents(self, docs: list[torch.Tensor]) -> None:
        """Append finished-response token tensors to the delta, each
        followed by one SEP_TOKEN (recorded lengths include it). A document
        longer than the delta keeps its newest delta_capacity - 1 tokens."""
        held = []
        for doc in docs:
            d = doc.reshape(-1)
            if (d.device != self.device or d.dtype != torch.int32
                    or not d.is_contiguous()):
                d = d.to(device=self.device, dtype=torch.int32).contiguous()
            if d.numel():
                held.append(d)  # alive until its copy is enqueued
        self._ingest([(d.data_ptr(), d.numel()) for d in held])

    def append_rows(self, token_ids: torch.Tensor, rows: list[int],
                    lengths: list[int]) -> None:
        """append_documents of ``token_ids[r, :length]`` for each row r,
        without slicing on the host (harvest_finished's documents)."""
        if token_ids.dtype != torch.int32 or token_ids.device != self.device \
                or token_ids.stride(1) != 1:
            self.append_documents([token_ids[r, :ln]
                                   for r, ln in zip(rows, lengths)])
            return
        base = token_ids.data_ptr()
        pitch = 4 * token_ids.stride(0)
        width = token_ids.shape[1]
        self._ingest([(base + pitch * r, min(ln, width))
                      for r, ln in zip(rows, lengths) if ln > 0])

    def _ingest(self, docs: list[tuple[int, int]]) -> None:
        """Documents given as (device address, tokens) go after the delta's
        documents. Writes are batched; a document that does not fit first
        makes room (a rebuild, or dropping the oldest documents while one is
        in flight), and the batch before it is written before that."""
        cap = self.delta_capacity
        batch: list[tuple[int, int]] = []
        start = self.delta_len
        for addr, n in docs:
            if n + 1 > cap:  # keep the newest cap - 1 tokens
                addr += 4 * (n - (cap - 1))
                n = cap - 1
            if self.delta_len + n + 1 > cap:
                self._write_docs(self.delta, cap, start, batch)
                batch = []
                self._make_room(n + 1)
                start = self.delta_len
            batch.append((addr, n))
            self.delta_len += n + 1
            self.delta_doc_lens.append(n + 1)
        self._write_docs(self.delta, cap, start, batch)
        self.maybe_rebuild()

    def _write_docs(self, buf: torch.Tensor, capacity: int, start: int,
                    docs: list[tuple[int, int]], set_len: bool = True
                    ) -> None:
        """One sg_append_documents call: docs (and SEPs) from ``start``
        on; with set_len the delta's device length follows."""
        if not docs:
            return
        n = len(docs)
        addrs = (ctypes.c_void_p * n)(*(a for a, _ in docs))
        lens = (ctypes.c_int64 * n)(*(ln for _, ln in docs))
        call("sg_append_documents", buf.data_ptr(), capacity, start, addrs,
             lens, n, ptr(self.delta_len_t) if set_len else None,
             stream_of(self.device))

    def _make_room(self, needed: int) -> None:
        """Room for ``needed`` more delta tokens: a rebuild absorbs the
        delta; while one is in flight (its staging buffers busy) the
        oldest delta documents are dropped instead."""
        self.poll_rebuild()
        if self._rebuild_event is None:
            self._launch_rebuild()
        short = self.delta_len + needed - self.delta_capacity
        if short > 0:
            n = self.delta_doc_lens.count_covering(short)
            self._shift_delta(n)

    def _shift_delta(self, docs: int) -> None:
        """The ``docs`` oldest delta documents leave the delta: the rest
        moves to its front (one launch, device length included)."""
        gone = self.delta_doc_lens.oldest_tokens(docs)
        self.delta_doc_lens.drop_oldest(docs)
        left = self.delta_len - gone
        call("sg_delta_compact", ptr(self.delta), self.delta_capacity, gone,
             left, ptr(self.delta_len_t), stream_of(self.device))
        self.delta_len = left

    # ------------------------------------------------------------------
    # rebuild (global_index.py:138-253)
    # ------------------------------------------------------------------
    def maybe_rebuild(self) -> None:
        """A rebuild starts once the delta holds rebuild_threshold tokens
        and none is in flight."""
        self.poll_rebuild()
        if self._rebuild_event is None and self.delta_len \
                and self.delta_len >= self.rebuild_threshold:
            self._launch_rebuild()

    def _launch_rebuild(self) -> None:
        """Snapshot (plan_snapshot: kept corpus + absorbed delta documents)
        into the staging buffers, absorbed documents out of the delta at
        once, then the staging SA build, synchronous or in the background;
        the swap applies the plan to the active state."""
        if self._rebuild_event is not None:
            return
        plan = plan_snapshot(self.active_doc_lens, self.delta_doc_lens,
                             self.capacity)
        kept = self.active_len - plan.evict_tokens
        n_new = kept + plan.absorb_tokens
        if n_new == 0:
            return
        self._stage(plan.evict_tokens, kept, plan.absorb_tokens)
        absorbed = self.delta_doc_lens.oldest_lengths(plan.absorb_docs)
        if plan.absorb_docs:
            self._shift_delta(plan.absorb_docs)
        # the SA covers the real tokens plus one sentinel column
        m = min(n_new + 1, self.capacity)
        build = self._build_plan(m, plan.evict_tokens, kept)
        swap = (n_new, plan.evict_docs, absorbed)
        if self.rebuild_stream is None:
            self._build_staging_sa(self.staging_corpus, m, None, build)
            self._finish_swap(*swap)
            return
        self.rebuild_stream.wait_stream(
            torch.cuda.current_stream(self.device))
        ev = _ThreadEvent()
        self._pending = swap
        self._rebuild_event = ev

        def work():
            try:
                with torch.cuda.device(self.device):
                    self._build_staging_sa(
                        self.staging_corpus, m,
                        self.rebuild_stream.cuda_stream, build)
            except BaseException as e:  # surfaced at poll time
                ev.error = e
            ev.set()

        if self._worker is None:
            self._jobs = queue.SimpleQueue()
            self._worker = threading.Thread(
                target=_serve_builds, args=(self._jobs,), daemon=True)
            self._worker.start()
            weakref.finalize(self, self._jobs.put, None)
        self._jobs.put(work)

    def _stage(self, evicted: int, kept: int, absorbed: int) -> None:
        """staging corpus = active corpus[evicted : evicted + kept], then
        delta[:absorbed], then PAD up to the capacity."""
        dst = self.staging_corpus
        n_new = kept + absorbed
        if kept:
            dst[:kept].copy_(self.corpus[evicted:evicted + kept])
        if absorbed:
            dst[kept:n_new].copy_(self.delta[:absorbed])
        if n_new < self.capacity:
            dst[n_new:].fill_(PAD_TOKEN)

    def _build_plan(self, m: int, evicted: int, kept: int):
        """How to build a staging snapshot of m tokens whose first `kept`
        are the active corpus from `evicted` on: None for a full build, or
        the arguments of an incremental one (decided and captured on the
        calling thread)."""
        if self._sa_ws is None:
            from suffixgpu_b200 import _lib
            need = int(_lib.lib().sg_suffix_array_append_workspace_size(
                self.capacity))
            self._sa_ws = torch.empty(need, dtype=torch.uint8,
                                      device=self.device)
        r = self._sa_rounds
        if not self.incremental_rebuild or r is None or kept <= 0:
            return None
        if r > _APPEND_MAX_ROUNDS:
            return None  # long repeats: merge comparisons would run deep
        if 2 * (kept - (1 << r)) < m:
            return None  # over half of the snapshot would be re-sorted
        prev_n = min(self.active_len + 1, self.capacity)
        return (prev_n, evicted, kept, r)

    def _build_staging_sa(self, dst: torch.Tensor, m: int,
                          stream: int | None, plan=None) -> None:
        t0 = time.perf_counter()
        if plan is None:
            self.last_rounds = ops.build_suffix_array_into(
                dst[:m], self.staging_sa[:m], workspace=self._sa_ws,
                stream=stream)
            self.last_build = "full"
        else:
            prev_n, evicted, kept, r = plan
            self.last_rounds = ops.append_suffix_array_into(
                dst[:m], self.staging_sa[:m], self.sa, prev_n, evicted,
                kept, r, workspace=self._sa_ws, stream=stream)
            self.last_build = "append"
        self._staging_rounds = self.last_rounds
        self.build_log.append((self.last_build, time.perf_counter() - t0, m))
        if m < self.capacity:
            # all-sentinel suffixes compare greater than any real pattern
            if stream is None:
                self.staging_sa[m:].copy_(self._arange[m:])
            else:
                with torch.cuda.stream(torch.cuda.ExternalStream(stream)):
                    self.staging_sa[m:].copy_(self._arange[m:])
                torch.cuda.ExternalStream(stream).synchronize()

    def _finish_swap(self, n_new: int, evicted_docs: int,
                     new_lens) -> None:
        """The staging pair becomes the active one: in-place copies keep
        the active tensors' storage (graph safety); the oldest
        ``evicted_docs`` active documents leave the ledger and ``new_lens``
        join it."""
        self.corpus.copy_(self.staging_corpus)
        self.sa.copy_(self.staging_sa)
        self.active_len = n_new
        self.active_doc_lens.drop_oldest(evicted_docs)
        self.active_doc_lens.extend(new_lens)
        self._sa_rounds = self._staging_rounds
        self._rebuild_event = None
        self._pending = None
        self.rebuilds += 1
        for fn in self.on_swap:
            fn()

    def poll_rebuild(self) -> None:
        """Swap in a finished background rebuild (non-blocking)."""
        if self._rebuild_event is None:
            return
        done = self._rebuild_event.query()
        if self.rebuild_agree is not None:
            done = self.rebuild_agree(done)
        if done:
            err = getattr(self._rebuild_event, "error", None)
            if err is not None:
                self._rebuild_event = None
                self._pending = None
                raise RuntimeError("background suffix-array build failed") \
                    from err
            self._finish_swap(*self._pending)

    # ------------------------------------------------------------------
    # bulk load and persistence (no reference counterpart; the reference
    # lists "global tree save & load" as a TODO, README.md:212-217)
    # ------------------------------------------------------------------
    def load_documents(self, docs: list[torch.Tensor]) -> None:
        """Load many finished documents at once: the state equals appending
        them (each trimmed to its last capacity - 1 tokens, so that it fits
        with its SEP) to an otherwise empty, unbounded delta and running the
        rebuild (eviction and snapshot rules of global_index.py:147-223)
        until the delta is empty. One suffix-array build, synchronous."""
        self.wait_rebuild()
        if self.delta_len:
            raise ValueError("load_documents needs an empty delta")
        cap = self.capacity
        docs = [d.reshape(-1).to(device=self.device,
                                 dtype=torch.int32).contiguous()[-(cap - 1):]
                for d in docs if d.numel() > 0]
        if not docs:
            return
        new_lens = [int(d.numel()) + 1 for d in docs]
        bp = plan_bulk_load(self.active_doc_lens, new_lens, cap)
        if bp.rebuilds == 0:
            return
        keep = bp.keep_tokens
        chosen = docs[bp.first_new:bp.first_new + bp.new_docs]
        n_new = keep + sum(new_lens[bp.first_new:bp.first_new + bp.new_docs])
        dst = self.staging_corpus
        if keep:
            dst[:keep].copy_(
                self.corpus[self.active_len - keep:self.active_len])
        self._write_docs(dst, cap, keep,
                         [(d.data_ptr(), d.numel()) for d in chosen],
                         set_len=False)
        if n_new < cap:
            dst[n_new:].fill_(PAD_TOKEN)
        m = min(n_new + 1, cap)
        build = self._build_plan(m, self.active_len - keep, keep)
        self._build_staging_sa(dst, m, None, build)
        self._finish_swap(n_new, len(self.active_doc_lens) - bp.keep_docs,
                          new_lens[bp.first_new:bp.first_new + bp.new_docs])

    def state_dict(self) -> dict:
        """Corpus, suffix array, delta and document lengths as host tensors
        (raw int32 arrays plus length lists), for torch.save. Waits for an
        in-flight rebuild first."""
        self.wait_rebuild()
        n = self.active_len
        return {
            "capacity": self.capacity,
            "delta_capacity": self.delta_capacity,
            "corpus": self.corpus[:n].cpu(),
            "sa": self.sa[:min(n + 1, self.capacity)].cpu(),
            "delta": self.delta[:self.delta_len].cpu(),
            "active_doc_lens": list(self.active_doc_lens),
            "delta_doc_lens": list(self.delta_doc_lens),
            "sa_rounds": self._sa_rounds,
        }

    def load_state_dict(self, state: dict) -> None:
        """Restore a state_dict() of an index with the same capacities into
        the existing device buffers (tensor identity is kept, so captured
        CUDA graphs stay valid); no rebuild runs."""
        if (int(state["capacity"]) != self.capacity
                or int(state["delta_capacity"]) != self.delta_capacity):
            raise ValueError("state_dict capacities differ from this index")
        self.wait_rebuild()
        corpus = state["corpus"].to(torch.int32)
        sa = state["sa"].to(torch.int32)
        delta = state["delta"].to(torch.int32)
        n = corpus.numel()
        self.corpus.fill_(PAD_TOKEN)
        self.corpus[:n].copy_(corpus)
        self.sa.copy_(self._arange)
        self.sa[:sa.numel()].copy_(sa)
        self.delta[:delta.numel()].copy_(delta)
        self.delta_len = int(delta.numel())
        self.delta_len_t.fill_(self.delta_len)
        self.active_len = n
        self.active_doc_lens = DocLedger(int(x)
                                         for x in state["active_doc_lens"])
        self.delta_doc_lens = DocLedger(int(x) for x in state["delta_doc_lens"])
        r = state.get("sa_rounds")
        self._sa_rounds = None if r is None else int(r)
        for fn in self.on_swap:
            fn()

    def wait_rebuild(self) -> None:
        """Block until an in-flight background rebuild has finished and
        swap it in (deterministic schedules in tests)."""
        if self._rebuild_event is None:
            return
        wait = getattr(self._rebuild_event, "wait", None)
        if wait is not None:
            wait()
        self.poll_rebuild()

    # ------------------------------------------------------------------
    # queries (global_index.py:257-370, 443-553)
    # ------------------------------------------------------------------
    def query(self, query: torch.Tensor, query_len: torch.Tensor,
              max_len: int):
        """Longest-suffix match against corpus + delta: (match_len [B] i64,
        cont [B, R, k] int32 (-1 padded), occ_count [B] i64)."""
        caps = torch.full((1,), max_len, dtype=torch.int64,
                          device=self.device)
        ml, cont, occ = self._query_backoff(query, query_len, max_len, caps)
        return ml[:, 0], cont[:, 0], occ[:, 0]

    def _query_backoff(self, query, query_len, max_len: int, caps,
                       row_mask=None, spec=None):
        """Per-cap matches against corpus + delta: (match_len [B, C] i64,
        cont [B, C, R, k] int32, occ_count [B, C] i64) and, with
        spec=(has_factor, factor, offset), the spec caps [B, C] i64."""
        query = ops.as_i32(query)
        query_len = ops.as_i64(query_len)
        caps = ops.as_i64(caps)
        found = self._searches(query, query_len, max_len, caps, row_mask)
        return self._candidates(found, query.shape[0], caps.numel(), spec)

    def _searches(self, query, query_len, max_len: int, caps, row_mask):
        """SA walk and delta scan per cap (global_index.py:286-320):
        (sa_len, sa_start, sa_end, d_len, d_pos, d_cnt)."""
        sa_len, sa_start, sa_end = ops.suffix_match_backoff(
            self.sa, self.corpus, query, query_len, max_len, caps,
            row_mask=row_mask)
        d_len, d_pos, d_cnt = self._delta_match_backoff(
            query, query_len, max_len, caps, row_mask=row_mask)
        return sa_len, sa_start, sa_end, d_len, d_pos, d_cnt

    def _candidates(self, found, b: int, cnum: int, spec=None):
        """The tail of _query_backoff (global_index.py:321-370) and
        _gather_cont (:443-463) on the search results."""
        dev = self.device
        r = self.max_occurrences
        sa_len, sa_start, sa_end, d_len, d_pos, d_cnt = found
        match_len = torch.empty(b, cnum, dtype=torch.int64, device=dev)
        cont = torch.empty(b, cnum, r, self.k, dtype=torch.int32, device=dev)
        occ = torch.empty(b, cnum, dtype=torch.int64, device=dev)
        cap_out = None
        has_f, fac, off = 0, 0.0, 0.0
        if spec is not None:
            cap_out = torch.empty(b, cnum, dtype=torch.int64, device=dev)
            has_f, fac, off = spec
        call("sg_global_candidates", ptr(sa_len), ptr(sa_start), ptr(sa_end),
             ptr(d_len), ptr(d_pos), ptr(d_cnt), ptr(self.sa),
             ptr(self.corpus), self.capacity, ptr(self.delta),
             self.delta_capacity, ptr(self.delta_len_t), b, cnum, r, self.k,
             int(has_f), float(fac), float(off), ptr(match_len), ptr(cont),
             ptr(occ), ptr(cap_out), stream_of(dev))
        if spec is not None:
            return match_len, cont, occ, cap_out
        return match_len, cont, occ

    def _delta_match_backoff(self, query, query_len, max_len: int, caps,
                             row_mask=None):
        """(match_len [B, C], start positions [B, C, R], count [B, C]),
        int64 (global_index.py:465-546)."""
        dev = self.device
        query = ops.as_i32(query)
        query_len = ops.as_i64(query_len)
        caps = ops.as_i64(caps)
        b, q = query.shape
        cnum = caps.numel()
        r = self.max_occurrences
        lo = torch.empty(b, cnum, dtype=torch.int64, device=dev)
        pos = torch.empty(b, cnum, r, dtype=torch.int64, device=dev)
        cnt = torch.empty(b, cnum, dtype=torch.int64, device=dev)
        rm = None if row_mask is None else row_mask.to(torch.bool).contiguous()
        call("sg_delta_match_backoff", ptr(self.delta), self.delta_capacity,
             ptr(self.delta_len_t), ptr(query), b, q, ptr(query_len),
             max_len, ptr(caps), cnum, r, ptr(rm), ptr(lo), ptr(pos),
             ptr(cnt), stream_of(dev))
        return lo, pos, cnt

    def draft(self, query, query_len, max_len: int, k: int,
              min_token_prob: float = 0.0,
              max_spec_factor: float | None = None,
              max_spec_offset: float = 0.0, caps=None, alpha: float = 0.0):
        """Multi-length scored draft over corpus + delta
        (global_index.py:372-441): (chain [B, k] int32, num_valid [B] i64,
        match_len [B] i64, occ_count [B] i64, score [B] f32)."""
        dev = self.device
        b = query.shape[0]
        if caps is None:
            caps = torch.tensor(
                sorted({max_len, max(2, max_len // 2),
                        max(2, max_len // 4), 2}, reverse=True),
                dtype=torch.int64, device=dev)
        cnum = caps.numel()
        spec = (max_spec_factor is not None, max_spec_factor or 0.0,
                max_spec_offset)
        match_len, cont, occ, cap_emit = self._query_backoff(
            query, query_len, max_len, caps, spec=spec)
        if max_spec_factor is None:
            cap_emit = torch.full_like(cap_emit, k)
        chain, _, num_emit, score = ops.expand_chain(
            cont.reshape(b * cnum, self.max_occurrences, self.k),
            occ.reshape(b * cnum), k, min_token_prob=min_token_prob,
            cap=cap_emit.reshape(-1), alpha=alpha)
        score = score.reshape(b, cnum)
        best = score.argmax(dim=1)
        bidx = torch.arange(b, device=dev)
        best_chain = chain.reshape(b, cnum, k)[bidx, best]
        best_emit = num_emit.reshape(b, cnum)[bidx, best]
        best_len = match_len[bidx, best]
        best_occ = occ[bidx, best]
        best_score = score[bidx, best]
        slot = torch.arange(k, device=dev).unsqueeze(0)
        best_chain = torch.where(slot < best_emit.unsqueeze(1), best_chain,
                                 -1)
        return best_chain, best_emit, best_len, best_occ, best_score

    def expand(self, cont: torch.Tensor, occ_count: torch.Tensor,
               min_token_prob: float = 0.0):
        chain, num_valid, _, _ = ops.expand_chain(
            cont, occ_count, self.k, min_token_prob=min_token_prob)
        return chain, num_valid

    # ------------------------------------------------------------------
    # drafter step (proposer.py:246-320)
    # ------------------------------------------------------------------
    def start_global_step(self, drafter, counts: torch.Tensor,
                          token_ids: torch.Tensor, sampled=None,
                          valid_count=None, limit: int | None = None,
                          mask=None, streams=None) -> dict:
        """First half of the drafter's global step (proposer.py:243-304):
        the rows' tails as update_state leaves them (read before the scatter,
        sg_gather_tails_update), the SA backoff search and the delta scan.
        Its buffers belong to the current stream. With streams =
        (s0, s1, four events) the work forks off the current stream: tails
        then the SA search on s0, the delta scan on s1 after the tails, so
        both searches run while the local step (which performs the scatter)
        runs on the current stream; finish_global_step joins them."""
        dev = self.device
        b, s = token_ids.shape
        p = drafter.max_pattern_len
        caps = drafter._global_caps
        cnum = caps.numel()
        r = self.max_occurrences
        counts = ops.as_i32(counts)
        samp = None if sampled is None else ops.as_i32(sampled)
        vc = None if (sampled is None or valid_count is None) \
            else ops.as_i32(valid_count)
        m8 = None if (sampled is not None or mask is None) \
            else mask.to(torch.uint8).contiguous()
        # Eager steps keep their buffers per shape (the fork waits for
        # everything already queued on the current stream, the previous
        # step's use of them included); a step being captured into a CUDA
        # graph allocates its own from the graph's pool, so that replays
        # never share them with eager calls on other streams.
        capturing = torch.cuda.is_current_stream_capturing()
        key = (b, p, cnum, r)
        st = None if capturing else self._step_bufs.get(key)
        if st is None:
            i64 = dict(dtype=torch.int64, device=dev)
            st = {"tails": torch.empty(b, p, dtype=torch.int32, device=dev),
                  "tail_len": torch.empty(b, **i64),
                  "row_mask": torch.empty(b, dtype=torch.uint8, device=dev),
                  "found": [torch.empty(b, cnum, **i64) for _ in range(4)]}
            st["found"].insert(4, torch.empty(b, cnum, r, **i64))
            st["found"].append(torch.empty(b, cnum, **i64))
            if not capturing:
                self._step_bufs[key] = st
        sa_len, sa_start, sa_end, d_len, d_pos, d_cnt = st["found"]
        tails, tail_len, row_mask = st["tails"], st["tail_len"], st["row_mask"]
        lim = s if limit is None else int(limit)
        handles = _stream_handles(streams)
        if handles is not None:
            # one dispatcher hop: the same three calls and the fork in C++
            torch_ops().global_start(
                counts, token_ids, samp, vc, m8, lim, self.sa, self.corpus,
                self.capacity, self.delta, self.delta_capacity,
                self.delta_len_t, caps, tails, tail_len, row_mask,
                st["found"], r, handles[0], handles[1], handles[2],
                handles[3])
            return st
        if streams is None:
            s_tails = s_sa = s_delta = stream_of(dev)
        else:
            s0, s1, ev = streams
            ev[0].record(torch.cuda.current_stream(dev))
            s0.wait_event(ev[0])
            s_tails = s_sa = s0.cuda_stream
            s_delta = s1.cuda_stream
        call("sg_gather_tails_update", ptr(token_ids), token_ids.stride(0), s,
             ptr(counts), ptr(samp), 0 if samp is None else samp.shape[1],
             ptr(vc), s if limit is None else int(limit), ptr(m8), b, p,
             ptr(tails), ptr(tail_len), ptr(row_mask), s_tails)
        if streams is not None:
            ev[1].record(s0)  # the delta scan needs the tails
            s1.wait_event(ev[1])
        call("sg_suffix_match_backoff", ptr(self.sa), ptr(self.corpus),
             self.capacity, ptr(tails), b, p, ptr(tail_len), p, ptr(caps),
             cnum, ptr(row_mask), ptr(sa_len), ptr(sa_start), ptr(sa_end),
             s_sa)
        call("sg_delta_match_backoff", ptr(self.delta), self.delta_capacity,
             ptr(self.delta_len_t), ptr(tails), b, p, ptr(tail_len), p,
             ptr(caps), cnum, r, ptr(row_mask), ptr(d_len), ptr(d_pos),
             ptr(d_cnt), s_delta)
        return st

    def finish_global_step(self, pending: dict, local: dict, drafter,
                           streams=None) -> tuple[torch.Tensor, torch.Tensor]:
        """Second half: joins the searches, then global candidates expanded
        and scored and combined with the local winner in place (global wins
        only on a strictly greater score; proposer.py:305-320)."""
        dev = self.device
        handles = _stream_handles(streams)
        if handles is not None and self.k == drafter.k:
            # join + fused step in one dispatcher hop
            code = torch_ops().global_finish(
                pending["found"], pending["row_mask"], self.sa, self.corpus,
                self.capacity, self.delta, self.delta_capacity,
                self.delta_len_t, self.max_occurrences, drafter.k,
                drafter.max_spec_factor is not None,
                float(drafter.max_spec_factor or 0.0),
                float(drafter.max_spec_offset),
                float(drafter.min_token_prob),
                float(drafter.vote_smoothing_alpha), local["best_score"],
                local["draft"], local["num_valid"], handles[0], handles[1],
                handles[4], handles[5])
            if code == 0:
                return local["draft"], local["num_valid"]
            streams = None  # joined already; the separate steps follow
        if streams is not None:
            s0, s1, ev = streams
            cur = torch.cuda.current_stream(dev)
            ev[2].record(s0)
            ev[3].record(s1)
            cur.wait_event(ev[2])
            cur.wait_event(ev[3])
        found = pending["found"]
        row_mask = pending["row_mask"]
        b = row_mask.shape[0]
        caps = drafter._global_caps
        cnum = caps.numel()
        spec = (drafter.max_spec_factor is not None,
                drafter.max_spec_factor or 0.0, drafter.max_spec_offset)
        draft, nv = local["draft"], local["num_valid"]
        st = stream_of(dev)
        # fused candidates + expand + selection (continuations on chip);
        # the continuation width must be the draft length
        st_code = _UNSUPPORTED if self.k != drafter.k else lib().sg_global_draft(
            *(ptr(x) for x in found[:6]), ptr(self.sa), ptr(self.corpus),
            self.capacity, ptr(self.delta), self.delta_capacity,
            ptr(self.delta_len_t), b, cnum, self.max_occurrences, drafter.k,
            int(spec[0]), float(spec[1]), float(spec[2]),
            float(drafter.min_token_prob),
            float(drafter.vote_smoothing_alpha), ptr(local["best_score"]),
            ptr(row_mask), ptr(draft), ptr(nv), st)
        if st_code == 0:
            return draft, nv
        if st_code != _UNSUPPORTED:
            check("sg_global_draft", st_code)
        # the row's continuation block does not fit on chip: separate steps
        match_len, cont, occ, cap = self._candidates(found, b, cnum, spec)
        chain, _, emit, score = ops.expand_chain(
            cont.reshape(b * cnum, self.max_occurrences, self.k),
            occ.reshape(-1), drafter.k,
            min_token_prob=drafter.min_token_prob, cap=cap.reshape(-1),
            alpha=drafter.vote_smoothing_alpha)
        call("sg_global_combine", ptr(draft), ptr(nv),
             ptr(local["best_score"]), ptr(row_mask), ptr(chain), ptr(emit),
             ptr(score), b, cnum, drafter.k, st)
        return draft, nv

    def propose_combine(self, counts: torch.Tensor, token_ids: torch.Tensor,
                        local: dict, drafter) -> tuple[torch.Tensor,
                                                       torch.Tensor]:
        """Global candidates for the rows the local kernel just drafted (and
        updated), expanded, scored and combined with the local winner, on
        the current stream."""
        pend = self.start_global_step(drafter, counts, token_ids,
                                      mask=local["row_mask"])
        return self.finish_global_step(pend, local, drafter)
