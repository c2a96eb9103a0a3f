"""Multi-GPU drafters for benchmark config 5 (the 8-GPU global drafter).

The reference has no multi-GPU code; its semantics are those of one
drafter with one global index. Both drafters here keep them bit for bit,
one process per GPU under torch.distributed, request rows data-parallel
(each rank drafts its own rows), and the same ingestion: documents
harvested on any rank are all-gathered (rank order, each rank's in its own
order) and appended on every rank, and a background rebuild swaps in only
when every rank's has finished (a MIN all-reduce at poll time). Ingestion
calls (harvest_rows / harvest_finished / ingest_active / poll) are
therefore collective: every rank calls them, possibly with nothing to add.

* ``ShardedSuffixDrafter`` (config 5 as specified): the corpus is split by
  position into one shard per rank, and each rank queries only its shard's
  part of the suffix array: the suffixes that start in its shard, in
  suffix-array order, with their global ranks (``SuffixArrayShard``). A
  propose step gathers every rank's query tails, searches all of them on
  the local shard, sums the per-(row, length) interval bounds over the
  ranks (whole-corpus intervals), resolves the reference's strided
  suffix-array samples on the shard that holds them, and returns each
  row's samples to its owner (a sum reduce-scatter); the owner drafts from
  its copy of the corpus. Collectives per step: all-gather (tails),
  all-reduce SUM (bounds), reduce-scatter (samples), and from 8 ranks on
  an all-reduce MAX before the bounds (each row's longest match, so that only
  the lengths the caps select are searched). They run on a side stream
  while the local step and the delta scan of the rank's own rows run on
  the caller's.
* ``ReplicatedSuffixDrafter``: every rank holds the whole suffix array and
  its propose path has no collective.

The corpus itself, the delta and the suffix-array build are the same on
every rank in both modes (the build is replicated; a distributed suffix
sort is not part of this package). Works with NCCL (CUDA tensors); the
ingestion helpers also run on gloo (host tensors). Without an initialised
process group both drafters run as the only rank of a one-GPU job.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from suffixgpu_b200 import ops
from suffixgpu_b200._lib import call, check, lib, ptr, stream_of
from suffixgpu_b200.proposer import SuffixGPUDrafter


def _comm_device(group) -> torch.device:
    backend = dist.get_backend(group)
    if backend == "nccl":
        return torch.device("cuda", torch.cuda.current_device())
    return torch.device("cpu")


def exchange_documents(docs: list[torch.Tensor], group=None
                       ) -> list[torch.Tensor]:
    """All ranks' documents in rank order (each rank's in its own order),
    as int32 tensors on the communication device: three all-gathers
    (counts, lengths, tokens padded to the largest rank's total)."""
    world = dist.get_world_size(group)
    dev = _comm_device(group)
    docs = [d.reshape(-1).to(device=dev, dtype=torch.int32) for d in docs]
    if world == 1:
        return docs
    n = torch.tensor([len(docs)], dtype=torch.int64, device=dev)
    counts = [torch.zeros_like(n) for _ in range(world)]
    dist.all_gather(counts, n, group=group)
    counts = [int(c.item()) for c in counts]
    max_n = max(counts)
    if max_n == 0:
        return []
    lens = torch.zeros(max_n, dtype=torch.int64, device=dev)
    if docs:
        lens[:len(docs)] = torch.tensor([d.numel() for d in docs],
                                        dtype=torch.int64)
    all_lens = [torch.zeros_like(lens) for _ in range(world)]
    dist.all_gather(all_lens, lens, group=group)
    all_lens = [ln.tolist() for ln in all_lens]
    totals = [sum(ln[:c]) for ln, c in zip(all_lens, counts)]
    max_total = max(max(totals), 1)
    flat = torch.zeros(max_total, dtype=torch.int32, device=dev)
    if docs and totals[dist.get_rank(group)] > 0:
        flat[:totals[dist.get_rank(group)]] = torch.cat(docs)
    all_flat = [torch.zeros_like(flat) for _ in range(world)]
    dist.all_gather(all_flat, flat, group=group)
    out = []
    for r in range(world):
        pos = 0
        for ln in all_lens[r][:counts[r]]:
            out.append(all_flat[r][pos:pos + ln])
            pos += ln
    return out


def agree_all(flag: bool, group=None) -> bool:
    """True on every rank iff it is true on every rank (MIN all-reduce)."""
    if dist.get_world_size(group) == 1:
        return flag
    t = torch.tensor([1 if flag else 0], dtype=torch.int32,
                     device=_comm_device(group))
    dist.all_reduce(t, op=dist.ReduceOp.MIN, group=group)
    return bool(t.item())


class ReplicatedSuffixDrafter(SuffixGPUDrafter):
    """SuffixGPUDrafter for one rank of a multi-GPU job with the whole index
    on every rank: same constructor arguments plus ``group`` (default: the
    world). ``propose``, ``update_state`` and ``propose_with_update`` act on
    this rank's rows only and issue no collective; the ingestion calls are
    collective."""

    def __init__(self, *args, group=None, **kwargs):
        super().__init__(*args, **kwargs)
        self.group = group
        # without an initialised process group: one rank, no exchange
        self._distributed = dist.is_initialized()
        self.rank = dist.get_rank(group) if self._distributed else 0
        self.world_size = dist.get_world_size(group) \
            if self._distributed else 1
        if self.global_index is not None and self.world_size > 1:
            self.global_index.rebuild_agree = (
                lambda done: agree_all(done, self.group))

    def _append_docs(self, docs: list[torch.Tensor]) -> None:
        all_docs = exchange_documents(docs, self.group) \
            if self._distributed else docs
        if all_docs:
            self.global_index.append_documents(all_docs)

    def _append_rows(self, token_ids: torch.Tensor, rows: list[int],
                     lengths: list[int]) -> None:
        self._append_docs([token_ids[r, :ln]
                           for r, ln in zip(rows, lengths) if ln > 0])

    def load_documents(self, docs: list[torch.Tensor]) -> None:
        """Bulk-load documents that every rank holds (the same list on
        every rank, e.g. generated from a shared seed): no exchange."""
        super().load_documents(docs)


class SuffixArrayShard:
    """Shard ``part`` of ``parts`` of a GlobalIndex's suffix array: the
    suffixes that start in corpus positions [part * capacity / parts,
    (part + 1) * capacity / parts), in suffix-array order (``pos``), with
    their indices in the whole suffix array (``rank``). Re-extracted on the
    current stream whenever the index swaps in a new suffix array."""

    def __init__(self, index, part: int, parts: int):
        if not 0 <= part < parts:
            raise ValueError(f"part {part} of {parts}")
        self.index = index
        cap = index.capacity
        self.lo = part * cap // parts
        self.hi = (part + 1) * cap // parts
        n = self.hi - self.lo
        dev = index.device
        self.pos = torch.empty(max(n, 1), dtype=torch.int32, device=dev)
        self.rank = torch.empty(max(n, 1), dtype=torch.int32, device=dev)
        self._ws = torch.empty(
            int(lib().sg_shard_extract_workspace_size(cap)),
            dtype=torch.uint8, device=dev)
        self.refresh()
        index.on_swap.append(self.refresh)

    @property
    def size(self) -> int:
        return self.hi - self.lo

    def refresh(self) -> None:
        ix = self.index
        call("sg_shard_extract", ptr(ix.sa), ix.capacity, self.lo, self.hi,
             ptr(self.pos), ptr(self.rank), ptr(self._ws), self._ws.numel(),
             stream_of(ix.device))

    def longest(self, rows: torch.Tensor, max_len: int,
                out: torch.Tensor | None = None) -> torch.Tensor:
        """Per packed row, the longest tail suffix that starts one of this
        shard's suffixes (sg_shard_longest): int32 [B]."""
        b = rows.shape[0]
        if out is None:
            out = torch.empty(b, dtype=torch.int32, device=rows.device)
        ix = self.index
        call("sg_shard_longest", ptr(self.pos), self.size, ptr(ix.corpus),
             ix.capacity, ptr(rows), b, max_len, ptr(out),
             stream_of(ix.device))
        return out

    def bounds(self, rows: torch.Tensor, max_len: int,
               out: torch.Tensor | None = None,
               longest: torch.Tensor | None = None,
               caps: torch.Tensor | None = None) -> torch.Tensor:
        """Per packed row and length, this shard's (lower, upper) bounds:
        int32 [B, max_len, 2]; with ``longest`` (the job-wide longest match
        per row) and ``caps``, only the lengths the caps select."""
        b = rows.shape[0]
        if out is None:
            out = torch.empty(b, max_len, 2, dtype=torch.int32,
                              device=rows.device)
        ix = self.index
        call("sg_shard_bounds", ptr(self.pos), self.size, ptr(ix.corpus),
             ix.capacity, ptr(rows), b, max_len, ptr(longest), ptr(caps),
             0 if caps is None else caps.numel(), ptr(out),
             stream_of(ix.device))
        return out

    def resolve(self, bounds_sum: torch.Tensor, bounds_local: torch.Tensor,
                rows: torch.Tensor, caps: torch.Tensor, max_occ: int,
                own_lo: int, own_n: int, samples: torch.Tensor,
                plan: list[torch.Tensor]) -> None:
        """sg_shard_resolve: this shard's samples of every row into
        ``samples`` [B, C, R] and the per-cap plan of rows own_lo ..
        own_lo + own_n - 1 into ``plan`` (sa_len, start, end)."""
        b, max_len = bounds_sum.shape[:2]
        call("sg_shard_resolve", ptr(bounds_sum), ptr(bounds_local),
             ptr(rows), b, max_len, ptr(caps), caps.numel(), max_occ,
             ptr(self.pos), ptr(self.rank), ptr(samples), own_lo, own_n,
             ptr(plan[0]), ptr(plan[1]), ptr(plan[2]),
             stream_of(self.index.device))


class _Collectives:
    """The three collectives of a sharded step over a process group."""

    def __init__(self, group):
        self.group = group

    def all_gather(self, out: torch.Tensor, inp: torch.Tensor) -> None:
        dist.all_gather_into_tensor(out, inp, group=self.group)

    def all_reduce_sum(self, t: torch.Tensor) -> None:
        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)

    def all_reduce_max(self, t: torch.Tensor) -> None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)

    def reduce_scatter_sum(self, out: torch.Tensor, inp: torch.Tensor) -> None:
        dist.reduce_scatter_tensor(out, inp, op=dist.ReduceOp.SUM,
                                   group=self.group)


class _LocalCollectives:
    """The collectives of a one-rank job: copies."""

    def all_gather(self, out: torch.Tensor, inp: torch.Tensor) -> None:
        out.copy_(inp)

    def all_reduce_sum(self, t: torch.Tensor) -> None:
        pass

    def all_reduce_max(self, t: torch.Tensor) -> None:
        pass

    def reduce_scatter_sum(self, out: torch.Tensor, inp: torch.Tensor) -> None:
        out.copy_(inp)


class ShardedSuffixDrafter(ReplicatedSuffixDrafter):
    """One rank of the multi-GPU global drafter with the suffix array split
    into per-rank shards (module docstring). Needs ``enable_global=True``;
    every rank must call propose / propose_with_update together, with the
    same number of rows (rank r's rows are rows r * B .. r * B + B - 1 of
    the job)."""

    def __init__(self, *args, group=None, **kwargs):
        super().__init__(*args, group=group, **kwargs)
        if self.global_index is None:
            raise ValueError("ShardedSuffixDrafter needs enable_global=True")
        self.shard = SuffixArrayShard(self.global_index, self.rank,
                                      self.world_size)
        self._comm = _Collectives(group) if self._distributed \
            else _LocalCollectives()
        self._bufs: dict = {}
        self._side = None
        # "all" (every length's bounds in one round), "longest" (the job-wide
        # longest match first), or "auto": longest first from
        # longest_first_from ranks on
        self.length_search = "auto"
        self.longest_first_from = 8
        # a list to collect (phase, event) pairs of eager steps, or None
        self.phase_events = None

    # the local step, the global step's own-row parts, the exchange
    def propose_with_update(self, num_tokens_no_spec, token_ids_gpu,
                            sampled_token_ids,
                            valid_sampled_tokens_count=None,
                            max_model_len=None, *, out=None):
        s = token_ids_gpu.shape[1]
        limit = s if max_model_len is None else min(max_model_len, s)
        sampled = self._on_device(sampled_token_ids)
        vc = self._on_device(valid_sampled_tokens_count)
        draft, nv, new = self._step(num_tokens_no_spec, token_ids_gpu,
                                    sampled, vc, limit, None)
        return (*self._into(out, draft, nv), new)

    def propose(self, num_tokens_no_spec, token_ids_gpu, combined_mask=None,
                *, out=None):
        draft, nv, _ = self._step(num_tokens_no_spec, token_ids_gpu, None,
                                  None, token_ids_gpu.shape[1], combined_mask)
        return self._into(out, draft, nv)

    def _buffers(self, b: int, p: int, cnum: int, r: int) -> dict:
        key = (b, p, cnum, r)
        st = self._bufs.get(key)
        if st is None or torch.cuda.is_current_stream_capturing():
            dev = self.device
            g = self.world_size
            i32 = dict(dtype=torch.int32, device=dev)
            i64 = dict(dtype=torch.int64, device=dev)
            st = {"tails": torch.empty(b, p, **i32),
                  "tail_len": torch.empty(b, **i64),
                  "row_mask": torch.empty(b, dtype=torch.uint8, device=dev),
                  "rows_own": torch.empty(b, p + 2, **i32),
                  "rows_all": torch.empty(g * b, p + 2, **i32),
                  "longest": torch.empty(g * b, **i32),
                  "bounds_local": torch.empty(g * b, p, 2, **i32),
                  "bounds_sum": torch.empty(g * b, p, 2, **i32),
                  "samples_all": torch.empty(g * b, cnum, r, **i32),
                  "samples": torch.empty(b, cnum, r, **i32),
                  "plan": [torch.empty(b, cnum, **i64) for _ in range(3)],
                  "delta": [torch.empty(b, cnum, **i64),
                            torch.empty(b, cnum, r, **i64),
                            torch.empty(b, cnum, **i64)]}
            if not torch.cuda.is_current_stream_capturing():
                self._bufs[key] = st
        return st

    def _longest_first(self) -> bool:
        """Whether the step searches each row's longest match first (two
        rounds: a MAX, then only the cap-selected lengths' bounds) instead
        of every length's bounds in one round. Every rank searches every
        row of the job, so the saved search work grows with the world size
        while the extra round costs a fixed latency."""
        mode = self.length_search
        if mode == "auto":
            return self.world_size >= self.longest_first_from
        return mode == "longest"

    def _streams(self):
        """The side stream of the shard chain and its fork / join events
        (created on first use, reused)."""
        if self._side is None:
            self._side = (torch.cuda.Stream(self.device),
                          torch.cuda.Event(), torch.cuda.Event())
        return self._side

    def _mark(self, name: str, lane: str = "chain") -> None:
        """Per-phase timing (eager): an event on the current stream; lane
        names the stream's sequence of phases ("chain": the shard chain on
        the side stream, "own": the rank's own rows)."""
        if self.phase_events is not None:
            # under graph capture the record becomes an event-record node
            ev = torch.cuda.Event(
                enable_timing=True,
                external=torch.cuda.is_current_stream_capturing())
            ev.record()
            self.phase_events.append((lane, name, ev))

    def _step(self, counts, token_ids, sampled, vc, limit, mask):
        gi = self.global_index
        dev = self.device
        b, s = token_ids.shape
        p = self.max_pattern_len
        caps = self._global_caps
        cnum = caps.numel()
        r = gi.max_occurrences
        st = self._buffers(b, p, cnum, r)
        counts = ops.as_i32(counts)
        samp = None if sampled is None else ops.as_i32(sampled)
        vci = None if (sampled is None or vc is None) else ops.as_i32(vc)
        m8 = None if (sampled is not None or mask is None) \
            else mask.to(torch.uint8).contiguous()
        cur = torch.cuda.current_stream(dev)
        stream = stream_of(dev)
        # this rank's tails as the update leaves them (read before the local
        # step's scatter) and its drafting mask, packed for the exchange
        call("sg_gather_tails_update", ptr(token_ids), token_ids.stride(0),
             s, ptr(counts), ptr(samp),
             0 if samp is None else samp.shape[1], ptr(vci), int(limit),
             ptr(m8), b, p, ptr(st["tails"]), ptr(st["tail_len"]),
             ptr(st["row_mask"]), stream)
        call("sg_shard_pack_rows", ptr(st["tails"]), ptr(st["tail_len"]),
             ptr(st["row_mask"]), b, p, ptr(st["rows_own"]), stream)
        side, fork, join = self._streams()
        self._mark("start", "own")
        fork.record(cur)
        side.wait_event(fork)
        with torch.cuda.stream(side):
            # every rank's rows on this shard; per row the job-wide longest
            # match, then the bounds of the lengths the caps select, summed
            self._mark("start")
            self._comm.all_gather(st["rows_all"], st["rows_own"])
            self._mark("gather_tails")
            if self._longest_first():
                self.shard.longest(st["rows_all"], p, out=st["longest"])
                self._mark("shard_longest")
                self._comm.all_reduce_max(st["longest"])
                self._mark("max_longest")
                self.shard.bounds(st["rows_all"], p, out=st["bounds_local"],
                                  longest=st["longest"], caps=caps)
            else:
                self.shard.bounds(st["rows_all"], p, out=st["bounds_local"])
            self._mark("shard_bounds")
            st["bounds_sum"].copy_(st["bounds_local"])
            self._comm.all_reduce_sum(st["bounds_sum"])
            self._mark("sum_bounds")
            self.shard.resolve(st["bounds_sum"], st["bounds_local"],
                               st["rows_all"], caps, r, self.rank * b, b,
                               st["samples_all"], st["plan"])
            self._mark("resolve")
            self._comm.reduce_scatter_sum(st["samples"].view(-1),
                                          st["samples_all"].view(-1))
            self._mark("return_samples")
            join.record(side)
        # own rows meanwhile: delta scan, local step (performs the update)
        d_len, d_pos, d_cnt = st["delta"]
        call("sg_delta_match_backoff", ptr(gi.delta), gi.delta_capacity,
             ptr(gi.delta_len_t), ptr(st["tails"]), b, p, ptr(st["tail_len"]),
             p, ptr(caps), cnum, r, ptr(st["row_mask"]), ptr(d_len),
             ptr(d_pos), ptr(d_cnt), stream)
        o = self.local_kernel.run(counts, token_ids, sampled=samp,
                                  valid_count=vci, limit=limit,
                                  mask=None if samp is not None else mask,
                                  extras=True)
        self._mark("delta_and_local", "own")
        cur.wait_event(join)
        self._mark("wait_for_chain", "own")
        sa_len, s_start, s_end = st["plan"]
        draft, nv = o["draft"], o["num_valid"]
        check("sg_global_draft_samples", lib().sg_global_draft_samples(
            ptr(sa_len), ptr(s_start), ptr(s_end), ptr(d_len), ptr(d_pos),
            ptr(d_cnt), ptr(st["samples"]), st["samples"].numel(),
            ptr(gi.corpus), gi.capacity, ptr(gi.delta), gi.delta_capacity,
            ptr(gi.delta_len_t), b, cnum, r, self.k,
            int(self.max_spec_factor is not None),
            float(self.max_spec_factor or 0.0), float(self.max_spec_offset),
            float(self.min_token_prob), float(self.vote_smoothing_alpha),
            ptr(o["best_score"]), ptr(st["row_mask"]), ptr(draft), ptr(nv),
            stream))
        self._mark("global_step", "own")
        return draft, nv, o.get("new_counts")


__all__ = ["ShardedSuffixDrafter", "ReplicatedSuffixDrafter",
           "SuffixArrayShard", "exchange_documents", "agree_all"]
