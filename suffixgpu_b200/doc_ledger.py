"""Document bookkeeping of the global index, as running token totals.

The global index keeps two queues of whole documents, oldest first: the
documents of the active corpus (covered by the suffix array) and those of
the delta buffer (not yet indexed). A rebuild takes a snapshot made of the
active corpus minus its oldest documents plus the oldest delta documents
that fit; when the delta overflows while a rebuild is in flight, its
oldest documents are discarded. The rules are those of the reference
(suffix_gpu/global_index.py:110-205); the representation is this
module's: each queue is a ``DocLedger`` of cumulative document ends, so
that "how many oldest documents cover t tokens" and "how many fit in t
tokens" are binary searches, and dropping the oldest documents moves a
head index, instead of walks over per-document lists.
"""

from __future__ import annotations

from bisect import bisect_left, bisect_right
from dataclasses import dataclass


class DocLedger:
    """Lengths of a queue of documents (oldest first), stored as running
    totals. Iterating yields the lengths."""

    __slots__ = ("_ends", "_head")

    def __init__(self, lengths=()):
        # _ends[i] = tokens of documents [0, i) ever appended; the live
        # documents are those from _head on
        self._ends = [0]
        self._head = 0
        self.extend(lengths)

    def __len__(self) -> int:
        return len(self._ends) - 1 - self._head

    def __iter__(self):
        e = self._ends
        for i in range(self._head, len(e) - 1):
            yield e[i + 1] - e[i]

    def __repr__(self) -> str:
        return f"DocLedger({list(self)})"

    @property
    def tokens(self) -> int:
        """Tokens of all live documents."""
        return self._ends[-1] - self._ends[self._head]

    def append(self, length: int) -> None:
        self._ends.append(self._ends[-1] + length)

    def extend(self, lengths) -> None:
        ends = self._ends
        total = ends[-1]
        for ln in lengths:
            total += ln
            ends.append(total)

    def oldest_tokens(self, count: int) -> int:
        """Tokens of the ``count`` oldest documents."""
        return self._ends[self._head + count] - self._ends[self._head]

    def oldest_lengths(self, count: int) -> list[int]:
        e, h = self._ends, self._head
        return [e[i + 1] - e[i] for i in range(h, h + count)]

    def count_covering(self, tokens: int) -> int:
        """Fewest oldest documents that hold at least ``tokens`` tokens
        (every document when all of them hold fewer)."""
        if tokens <= 0:
            return 0
        e, h = self._ends, self._head
        i = bisect_left(e, e[h] + tokens, h)
        return min(i - h, len(self))

    def count_within(self, tokens: int) -> int:
        """Most oldest documents that hold at most ``tokens`` tokens."""
        if tokens <= 0:
            return 0
        e, h = self._ends, self._head
        return bisect_right(e, e[h] + tokens, h) - 1 - h

    def drop_oldest(self, count: int) -> None:
        if count < 0 or count > len(self):
            raise ValueError(f"cannot drop {count} of {len(self)} documents")
        self._head += count
        # keep the totals list proportional to the live documents
        if self._head > 1024 and 2 * self._head > len(self._ends):
            self._ends = self._ends[self._head:]
            self._head = 0


@dataclass(frozen=True)
class SnapshotPlan:
    """What a rebuild takes: the oldest ``evict_docs`` active documents
    (``evict_tokens`` tokens) leave, the oldest ``absorb_docs`` delta
    documents (``absorb_tokens``) join after the rest of the corpus."""

    evict_docs: int
    evict_tokens: int
    absorb_docs: int
    absorb_tokens: int


def plan_snapshot(active: DocLedger, delta: DocLedger,
                  capacity: int) -> SnapshotPlan:
    """The rebuild snapshot rule (global_index.py:147-199): evict the
    fewest oldest active documents that let the whole delta fit beside the
    rest of the corpus (all of them if even that does not), then take the
    most oldest delta documents that fit in the room left."""
    overflow = active.tokens + delta.tokens - capacity
    evict = active.count_covering(overflow)
    evict_tokens = active.oldest_tokens(evict)
    room = capacity - (active.tokens - evict_tokens)
    absorb = delta.count_within(min(delta.tokens, room))
    return SnapshotPlan(evict, evict_tokens, absorb,
                        delta.oldest_tokens(absorb))


@dataclass(frozen=True)
class BulkPlan:
    """Outcome of a bulk load: the corpus ends up as the newest
    ``keep_docs`` documents of the current corpus (``keep_tokens`` tokens)
    followed by new documents ``first_new .. first_new + new_docs - 1``,
    after ``rebuilds`` rebuilds of the literal process."""

    keep_docs: int
    keep_tokens: int
    first_new: int
    new_docs: int
    rebuilds: int


def plan_bulk_load(active_doc_lens, new_doc_lens, capacity: int) -> BulkPlan:
    """Bulk load as the literal process would go: the new documents
    (lengths counting their SEP) sit in an unbounded delta, and rebuilds
    (plan_snapshot) run until the delta is empty or nothing fits. Eviction
    takes old documents before new ones, and absorption takes new ones in
    order, so the final corpus is a suffix of the old documents followed
    by a contiguous run of new ones."""
    active = DocLedger(active_doc_lens)
    n_old = len(active)
    delta = DocLedger(new_doc_lens)
    old_gone = new_gone = new_in = rebuilds = 0
    while len(delta):
        plan = plan_snapshot(active, delta, capacity)
        kept = active.tokens - plan.evict_tokens
        if kept + plan.absorb_tokens == 0:
            break  # a document longer than the capacity: nothing fits
        from_old = min(plan.evict_docs, n_old - old_gone)
        old_gone += from_old
        new_gone += plan.evict_docs - from_old
        active.drop_oldest(plan.evict_docs)
        active.extend(delta.oldest_lengths(plan.absorb_docs))
        delta.drop_oldest(plan.absorb_docs)
        new_in += plan.absorb_docs
        rebuilds += 1
    keep_docs = n_old - old_gone
    count = new_in - new_gone
    return BulkPlan(keep_docs, active.oldest_tokens(keep_docs),
                    new_gone if count else len(new_doc_lens), count,
                    rebuilds)


__all__ = ["DocLedger", "SnapshotPlan", "plan_snapshot", "BulkPlan",
           "plan_bulk_load"]
