"""Host-side logic of the global index that needs no GPU: the stream
handles the global-step operators take, the document bookkeeping of a
suffix-array swap, and the document ledger's eviction / absorption /
overflow answers against the oracle's literal walks over document lists
(the reference's rules, suffix_gpu/global_index.py:110-205)."""

from __future__ import annotations

from collections import deque
from types import SimpleNamespace

import numpy as np
import pytest

import torch

from oracle import suffix_oracle as so
from suffixgpu_b200.doc_ledger import DocLedger, plan_snapshot
from suffixgpu_b200.global_index import GlobalIndex, _stream_handles


def test_stream_handles():
    # everything on the current stream
    assert _stream_handles(None) == (0, 0, 0, 0, 0, 0)
    s0 = SimpleNamespace(cuda_stream=11)
    s1 = SimpleNamespace(cuda_stream=12)
    evs = tuple(SimpleNamespace(cuda_event=100 + i) for i in range(4))
    assert _stream_handles((s0, s1, evs)) == (11, 12, 100, 101, 102, 103)
    # an event without its CUDA event yet: the Python path is used
    evs0 = evs[:3] + (SimpleNamespace(cuda_event=0),)
    assert _stream_handles((s0, s1, evs0)) is None


def _bare_index(doc_lens):
    gi = object.__new__(GlobalIndex)
    gi.corpus = torch.zeros(16, dtype=torch.int32)
    gi.sa = torch.zeros(16, dtype=torch.int32)
    gi.staging_corpus = torch.arange(16, dtype=torch.int32)
    gi.staging_sa = torch.arange(16, dtype=torch.int32).flip(0)
    gi.active_len = sum(doc_lens)
    gi.active_doc_lens = DocLedger(doc_lens)
    gi._staging_rounds = 3
    gi._sa_rounds = 0
    gi._rebuild_event = object()
    gi._pending = object()
    gi.rebuilds = 0
    gi.on_swap = []
    return gi


def test_swap_applies_evicted_and_absorbed_documents():
    gi = _bare_index([4, 5, 6, 7])
    gi._finish_swap(6 + 7 + 2 + 3, 2, [2, 3])
    assert list(gi.active_doc_lens) == [6, 7, 2, 3]
    assert gi.active_len == 18
    assert torch.equal(gi.corpus, gi.staging_corpus)
    assert torch.equal(gi.sa, gi.staging_sa)
    assert gi._sa_rounds == 3 and gi.rebuilds == 1
    assert gi._rebuild_event is None and gi._pending is None


def test_swap_can_replace_every_document():
    gi = _bare_index([4, 5])
    gi._finish_swap(9, 2, [9])
    assert list(gi.active_doc_lens) == [9]
    assert gi.active_len == 9


def test_ledger_queries():
    led = DocLedger([3, 4, 5])
    assert len(led) == 3 and led.tokens == 12 and list(led) == [3, 4, 5]
    assert [led.count_covering(t) for t in (-1, 0, 1, 3, 4, 7, 8, 12, 13)] \
        == [0, 0, 1, 1, 2, 2, 3, 3, 3]
    assert [led.count_within(t) for t in (-1, 0, 2, 3, 6, 7, 11, 12, 99)] \
        == [0, 0, 0, 1, 1, 2, 2, 3, 3]
    led.drop_oldest(1)
    led.append(6)
    assert list(led) == [4, 5, 6] and led.tokens == 15
    assert led.oldest_tokens(2) == 9 and led.oldest_lengths(2) == [4, 5]
    assert led.count_covering(5) == 2 and led.count_within(5) == 1
    with pytest.raises(ValueError):
        led.drop_oldest(4)
    big = DocLedger([1] * 5000)
    big.drop_oldest(4000)  # compacts its totals
    assert len(big) == 1000 and big.tokens == 1000
    assert big.count_covering(10) == 10


@pytest.mark.parametrize("seed", range(20))
def test_snapshot_plan_matches_literal_walks(seed):
    """plan_snapshot against the oracle's GlobalIndex: its rebuild, run on
    the same document lists, evicts and absorbs the same documents, and
    the overflow drop takes the same count (count_covering)."""
    rng = np.random.default_rng(seed)
    capacity = int(rng.integers(20, 300))
    for _ in range(30):
        a_lens = [int(x) for x in rng.integers(1, 40, size=int(
            rng.integers(0, 12)))]
        d_lens = [int(x) for x in rng.integers(1, 40, size=int(
            rng.integers(0, 8)))]
        if sum(a_lens) > capacity:
            continue
        plan = plan_snapshot(DocLedger(a_lens), DocLedger(d_lens), capacity)
        o = so.GlobalIndex(capacity=capacity, delta_capacity=1 << 20, k=1)
        o.active_len = sum(a_lens)
        o.active_doc_lens = deque(a_lens)
        o.corpus[:o.active_len] = 1
        o.delta_len = sum(d_lens)
        o.delta_doc_lens = list(d_lens)
        o._launch_rebuild()
        kept_lens = a_lens[plan.evict_docs:]
        absorbed = d_lens[:plan.absorb_docs]
        if kept_lens or absorbed:
            assert list(o.active_doc_lens) == kept_lens + absorbed
            assert o.delta_doc_lens == d_lens[plan.absorb_docs:]
        assert plan.evict_tokens == sum(a_lens[:plan.evict_docs])
        assert plan.absorb_tokens == sum(absorbed)
        # the overflow drop of _drop_oldest_docs
        drop = int(rng.integers(1, 60))
        o2 = so.GlobalIndex(capacity=capacity, delta_capacity=1 << 20, k=1)
        o2.delta_len = sum(d_lens)
        o2.delta_doc_lens = list(d_lens)
        o2._drop_oldest_docs(drop)
        n = DocLedger(d_lens).count_covering(drop)
        assert o2.delta_doc_lens == d_lens[n:]
