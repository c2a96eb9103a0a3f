"""Host-side logic of the global index that needs no GPU: the stream
handles the global-step operators take, and the document bookkeeping of a
suffix-array swap."""

from __future__ import annotations

from collections import deque
from types import SimpleNamespace

import torch

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
    gi.active_doc_lens = deque(doc_lens)
    gi._staging_rounds = 3
    gi._sa_rounds = 0
    gi._rebuild_event = object()
    gi._pending = object()
    gi.rebuilds = 0
    return gi


def test_swap_applies_evicted_and_absorbed_documents():
    gi = _bare_index([4, 5, 6, 7])
    gi._finish_swap(6 + 7 + 2 + 3, (2, [2, 3]))
    assert list(gi.active_doc_lens) == [6, 7, 2, 3]
    assert gi.active_len == 18
    assert torch.equal(gi.corpus, gi.staging_corpus)
    assert torch.equal(gi.sa, gi.staging_sa)
    assert gi._sa_rounds == 3 and gi.rebuilds == 1
    assert gi._rebuild_event is None and gi._pending is None


def test_swap_takes_a_full_length_list():
    gi = _bare_index([4, 5])
    gi._finish_swap(9, deque([9]))
    assert list(gi.active_doc_lens) == [9]
    assert gi.active_len == 9
