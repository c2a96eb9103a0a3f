"""GlobalIndex's host logic on the CPU, against the oracle's index.

The index's device calls are replaced by host stand-ins that do the same
work on CPU tensors through their raw addresses (sg_append_documents,
sg_delta_compact) or through the oracle (the suffix-array build), so the
whole write / rebuild / eviction / overflow / bulk-load bookkeeping of
suffixgpu_b200/global_index.py runs here without a GPU and is compared,
state by state, with the oracle's restatement of the reference
(suffix_gpu/global_index.py:86-253). The stand-ins are test code; the
product has no CPU path.
"""

from __future__ import annotations

import ctypes
import threading
from collections import deque

import numpy as np
import pytest
import torch

from oracle import suffix_oracle as so
from suffixgpu_b200 import global_index as gim
from suffixgpu_b200.doc_ledger import DocLedger


def _i32_at(addr: int, n: int) -> np.ndarray:
    return np.ctypeslib.as_array((ctypes.c_int32 * max(n, 1)).from_address(
        addr))[:n]


def _set_i64(addr, v: int) -> None:
    if addr:
        ctypes.c_int64.from_address(addr).value = v


def _fake_call(name, *args):
    if name == "sg_append_documents":
        buf, cap, start, addrs, lens, n, len_out, _ = args
        pos = start
        out = _i32_at(buf, cap)
        for i in range(n):
            ln = lens[i]
            out[pos:pos + ln] = _i32_at(addrs[i], ln)
            out[pos + ln] = gim.SEP_TOKEN
            pos += ln + 1
        assert pos <= cap
        _set_i64(len_out, pos)
    elif name == "sg_delta_compact":
        buf, cap, start, count, len_out, _ = args
        out = _i32_at(buf, cap)
        out[:count] = out[start:start + count].copy()
        _set_i64(len_out, count)
    else:
        raise AssertionError(f"unexpected device call {name}")


def _fake_build(tokens, out, workspace=None, stream=None):
    out[:tokens.numel()] = torch.from_numpy(
        so.build_suffix_array(tokens.numpy()).astype(np.int32))
    return 1


@pytest.fixture
def host_index(monkeypatch):
    monkeypatch.setattr(gim, "call", _fake_call)
    monkeypatch.setattr(gim, "stream_of", lambda dev: 0)
    monkeypatch.setattr(gim.ops, "build_suffix_array_into", _fake_build)

    def make(capacity, delta_capacity, k=4, max_occurrences=8,
             rebuild_threshold=None):
        gi = object.__new__(gim.GlobalIndex)
        gi.capacity = capacity
        gi.delta_capacity = delta_capacity
        gi.k = k
        gi.max_occurrences = max_occurrences
        gi.rebuild_threshold = rebuild_threshold or max(
            1, delta_capacity // 2)
        gi.device = torch.device("cpu")
        gi.rebuild_stream = None
        gi.corpus = torch.full((capacity,), gim.PAD_TOKEN, dtype=torch.int32)
        gi.staging_corpus = gi.corpus.clone()
        gi.sa = torch.arange(capacity, dtype=torch.int32)
        gi.staging_sa = gi.sa.clone()
        gi._arange = gi.sa.clone()
        gi.delta = torch.zeros(delta_capacity, dtype=torch.int32)
        gi.delta_len_t = torch.zeros((), dtype=torch.int64)
        gi.active_len = gi.delta_len = 0
        gi.active_doc_lens = DocLedger()
        gi.delta_doc_lens = DocLedger()
        gi._rebuild_event = gi._pending = None
        gi._worker = gi._jobs = None
        gi.rebuilds = gi.last_rounds = 0
        gi._step_bufs = {}
        gi._sa_ws = torch.empty(0, dtype=torch.uint8)
        gi.incremental_rebuild = False
        gi._sa_rounds = 0
        gi._staging_rounds = None
        gi.last_build = None
        gi.build_log = deque(maxlen=16)
        gi.rebuild_agree = None
        gi.on_swap = []
        return gi
    return make


def _same(g, o, rebuilds=True):
    assert (g.active_len, g.delta_len) == (o.active_len, o.delta_len)
    assert int(g.delta_len_t) == o.delta_len
    assert list(g.active_doc_lens) == list(o.active_doc_lens)
    assert list(g.delta_doc_lens) == list(o.delta_doc_lens)
    np.testing.assert_array_equal(g.corpus.numpy(), o.corpus)
    np.testing.assert_array_equal(g.sa.numpy(), o.sa)
    np.testing.assert_array_equal(g.delta[:g.delta_len].numpy(),
                                  o.delta[:o.delta_len])
    if rebuilds:
        assert g.rebuilds == o.rebuilds


@pytest.mark.parametrize("seed", range(6))
def test_harvest_rebuild_eviction_vs_oracle(host_index, seed):
    """Random harvests (documents longer than the delta included) through
    append_documents and append_rows: every state equals the oracle's."""
    rng = np.random.default_rng(seed)
    kw = dict(capacity=int(rng.integers(120, 500)),
              delta_capacity=int(rng.integers(30, 120)),
              rebuild_threshold=int(rng.integers(10, 90)))
    g = host_index(**kw)
    o = so.GlobalIndex(k=4, max_occurrences=8, **kw)
    buf = torch.from_numpy(rng.integers(0, 7, size=(6, 200)).astype(
        np.int32))
    for _ in range(40):
        if rng.random() < 0.5:
            docs = [rng.integers(0, 7, size=int(rng.integers(0, 150))).astype(
                np.int32) for _ in range(int(rng.integers(1, 5)))]
            g.append_documents([torch.from_numpy(d) for d in docs])
            o.append_documents(docs)
        else:
            rows = [int(r) for r in rng.integers(0, 6, size=3)]
            lens = [int(x) for x in rng.integers(-2, 230, size=3)]
            g.append_rows(buf, rows, lens)
            o_docs = [buf[r].numpy()[:ln] for r, ln in zip(rows, lens)
                      if ln > 0]
            if o_docs:
                o.append_documents(o_docs)
        _same(g, o)
    assert o.rebuilds > 3


def test_overflow_while_rebuild_in_flight_vs_oracle(host_index):
    """With a rebuild that never finishes, an overflowing append drops the
    oldest delta documents like the reference (global_index.py:110-133)."""
    g = host_index(capacity=64, delta_capacity=18, rebuild_threshold=100000)
    o = so.GlobalIndex(capacity=64, delta_capacity=18, k=4,
                       max_occurrences=8, rebuild_threshold=100000)
    for idx, conv in ((g, torch.from_numpy), (o, lambda a: a)):
        idx.append_documents([conv(np.full(6, 1, np.int32)),
                              conv(np.full(6, 2, np.int32))])
        idx._rebuild_event = so.NeverDoneEvent()
        idx._pending = None
    for n in (10, 3, 17, 5):
        g.append_documents([torch.full((n,), n, dtype=torch.int32)])
        o.append_documents([np.full(n, n, np.int32)])
        _same(g, o)


def test_bulk_load_then_harvest_vs_oracle(host_index):
    rng = np.random.default_rng(9)
    g = host_index(capacity=700, delta_capacity=120, rebuild_threshold=60)
    o = so.GlobalIndex(capacity=700, delta_capacity=120, k=4,
                       max_occurrences=8, rebuild_threshold=60)
    for n_docs in (9, 14, 3):
        docs = [rng.integers(0, 6, size=int(rng.integers(1, 90))).astype(
            np.int32) for _ in range(n_docs)]
        docs.append(rng.integers(0, 6, size=730).astype(np.int32))
        # (a bulk load is one build here, the oracle's literal process
        # several: rebuild counts differ, states do not)
        g.load_documents([torch.from_numpy(d) for d in docs])
        o.load_documents(docs)
        _same(g, o, rebuilds=False)
        more = [rng.integers(0, 6, size=int(rng.integers(5, 40))).astype(
            np.int32) for _ in range(5)]
        g.append_documents([torch.from_numpy(d) for d in more])
        o.append_documents(more)
        _same(g, o, rebuilds=False)
        g.wait_rebuild()


def test_background_swap_applies_at_poll(host_index, monkeypatch):
    """A background rebuild (worker thread) leaves the active state alone
    until poll_rebuild swaps it in; then it equals the synchronous one."""
    g = host_index(capacity=300, delta_capacity=100, rebuild_threshold=50)
    o = so.GlobalIndex(capacity=300, delta_capacity=100, k=4,
                       max_occurrences=8, rebuild_threshold=50)

    class _Side:
        cuda_stream = 0

        def wait_stream(self, other):
            pass

    gate = threading.Event()
    real = gim.GlobalIndex._build_staging_sa

    def gated(self, dst, m, stream, plan=None):
        gate.wait(10)
        real(self, dst, m, None, plan)

    monkeypatch.setattr(gim.GlobalIndex, "_build_staging_sa", gated)
    monkeypatch.setattr(gim.torch.cuda, "current_stream", lambda dev: None)
    monkeypatch.setattr(gim.torch.cuda, "device", lambda dev: _NullCtx())
    g.rebuild_stream = _Side()
    docs = [np.arange(i, i + 30, dtype=np.int32) % 9 for i in range(3)]
    g.append_documents([torch.from_numpy(d) for d in docs])
    assert g._rebuild_event is not None and g.active_len == 0
    assert g.delta_len == 0  # the snapshot left the delta at once
    g.poll_rebuild()
    assert g._rebuild_event is not None  # not finished: nothing swapped
    gate.set()
    g._rebuild_event.wait()
    g.poll_rebuild()
    o.append_documents(docs)
    _same(g, o)


class _NullCtx:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False
