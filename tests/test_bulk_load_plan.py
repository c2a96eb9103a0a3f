"""Bulk loading of documents into the global index (CPU): the host
bookkeeping the product uses (one suffix-array build) against the oracle's
literal process, documents appended to an unbounded delta and the
reference's rebuild repeated until the delta is empty."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import suffix_oracle as so
from suffixgpu_b200.doc_ledger import plan_bulk_load


def _final_docs(active_docs, new_docs, capacity):
    """The product's plan applied to host document lists."""
    a_lens = [d.size + 1 for d in active_docs]
    n_lens = [d.size + 1 for d in new_docs]
    bp = plan_bulk_load(a_lens, n_lens, capacity)
    kept = active_docs[len(active_docs) - bp.keep_docs:]
    assert sum(d.size + 1 for d in kept) == bp.keep_tokens
    return kept + new_docs[bp.first_new:bp.first_new + bp.new_docs]


def _corpus(docs):
    out = []
    for d in docs:
        out.extend(d.tolist())
        out.append(so.SEP_TOKEN)
    return np.array(out, dtype=np.int32)


@pytest.mark.parametrize("seed", range(8))
def test_plan_matches_repeated_rebuilds(seed):
    rng = np.random.default_rng(seed)
    capacity = int(rng.integers(40, 400))
    o = so.GlobalIndex(capacity=capacity, delta_capacity=64, k=4,
                       max_occurrences=8, rebuild_threshold=1 << 30)
    # an existing corpus from an earlier load
    first_batch = [rng.integers(0, 5, size=int(rng.integers(1, 60))).astype(
        np.int32) for _ in range(int(rng.integers(0, 6)))]
    o.load_documents(first_batch)
    active_docs = []
    pos = 0
    for ln in o.active_doc_lens:
        active_docs.append(o.corpus[pos:pos + ln - 1].copy())
        pos += ln
    new_docs = [rng.integers(0, 5, size=int(rng.integers(1, 90))).astype(
        np.int32) for _ in range(int(rng.integers(1, 12)))]
    if seed % 3 == 0:  # a document longer than the capacity
        new_docs.insert(1, rng.integers(0, 5, size=capacity + 7).astype(
            np.int32))
    trimmed = [d[-(capacity - 1):] for d in new_docs]
    expect = _final_docs(active_docs, trimmed, capacity)
    o.load_documents(new_docs)
    np.testing.assert_array_equal(o.corpus[:o.active_len], _corpus(expect))
    assert list(o.active_doc_lens) == [d.size + 1 for d in expect]
    assert o.delta_len == 0
    sa = so.build_suffix_array(o.corpus[:min(o.active_len + 1, capacity)])
    np.testing.assert_array_equal(o.sa[:sa.size], sa)
