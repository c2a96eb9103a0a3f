"""The reference project's pinned drafter cases, on the CUDA path.

Each test restates one of the reference's own tests (cited per test, paths
inside the reference project) with its expected values, and where the
case has a larger state also compares with the numpy oracle:

* ingest_active chunking, overlap and final flush
  (tests/test_proposer_glue.py:90-139, code proposer.py:354-390);
* the golden drafts [7, 8, 9, 1] / [7, 8, -1, -1] and [6, -1, -1, -1]
  (tests/test_verification.py:289-336);
* no match or continuation across a document boundary, on the delta path
  and on the suffix-array path (tests/test_global_index.py:258-275);
* query results consistent across rebuild swaps
  (tests/test_verification.py:199-226);
* a propose captured in a CUDA graph before a background rebuild and
  replayed after the swap (the in-place swap of global_index.py:235-244
  exists so that captured graphs stay valid).
"""

from __future__ import annotations

import random

import numpy as np
import pytest
import torch

from oracle import suffix_oracle as so

pytestmark = pytest.mark.gpu

DEV = "cuda"
K, P = 4, 8


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def _host(t):
    return t.detach().cpu().numpy().copy()


def _glue_drafter(enable_global=False, **kw):
    """The drafter of tests/test_proposer_glue.py:15-19."""
    from suffixgpu_b200 import SuffixGPUDrafter
    return SuffixGPUDrafter(
        k=K, device=DEV, max_pattern_len=P, max_occurrences=8,
        enable_global=enable_global, global_capacity=1024,
        delta_capacity=256, rebuild_threshold=100000,
        vote_smoothing_alpha=0.0, **kw)


# ---------------------------------------------------------------------------
# ingest_active
# ---------------------------------------------------------------------------
def test_ingest_active_chunks_and_final():
    d = _glue_drafter(enable_global=True)
    gi = d.global_index
    row = torch.arange(100, 200, dtype=torch.int32, device=DEV)
    d.ingest_active(["r0"], [row], [10], chunk=16)
    assert gi.delta_len == 0                     # below the chunk size
    d.ingest_active(["r0"], [row], [20], chunk=16)
    assert gi.delta_len == 21                    # 20 tokens + SEP
    d.ingest_active(["r0"], [row], [30], chunk=16)
    assert gi.delta_len == 21                    # growth below the chunk
    d.ingest_active(["r0"], [row], [30], final=True, chunk=16)
    # the final flush re-sends the overlap (P + K tokens) with the tail
    assert gi.delta_len == 21 + (30 - (20 - (P + K))) + 1
    assert "r0" not in d._ingested
    exp = list(range(100, 120)) + [-2] + list(range(108, 130)) + [-2]
    assert _host(gi.delta[:gi.delta_len]).tolist() == exp


def test_ingest_active_overlap_keeps_boundary_patterns():
    d = _glue_drafter(enable_global=True)
    row = torch.arange(500, 564, dtype=torch.int32, device=DEV)
    d.ingest_active(["r"], [row], [32], chunk=32)
    d.ingest_active(["r"], [row], [64], chunk=32)
    # a pattern spanning the first chunk boundary (tokens 28..35)
    q = row[28:36].unsqueeze(0)
    qlen = torch.tensor([8], dtype=torch.int64, device=DEV)
    mlen, cont, occ = d.global_index.query(q, qlen, P)
    assert mlen[0].item() == 8
    chain, nv = d.global_index.expand(cont, occ)
    n = nv[0].item()
    assert n > 0
    assert chain[0, :n].tolist() == row[36:36 + n].tolist()


def test_ingest_then_cross_request_draft():
    d = _glue_drafter(enable_global=True)
    phrase = [11, 12, 13, 14, 15, 16, 17, 18]
    resp = torch.tensor(phrase * 8, dtype=torch.int32, device=DEV)
    d.ingest_active(["a"], [resp], [len(resp)], chunk=16)
    buf = torch.zeros(1, 32, dtype=torch.int32, device=DEV)
    cur = [99, 98] + phrase[:6]
    buf[0, :len(cur)] = torch.tensor(cur, dtype=torch.int32)
    counts = torch.tensor([len(cur)], dtype=torch.int32, device=DEV)
    mask = torch.ones(1, dtype=torch.bool, device=DEV)
    draft, nv = d.propose(counts, buf, mask)
    n = nv[0].item()
    assert n > 0
    assert draft[0, :n].tolist() == (phrase[6:] + phrase)[:n]


def test_ingest_active_many_keys_vs_oracle():
    """Several requests ingested in chunks of different sizes, finals
    interleaved, with rebuilds: delta, corpus and suffix array equal the
    oracle's."""
    from suffixgpu_b200 import SuffixGPUDrafter
    rng = np.random.default_rng(90)
    cfg = dict(k=K, max_pattern_len=P, max_occurrences=8,
               enable_global=True, global_capacity=2048, delta_capacity=300,
               rebuild_threshold=200)
    g = SuffixGPUDrafter(device=DEV, **cfg)
    o = so.SuffixDrafter(**cfg)
    rows = rng.integers(0, 9, size=(5, 400)).astype(np.int32)
    grows = [_dev(r) for r in rows]
    lens = [0] * 5
    for step in range(30):
        live = [i for i in range(5) if lens[i] < 400]
        if not live:
            break
        for i in live:
            lens[i] = min(400, lens[i] + int(rng.integers(3, 40)))
        final = step % 7 == 6
        chunk = int(rng.integers(8, 64))
        keys = [f"r{i}" for i in live]
        ls = [lens[i] for i in live]
        g.ingest_active(keys, [grows[i] for i in live], ls, final=final,
                        chunk=chunk)
        o.ingest_active(keys, [rows[i] for i in live], ls, final=final,
                        chunk=chunk)
        if final:
            for i in live:
                lens[i] = 400  # that request finished
        gi, oi = g.global_index, o.global_index
        assert (gi.active_len, gi.delta_len) == (oi.active_len, oi.delta_len)
        assert g._ingested == o._ingested
    np.testing.assert_array_equal(_host(gi.delta[:gi.delta_len]),
                                  oi.delta[:oi.delta_len])
    np.testing.assert_array_equal(_host(gi.corpus), oi.corpus)
    np.testing.assert_array_equal(_host(gi.sa), oi.sa)
    assert gi.rebuilds == oi.rebuilds > 0


# ---------------------------------------------------------------------------
# golden drafts (tests/test_verification.py:289-336; K = 4, P = 8, R = 16)
# ---------------------------------------------------------------------------
def _verification_drafter(**kw):
    from suffixgpu_b200 import SuffixGPUDrafter
    return SuffixGPUDrafter(k=K, device=DEV, max_pattern_len=P,
                            max_occurrences=16, enable_global=False,
                            vote_smoothing_alpha=0.0, **kw)


def _one_row(seq):
    buf = torch.zeros(1, 16, dtype=torch.int32, device=DEV)
    buf[0, :len(seq)] = torch.tensor(seq, dtype=torch.int32)
    return torch.tensor([len(seq)], dtype=torch.int32, device=DEV), buf


def test_golden_adaptive_max_spec_factor():
    nts, buf = _one_row([1, 2, 7, 8, 9, 1, 2])
    draft, nv = _verification_drafter().propose(nts, buf)
    assert nv[0].item() == 4
    assert draft[0].tolist() == [7, 8, 9, 1]
    draft, nv = _verification_drafter(max_spec_factor=1.0).propose(nts, buf)
    assert nv[0].item() == 2  # 1.0 * match length 2 + 0
    assert draft[0].tolist() == [7, 8, -1, -1]


def test_golden_adaptive_min_token_prob():
    nts, buf = _one_row([5, 6, 0, 5, 6, 1, 5, 7, 2, 5])
    draft, nv = _verification_drafter(min_token_prob=0.5).propose(nts, buf)
    assert nv[0].item() == 1  # 2/3 passes at depth 0, 1/3 cut at depth 1
    assert draft[0].tolist() == [6, -1, -1, -1]
    draft, nv = _verification_drafter(min_token_prob=0.7).propose(nts, buf)
    assert nv[0].item() == 0  # 2/3 < 0.7
    assert draft[0].tolist() == [-1, -1, -1, -1]


# ---------------------------------------------------------------------------
# no cross-document match (tests/test_global_index.py:258-275; K=4, R=8)
# ---------------------------------------------------------------------------
def _index_query(idx, query):
    q = torch.tensor([query], dtype=torch.int32, device=DEV)
    qlen = torch.tensor([len(query)], dtype=torch.int64, device=DEV)
    match_len, cont, occ = idx.query(q, qlen, P)
    chain, nv = idx.expand(cont, occ)
    return chain[0].tolist()[:nv[0].item()], match_len[0].item(), \
        occ[0].item()


@pytest.mark.parametrize("threshold", [100000, 1])  # delta path, SA path
def test_no_cross_document_match(threshold):
    from suffixgpu_b200.global_index import GlobalIndex
    idx = GlobalIndex(capacity=256, delta_capacity=64, k=K,
                      max_occurrences=8, rebuild_threshold=threshold,
                      device=DEV)
    idx.append_documents([_dev(np.array([1, 2, 3, 7, 8, 9], np.int32)),
                          _dev(np.array([100, 101, 102, 55, 56], np.int32))])
    if threshold == 1:
        assert idx.active_len == 13 and idx.delta_len == 0
    else:
        assert idx.active_len == 0 and idx.delta_len == 13
    # the tail of doc 1 matches, but its continuation is the boundary
    assert _index_query(idx, [7, 8, 9]) == ([], 3, 1)
    # a pattern spanning the boundary does not match across it
    assert _index_query(idx, [8, 9, 100]) == ([101, 102, 55, 56], 1, 1)


# ---------------------------------------------------------------------------
# query consistency across rebuilds (tests/test_verification.py:199-226)
# ---------------------------------------------------------------------------
def _naive_longest_suffix_match(corpus, query, max_len):
    best = 0
    for ln in range(1, min(max_len, len(query)) + 1):
        pat = query[-ln:]
        if any(corpus[s:s + ln] == pat
               for s in range(len(corpus) - ln + 1)):
            best = ln
    return best


def _naive_occurrences(corpus, pat):
    return [s for s in range(len(corpus) - len(pat) + 1)
            if corpus[s:s + len(pat)] == pat]


def test_query_consistency_across_rebuilds():
    from suffixgpu_b200 import SuffixGPUDrafter
    cfg = dict(k=K, max_pattern_len=P, max_occurrences=16,
               enable_global=True, global_capacity=1 << 16,
               delta_capacity=1 << 12, rebuild_threshold=1 << 10,
               vote_smoothing_alpha=0.0)
    idx = SuffixGPUDrafter(device=DEV, **cfg).global_index
    oidx = so.SuffixDrafter(**cfg).global_index
    idx.rebuild_threshold = oidx.rebuild_threshold = 16  # frequent rebuilds
    g = random.Random(3)
    corpus: list[int] = []
    for d in range(8):
        doc = [g.randint(0, 4) for _ in range(24)]
        idx.append_documents([torch.tensor(doc, dtype=torch.int32,
                                           device=DEV)])
        oidx.append_documents([np.array(doc, dtype=np.int32)])
        corpus.extend(doc)
        query = doc[-6:]
        q = np.array([query + [0] * (P - 6)], dtype=np.int32)
        qlen = np.array([6], dtype=np.int64)
        mlen, cont, occ = idx.query(_dev(q), _dev(qlen), P)
        exp_len = _naive_longest_suffix_match(corpus, query, P)
        assert int(mlen[0].item()) == exp_len, f"doc {d}"
        if exp_len > 0:
            exp_occ = _naive_occurrences(corpus, query[-exp_len:])
            assert 1 <= int(occ[0].item()) <= min(len(exp_occ), 16)
        # and exactly the oracle's answer, continuations included
        for a, b in zip((mlen, cont, occ), oidx.query(q, qlen, P)):
            np.testing.assert_array_equal(_host(a), b)
    assert idx.rebuilds == oidx.rebuilds >= 4


# ---------------------------------------------------------------------------
# a captured propose replayed across a background rebuild swap
# ---------------------------------------------------------------------------
def test_captured_propose_replayed_across_swap():
    """propose is captured into a CUDA graph; documents are then harvested
    (a background rebuild on the rebuild stream), the rebuild is swapped in
    at poll, and the same graph is replayed: its drafts equal the oracle's
    on the new index, before and after the swap."""
    from suffixgpu_b200 import SuffixGPUDrafter
    from suffixgpu_b200 import workloads as wl
    rng = np.random.default_rng(77)
    z = wl.Zipf(1.1, 300)
    templates = z.draw(rng, (10, 48))
    docs = wl.template_docs(rng, 80, 160, templates, z)
    b, s = 16, 1024
    rows = wl.template_docs(rng, b, s, templates, z)
    counts = rng.integers(300, 1000, size=b).astype(np.int32)
    cfg = dict(k=8, max_pattern_len=16, max_occurrences=32,
               enable_global=True, global_capacity=1 << 14,
               delta_capacity=4096, rebuild_threshold=1500,
               max_spec_factor=2.0, min_token_prob=0.05)
    side = torch.cuda.Stream()
    g = SuffixGPUDrafter(device=DEV, rebuild_stream=side, **cfg)
    o = so.SuffixDrafter(**cfg)
    # harvest in batches of 8 documents (1288 tokens): a batch crosses the
    # threshold at most once and never overflows the delta, so the GPU's
    # background rebuilds land where the oracle's synchronous ones do
    for i in range(0, 40, 8):
        g.harvest_rows([_dev(d) for d in docs[i:i + 8]], [160] * 8)
        g.global_index.wait_rebuild()
        o.harvest_rows(list(docs[i:i + 8]), [160] * 8)
    assert g.global_index.rebuilds == o.global_index.rebuilds > 0
    tok, n = _dev(rows), _dev(counts)
    cap_stream = torch.cuda.Stream()
    cap_stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(cap_stream):
        g.propose(n, tok)  # creates the side streams and buffers
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=cap_stream):
        draft, nv = g.propose(n, tok)
    graph.replay()
    torch.cuda.synchronize()
    do, nvo = o.propose(counts, rows)
    np.testing.assert_array_equal(_host(draft), do)
    np.testing.assert_array_equal(_host(nv), nvo)
    before = g.global_index.rebuilds
    # more documents: a rebuild starts in the background; swap at poll
    for i in range(40, 56, 8):
        g.harvest_rows([_dev(d) for d in docs[i:i + 8]], [160] * 8)
        o.harvest_rows(list(docs[i:i + 8]), [160] * 8)
        if g.global_index._rebuild_event is not None:
            break
    assert g.global_index._rebuild_event is not None
    g.global_index._rebuild_event.wait()
    g.poll()
    assert g.global_index._rebuild_event is None
    assert g.global_index.rebuilds == o.global_index.rebuilds > before
    graph.replay()
    torch.cuda.synchronize()
    do, nvo = o.propose(counts, rows)
    np.testing.assert_array_equal(_host(draft), do)
    np.testing.assert_array_equal(_host(nv), nvo)
    np.testing.assert_array_equal(_host(g.global_index.sa),
                                  o.global_index.sa)
    del graph
