"""GPU parity of the suffix-array build, the SA search, the delta scan and
the global drafter path against the reference goldens and the oracle.
Bit-exact (integer outputs; scores compared as fp32 bit patterns)."""

from __future__ import annotations

import os

import numpy as np
import pytest
import torch

import scenarios
from oracle import suffix_oracle as so

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def _host(t):
    return t.detach().cpu().numpy().copy()


# ---------------------------------------------------------------------------
# suffix array
# ---------------------------------------------------------------------------
def test_suffix_array_goldens(golden_dir):
    from suffixgpu_b200 import ops
    z = np.load(os.path.join(golden_dir, "sa_cases.npz"))
    for i in range(int(z["n"])):
        sa = ops.build_suffix_array(_dev(z[f"t{i}"]))
        np.testing.assert_array_equal(_host(sa), z[f"sa{i}"], f"case {i}")


@pytest.mark.parametrize("n,vocab", [(2, 1), (3, 2), (31, 3), (64, 8),
                                     (200, 16), (1000, 2), (5000, 3),
                                     (70000, 50000), (300000, 4)])
def test_suffix_array_random_vs_oracle(n, vocab):
    from suffixgpu_b200 import ops
    rng = np.random.default_rng(n + vocab)
    tok = rng.integers(-3, vocab, size=n).astype(np.int32)
    got = _host(ops.build_suffix_array(_dev(tok)))
    np.testing.assert_array_equal(got, so.build_suffix_array(tok))


def test_suffix_array_edge_tokens():
    """PAD (int32 max), SEP (-2), int32 min, long runs, empty and single."""
    from suffixgpu_b200 import ops
    t = np.array([2 ** 31 - 1] * 7 + [-2, 5, -2, -(2 ** 31), 0, 0, 0] * 3,
                 dtype=np.int32)
    np.testing.assert_array_equal(_host(ops.build_suffix_array(_dev(t))),
                                  so.build_suffix_array(t))
    run = np.full(4097, 9, dtype=np.int32)
    np.testing.assert_array_equal(_host(ops.build_suffix_array(_dev(run))),
                                  so.build_suffix_array(run))
    assert ops.build_suffix_array(_dev(np.zeros(0, np.int32))).numel() == 0
    assert _host(ops.build_suffix_array(_dev(np.array([7], np.int32)))) \
        .tolist() == [0]


@pytest.mark.parametrize("case", ["distinct", "distinct_pad", "wide_range",
                                  "pad_only"])
def test_suffix_array_dense_id_paths(case):
    """Both ways to the dense token ids (a presence bitmap when the non-PAD
    tokens span at most 64 n values, the first-token sort otherwise) give
    the oracle's array, and rounds = 0 exactly when every token differs."""
    from suffixgpu_b200 import ops
    rng = np.random.default_rng(17)
    n = 3000
    if case == "distinct":
        tok = rng.permutation(n).astype(np.int32) - 7
    elif case == "distinct_pad":
        tok = rng.permutation(n).astype(np.int32)
        tok[-1] = 2 ** 31 - 1
    elif case == "wide_range":
        tok = rng.integers(0, 50, size=n).astype(np.int32)
        tok[::97] = rng.integers(-2 ** 31, 2 ** 31 - 2, size=tok[::97].size)
    else:
        tok = np.full(n, 2 ** 31 - 1, dtype=np.int32)
    t = _dev(tok)
    out = torch.empty(n, dtype=torch.int32, device=DEV)
    rounds = ops.build_suffix_array_into(t, out)
    np.testing.assert_array_equal(_host(out), so.build_suffix_array(tok))
    assert (rounds == 0) == (np.unique(tok).size == n)


def _sa_is_sorted(tok: np.ndarray, sa: np.ndarray) -> None:
    """Linear-time certificate that sa is the suffix array of tok: a
    permutation, and consecutive suffixes ordered by (token, rank of the
    next suffix) with the end of string smallest."""
    n = tok.shape[0]
    assert np.array_equal(np.sort(sa), np.arange(n))
    rank = np.empty(n + 1, dtype=np.int64)
    rank[sa] = np.arange(n)
    rank[n] = -1
    a, b = sa[:-1], sa[1:]
    ta, tb = tok[a].astype(np.int64), tok[b].astype(np.int64)
    ok = (ta < tb) | ((ta == tb) & (rank[a + 1] < rank[b + 1]))
    assert ok.all(), f"{(~ok).sum()} unsorted neighbours"


def test_suffix_array_config4_size_property():
    """benchmark config 4 at full size (2^24 tokens, 50% copies): checked by
    the linear-time sortedness certificate."""
    from suffixgpu_b200 import ops
    from suffixgpu_b200 import workloads as wl
    tok = wl.config4(n=1 << 24, n_queries=1)["tokens"]
    sa = _host(ops.build_suffix_array(_dev(tok)))
    _sa_is_sorted(tok, sa)


def test_suffix_array_config4_shape_vs_oracle():
    from suffixgpu_b200 import ops
    from suffixgpu_b200 import workloads as wl
    tok = wl.config4(seed=9, n=1 << 18, n_queries=1)["tokens"]
    np.testing.assert_array_equal(_host(ops.build_suffix_array(_dev(tok))),
                                  so.build_suffix_array(tok))


# ---------------------------------------------------------------------------
# SA search
# ---------------------------------------------------------------------------
def test_sa_search_goldens(golden_dir):
    from suffixgpu_b200 import ops
    z = np.load(os.path.join(golden_dir, "sa_search_cases.npz"))
    s, e = ops.search_interval(_dev(z["sa"]), _dev(z["corpus"]),
                               _dev(z["pat"]), _dev(z["plen"]))
    np.testing.assert_array_equal(_host(s), z["start"])
    np.testing.assert_array_equal(_host(e), z["end"])
    ml, bs, be = ops.suffix_match_backoff(
        _dev(z["sa"]), _dev(z["corpus"]), _dev(z["q"]), _dev(z["qlen"]), 12,
        _dev(z["caps"]))
    np.testing.assert_array_equal(_host(ml), z["b_len"])
    np.testing.assert_array_equal(_host(bs), z["b_start"])
    np.testing.assert_array_equal(_host(be), z["b_end"])


def test_sa_search_random_vs_oracle():
    """Random corpora incl. PAD tails, patterns longer than the width and
    negative / zero lengths (the comparator's clamped column rule)."""
    from suffixgpu_b200 import ops
    rng = np.random.default_rng(5)
    for trial in range(4):
        n = int(rng.integers(50, 3000))
        corpus = rng.integers(0, 4, size=n).astype(np.int32)
        corpus[-int(rng.integers(0, 10)):] = so.PAD_TOKEN
        sa = so.build_suffix_array(corpus).astype(np.int32)
        m = 8
        pat = rng.integers(0, 4, size=(64, m)).astype(np.int32)
        for i in range(0, 64, 3):
            st = int(rng.integers(0, n - m))
            pat[i] = corpus[st:st + m]
        plen = rng.integers(-1, m + 3, size=64).astype(np.int64)
        s, e = ops.search_interval(_dev(sa), _dev(corpus), _dev(pat),
                                   _dev(plen))
        es, ee = so.search_interval(sa, corpus, pat, plen)
        np.testing.assert_array_equal(_host(s), es)
        np.testing.assert_array_equal(_host(e), ee)
        q = rng.integers(0, 4, size=(32, 10)).astype(np.int32)
        qlen = rng.integers(-1, 14, size=32).astype(np.int64)
        caps = np.array([16, 9, 5, 2, 1], dtype=np.int64)
        got = ops.suffix_match_backoff(_dev(sa), _dev(corpus), _dev(q),
                                       _dev(qlen), 12, _dev(caps))
        exp = so.suffix_match_backoff(sa, corpus, q, qlen, 12, caps)
        for g, x in zip(got, exp):
            np.testing.assert_array_equal(_host(g), x)


@pytest.mark.parametrize("width", [8, 40, 70, 140])
def test_sa_search_widths_vs_oracle(width):
    """Pattern widths of one, two and four columns per lane and beyond the
    warp path (one thread per bound); corpora with SEP (-2) and -1 tokens
    and PAD tails; lengths around the width."""
    from suffixgpu_b200 import ops
    rng = np.random.default_rng(50 + width)
    n = 4000
    corpus = rng.integers(-2, 3, size=n).astype(np.int32)
    for _ in range(30):  # long repeats so that matches run deep
        a, b = (int(x) for x in rng.integers(0, n - 300, size=2))
        ln = int(rng.integers(50, 300))
        if b + ln <= n:
            corpus[b:b + ln] = corpus[a:a + ln]
    corpus[-5:] = so.PAD_TOKEN
    sa = so.build_suffix_array(corpus).astype(np.int32)
    nb = 96
    pat = rng.integers(-2, 3, size=(nb, width)).astype(np.int32)
    for i in range(0, nb, 2):
        st = int(rng.integers(0, n - width))
        pat[i] = corpus[st:st + width]
    plen = rng.integers(-1, width + 3, size=nb).astype(np.int64)
    plen[::5] = width
    s, e = ops.search_interval(_dev(sa), _dev(corpus), _dev(pat), _dev(plen))
    es, ee = so.search_interval(sa, corpus, pat, plen)
    np.testing.assert_array_equal(_host(s), es)
    np.testing.assert_array_equal(_host(e), ee)
    q = pat[:40].copy()
    qlen = rng.integers(-1, width + 2, size=40).astype(np.int64)
    caps = np.array(sorted({width, max(2, width // 2), 4, 2, 1},
                           reverse=True), dtype=np.int64)
    got = ops.suffix_match_backoff(_dev(sa), _dev(corpus), _dev(q),
                                   _dev(qlen), width, _dev(caps))
    exp = so.suffix_match_backoff(sa, corpus, q, qlen, width, caps)
    for g, x in zip(got, exp):
        np.testing.assert_array_equal(_host(g), x)


def test_sa_search_config3_size_vs_oracle():
    """search_interval and suffix_match_backoff over a 2^22-token template
    corpus (the config-3 capacity) against the oracle's search on the same
    SA (built on the GPU; the SA itself is covered by the build tests)."""
    from suffixgpu_b200 import ops
    from suffixgpu_b200 import workloads as wl
    rng = np.random.default_rng(60)
    z = wl.Zipf(1.1, 32000)
    templates = z.draw(rng, (64, 256))
    corpus = wl.template_docs(rng, 4096, 1024, templates, z).reshape(-1)
    sa_t = ops.build_suffix_array(_dev(corpus))
    sa = _host(sa_t).astype(np.int32)
    pat = np.zeros((200, 32), dtype=np.int32)
    plen = np.zeros(200, dtype=np.int64)
    for i in range(200):
        ln = int(rng.integers(1, 33))
        st = int(rng.integers(0, corpus.size - ln))
        pat[i, :ln] = corpus[st:st + ln]
        plen[i] = ln if i % 7 else ln + 1
    s, e = ops.search_interval(_dev(sa), _dev(corpus), _dev(pat), _dev(plen))
    es, ee = so.search_interval(sa, corpus, pat, plen)
    np.testing.assert_array_equal(_host(s), es)
    np.testing.assert_array_equal(_host(e), ee)
    q = wl.template_docs(rng, 16, 300, templates, z)
    qlen = rng.integers(0, 300, size=16).astype(np.int64)
    caps = np.array(so.global_caps(32, 8), dtype=np.int64)
    got = ops.suffix_match_backoff(_dev(sa), _dev(corpus), _dev(q),
                                   _dev(qlen), 32, _dev(caps))
    exp = so.suffix_match_backoff(sa, corpus, q, qlen, 32, caps)
    for g, x in zip(got, exp):
        np.testing.assert_array_equal(_host(g), x)


# ---------------------------------------------------------------------------
# global index
# ---------------------------------------------------------------------------
def _gpu_drafter(**cfg):
    from suffixgpu_b200 import SuffixGPUDrafter
    return SuffixGPUDrafter(device=DEV, **cfg)


@pytest.mark.parametrize("seed", [41, 42])
def test_global_scenarios_match_goldens(golden_dir, seed):
    z = np.load(os.path.join(golden_dir, f"global_{seed}.npz"))
    sc = scenarios.global_scenario(seed)
    got = scenarios.run_scenario(sc, _gpu_drafter, _dev, _host)
    for key in ("draft", "num_valid", "new_counts", "final_tokens",
                "active_len", "delta_len", "corpus", "sa"):
        np.testing.assert_array_equal(got[key], z["out_" + key], key)


@pytest.mark.parametrize("seed", [3, 4, 5])
def test_global_scenarios_vs_oracle(seed):
    sc = scenarios.global_scenario(seed, steps=12)
    got = scenarios.run_scenario(sc, _gpu_drafter, _dev, _host)
    exp = scenarios.run_scenario(sc, so.SuffixDrafter, lambda a: a.copy(),
                                 lambda a: np.asarray(a).copy())
    for key in ("draft", "num_valid", "new_counts", "final_tokens",
                "active_len", "delta_len", "corpus", "sa"):
        np.testing.assert_array_equal(got[key], exp[key], key)


class _NoFusedDraft:
    """The kernel library with sg_global_draft answering "unsupported", as
    it does when a row's continuation block exceeds shared memory."""

    def __init__(self, real):
        self._real = real

    def sg_global_draft(self, *args):
        return 4

    def __getattr__(self, name):
        return getattr(self._real, name)


@pytest.mark.parametrize("seed", [41, 42])
def test_global_scenarios_unfused_match_goldens(golden_dir, seed,
                                                monkeypatch):
    """The separate candidates / expand / combine steps (taken when the
    fused global step does not fit on chip) give the same drafts."""
    from suffixgpu_b200 import _lib, global_index
    real = _lib.lib()
    monkeypatch.setattr(global_index, "lib", lambda: _NoFusedDraft(real))
    z = np.load(os.path.join(golden_dir, f"global_{seed}.npz"))
    sc = scenarios.global_scenario(seed)
    got = scenarios.run_scenario(sc, _gpu_drafter, _dev, _host)
    for key in ("draft", "num_valid", "new_counts"):
        np.testing.assert_array_equal(got[key], z["out_" + key], key)


def test_global_draft_rejects_oversized_rows():
    """sg_global_draft returns SG_ERR_UNSUPPORTED (no launch) when the
    continuation block of a row cannot fit in shared memory."""
    import ctypes
    from suffixgpu_b200 import _lib
    L = _lib.lib()
    i64 = torch.zeros(16 * 1024, dtype=torch.int64, device=DEV)
    i32 = torch.zeros(16 * 1024, dtype=torch.int32, device=DEV)
    f32 = torch.zeros(4, dtype=torch.float32, device=DEV)
    p64, p32 = i64.data_ptr(), i32.data_ptr()
    st = L.sg_global_draft(p64, p64, p64, p64, p64, p64, p32, p32, 1024, p32,
                           1024, p64, 1, 16, 1024, 64, 0,
                           ctypes.c_float(0.0), ctypes.c_float(0.0),
                           ctypes.c_float(0.0), ctypes.c_float(0.0),
                           f32.data_ptr(), None, p32, p32,
                           torch.cuda.current_stream().cuda_stream)
    assert st == 4


def _index_pair(**kw):
    from suffixgpu_b200.global_index import GlobalIndex
    return GlobalIndex(device=DEV, **kw), so.GlobalIndex(**kw)


def test_delta_and_query_vs_oracle():
    """Raw _delta_match_backoff / query outputs on a delta with repeats,
    SEP boundaries and a long tail of candidates."""
    rng = np.random.default_rng(11)
    g, o = _index_pair(capacity=4096, delta_capacity=2000, k=6,
                       max_occurrences=16, rebuild_threshold=100000)
    docs = [rng.integers(0, 5, size=int(rng.integers(5, 120))).astype(
        np.int32) for _ in range(20)]
    g.append_documents([_dev(d) for d in docs])
    o.append_documents(docs)
    assert g.delta_len == o.delta_len
    q = rng.integers(0, 5, size=(24, 9)).astype(np.int32)
    qlen = rng.integers(-1, 11, size=24).astype(np.int64)
    caps = np.array([9, 4, 2, 1, 0], dtype=np.int64)
    got = g._delta_match_backoff(_dev(q), _dev(qlen), 9, _dev(caps))
    exp = o._delta_match_backoff(q, qlen, 9, caps)
    for a, b in zip(got, exp):
        np.testing.assert_array_equal(_host(a), b)
    for max_len in (3, 9):
        got = g.query(_dev(q), _dev(qlen), max_len)
        exp = o.query(q, qlen, max_len)
        for a, b in zip(got, exp):
            np.testing.assert_array_equal(_host(a), b)


@pytest.mark.parametrize("delta_capacity,rows,max_len", [
    (1 << 16, 64, 32),   # config 3: one 8-CTA cluster per row
    ((1 << 17) + 5, 6, 16),  # an eighth too large for shared memory: tiles
])
def test_delta_full_size_vs_oracle(delta_capacity, rows, max_len):
    """_delta_match_backoff at the config-3 delta capacity, filled with
    template documents to a little under capacity (plus a capacity above
    the one-pass limit), against the oracle for every cap of the drafter."""
    from suffixgpu_b200 import workloads as wl
    rng = np.random.default_rng(13)
    z = wl.Zipf(1.1, 32000)
    templates = z.draw(rng, (64, 256))
    docs = wl.template_docs(rng, delta_capacity // 1100, 1024, templates, z)
    g, o = _index_pair(capacity=1 << 12, delta_capacity=delta_capacity,
                       k=16, max_occurrences=128,
                       rebuild_threshold=1 << 30)
    g.append_documents([_dev(d) for d in docs])
    o.append_documents(list(docs))
    assert g.delta_len == o.delta_len
    q = wl.template_docs(rng, rows, 600, templates, z)
    qlen = rng.integers(1, 600, size=rows).astype(np.int64)
    qlen[0] = 0
    caps = np.array(so.global_caps(max_len, 8), dtype=np.int64)
    got = g._delta_match_backoff(_dev(q), _dev(qlen), max_len, _dev(caps))
    exp = o._delta_match_backoff(q, qlen, max_len, caps)
    for a, b in zip(got, exp):
        np.testing.assert_array_equal(_host(a), b)


def test_rebuild_eviction_overflow_vs_oracle():
    """Small capacities force eviction, delta overflow and whole-doc
    snapshots; corpus, SA and queries stay identical."""
    rng = np.random.default_rng(12)
    g, o = _index_pair(capacity=300, delta_capacity=90, k=4,
                       max_occurrences=8, rebuild_threshold=60)
    for step in range(25):
        docs = [rng.integers(0, 6, size=int(rng.integers(1, 40))).astype(
            np.int32) for _ in range(int(rng.integers(1, 4)))]
        g.append_documents([_dev(d) for d in docs])
        o.append_documents(docs)
        assert (g.active_len, g.delta_len) == (o.active_len, o.delta_len)
        q = rng.integers(0, 6, size=(5, 6)).astype(np.int32)
        qlen = np.full(5, 6, dtype=np.int64)
        got = g.query(_dev(q), _dev(qlen), 6)
        exp = o.query(q, qlen, 6)
        for a, b in zip(got, exp):
            np.testing.assert_array_equal(_host(a), b)
    np.testing.assert_array_equal(_host(g.corpus), o.corpus)
    np.testing.assert_array_equal(_host(g.sa), o.sa)


def test_background_rebuild_swaps_at_poll():
    """With a rebuild stream the build runs in the background; after it is
    swapped in, the index equals the synchronous one."""
    rng = np.random.default_rng(13)
    from suffixgpu_b200.global_index import GlobalIndex
    side = torch.cuda.Stream()
    g = GlobalIndex(capacity=5000, delta_capacity=800, k=4,
                    max_occurrences=8, rebuild_threshold=400, device=DEV,
                    rebuild_stream=side)
    o = so.GlobalIndex(capacity=5000, delta_capacity=800, k=4,
                       max_occurrences=8, rebuild_threshold=400)
    for _ in range(6):
        docs = [rng.integers(0, 7, size=150).astype(np.int32)
                for _ in range(2)]
        g.append_documents([_dev(d) for d in docs])
        g.wait_rebuild()
        o.append_documents(docs)
    assert g.rebuilds == o.rebuilds and g.rebuilds > 0
    np.testing.assert_array_equal(_host(g.corpus), o.corpus)
    np.testing.assert_array_equal(_host(g.sa), o.sa)


class _NeverDoneEvent:
    def query(self) -> bool:
        return False


def test_delta_overflow_with_rebuild_in_flight():
    """Appends that overflow the delta while a rebuild is in flight drop
    the oldest docs (global_index.py:110-133), checked against the
    oracle with the same fake in-flight event."""
    g, o = _index_pair(capacity=64, delta_capacity=18, k=4,
                       max_occurrences=8, rebuild_threshold=100000)
    for idx in (g, o):
        idx.append_documents([np.full(6, 1, np.int32) if idx is o
                              else _dev(np.full(6, 1, np.int32)),
                              np.full(6, 2, np.int32) if idx is o
                              else _dev(np.full(6, 2, np.int32))])
        idx._rebuild_event = _NeverDoneEvent()
        idx._pending = (idx.active_len, idx.active_doc_lens)
    g.append_documents([_dev(np.full(10, 3, np.int32))])
    o.append_documents([np.full(10, 3, np.int32)])
    assert g.delta_len == o.delta_len <= 18
    for pat in ([3, 3], [2, 2], [1, 1]):
        q = np.array([pat], dtype=np.int32)
        ql = np.array([2], dtype=np.int64)
        got = g.query(_dev(q), _dev(ql), 8)
        exp = o.query(q, ql, 8)
        for a, b in zip(got, exp):
            np.testing.assert_array_equal(_host(a), b)


# ---------------------------------------------------------------------------
# bulk load and persistence
# ---------------------------------------------------------------------------
def _assert_index_equal(g, o):
    assert g.active_len == o.active_len
    assert list(g.active_doc_lens) == list(o.active_doc_lens)
    assert g.delta_len == o.delta_len
    np.testing.assert_array_equal(_host(g.corpus), o.corpus)
    np.testing.assert_array_equal(_host(g.sa), o.sa)
    np.testing.assert_array_equal(_host(g.delta[:g.delta_len]),
                                  o.delta[:o.delta_len])


def test_load_documents_vs_oracle():
    """Two bulk loads (the second evicting part of the first), then normal
    harvesting with rebuilds: corpus, SA, document lengths and queries stay
    identical to the oracle's literal repeated-rebuild process."""
    rng = np.random.default_rng(71)
    g, o = _index_pair(capacity=700, delta_capacity=120, k=5,
                       max_occurrences=12, rebuild_threshold=60)
    for n_docs in (9, 14):
        docs = [rng.integers(0, 6, size=int(rng.integers(1, 90))).astype(
            np.int32) for _ in range(n_docs)]
        docs.append(rng.integers(0, 6, size=730).astype(np.int32))  # trimmed
        g.load_documents([_dev(d) for d in docs])
        o.load_documents(docs)
        _assert_index_equal(g, o)
    q = rng.integers(0, 6, size=(20, 10)).astype(np.int32)
    qlen = rng.integers(0, 11, size=20).astype(np.int64)
    for a, b in zip(g.query(_dev(q), _dev(qlen), 8), o.query(q, qlen, 8)):
        np.testing.assert_array_equal(_host(a), b)
    more = [rng.integers(0, 6, size=int(rng.integers(5, 40))).astype(np.int32)
            for _ in range(6)]
    g.append_documents([_dev(d) for d in more])
    o.append_documents(more)
    _assert_index_equal(g, o)


def test_state_dict_round_trip():
    """state_dict -> torch.save -> load_state_dict into a fresh index gives
    the same corpus, SA, delta and queries, and later harvesting and
    rebuilds continue identically."""
    import io
    from suffixgpu_b200.global_index import GlobalIndex
    rng = np.random.default_rng(72)
    kw = dict(capacity=900, delta_capacity=200, k=5, max_occurrences=12,
              rebuild_threshold=100)
    g = GlobalIndex(device=DEV, **kw)
    docs = [_dev(rng.integers(0, 7, size=int(rng.integers(5, 70))).astype(
        np.int32)) for _ in range(12)]
    g.append_documents(docs)
    assert g.active_len > 0 and g.delta_len > 0
    buf = io.BytesIO()
    torch.save(g.state_dict(), buf)
    buf.seek(0)
    h = GlobalIndex(device=DEV, **kw)
    h.load_state_dict(torch.load(buf))
    for name in ("corpus", "sa"):
        assert torch.equal(getattr(g, name), getattr(h, name)), name
    assert torch.equal(g.delta[:g.delta_len], h.delta[:h.delta_len])
    assert list(g.active_doc_lens) == list(h.active_doc_lens)
    assert list(g.delta_doc_lens) == list(h.delta_doc_lens)
    q = _dev(rng.integers(0, 7, size=(16, 9)).astype(np.int32))
    qlen = _dev(rng.integers(0, 10, size=16).astype(np.int64))
    for a, b in zip(g.query(q, qlen, 8), h.query(q, qlen, 8)):
        assert torch.equal(a, b)
    more = [_dev(rng.integers(0, 7, size=30).astype(np.int32))
            for _ in range(5)]
    g.append_documents(more)
    h.append_documents(more)
    assert torch.equal(g.corpus, h.corpus) and torch.equal(g.sa, h.sa)


def test_tails_before_update_match_tails_after():
    """sg_gather_tails_update (tails read before the scatter, for the
    forked global searches) equals the scatter followed by the plain tail
    gather, with the drafting mask of propose_with_update / propose: -1
    sampled ids, explicit and implicit valid counts, rows that reach or pass
    the row end or the limit, and rows with an empty history."""
    from suffixgpu_b200 import ops
    from suffixgpu_b200._lib import call, ptr
    rng = np.random.default_rng(21)
    b, s, t, p = 40, 96, 6, 32
    tok = rng.integers(0, 50, size=(b, s)).astype(np.int32)
    base = rng.integers(0, s + 3, size=b).astype(np.int32)
    base[:4] = [0, 1, s - 1, s]
    samp = rng.integers(0, 50, size=(b, t)).astype(np.int32)
    samp[rng.random((b, t)) < 0.3] = -1
    for explicit in (False, True):
        vc = rng.integers(0, t + 1, size=b).astype(np.int32) if explicit \
            else None
        limit = s - 5
        # (device copies held in names: a pointer taken from a temporary
        # would outlive its memory)
        d_tok, d_base, d_samp = _dev(tok), _dev(base), _dev(samp)
        d_vc = None if vc is None else _dev(vc)
        tails = torch.empty(b, p, dtype=torch.int32, device=DEV)
        tlen = torch.empty(b, dtype=torch.int64, device=DEV)
        mask = torch.empty(b, dtype=torch.uint8, device=DEV)
        call("sg_gather_tails_update", ptr(d_tok), s, s, ptr(d_base),
             ptr(d_samp), t, ptr(d_vc), limit, ptr(None), b, p, ptr(tails),
             ptr(tlen), ptr(mask), torch.cuda.current_stream().cuda_stream)
        # reference: the scatter, then the tails of the updated rows
        upd = _dev(tok)
        new = ops.scatter_append(upd, d_base, d_vc, d_samp)
        exp_t = torch.empty(b, p, dtype=torch.int32, device=DEV)
        exp_l = torch.empty(b, dtype=torch.int64, device=DEV)
        call("sg_gather_tails", ptr(upd), s, s, ptr(new), b, p, ptr(exp_t),
             ptr(exp_l), torch.cuda.current_stream().cuda_stream)
        cnt = (samp != -1).sum(1) if vc is None else vc
        exp_m = (cnt > 0) & (_host(new) < limit)
        np.testing.assert_array_equal(_host(tlen), _host(exp_l))
        np.testing.assert_array_equal(_host(mask).astype(bool), exp_m)
        # the tails of rows that draft are what the searches read
        np.testing.assert_array_equal(_host(tails)[exp_m], _host(exp_t)[exp_m])
        # the buffer was not touched
        np.testing.assert_array_equal(_host(d_tok), tok)
    # propose (no update): tails of the rows as they are, the given mask
    m = (rng.random(b) < 0.7)
    d_tok, d_base, d_m = _dev(tok), _dev(base), _dev(m.astype(np.uint8))
    call("sg_gather_tails_update", ptr(d_tok), s, s, ptr(d_base), ptr(None),
         0, ptr(None), s, ptr(d_m), b, p, ptr(tails), ptr(tlen), ptr(mask),
         torch.cuda.current_stream().cuda_stream)
    call("sg_gather_tails", ptr(d_tok), s, s, ptr(d_base), b, p, ptr(exp_t),
         ptr(exp_l), torch.cuda.current_stream().cuda_stream)
    np.testing.assert_array_equal(_host(tails), _host(exp_t))
    np.testing.assert_array_equal(_host(mask).astype(bool), m)
