"""GPU parity of the incremental suffix-array rebuild
(sg_suffix_array_append): every merged array equals a from-scratch build of
the same snapshot (itself pinned to the oracle), bit for bit, over chains
of rebuilds with eviction; the reported rounds always bound the snapshot's
longest common prefix; and a GlobalIndex with incremental rebuilds stays
identical to the oracle's index."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import suffix_oracle as so

pytestmark = pytest.mark.gpu

DEV = "cuda"
PAD = 2 ** 31 - 1
SEP = -2


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def _host(t):
    return t.detach().cpu().numpy().copy()


def _full(tok: np.ndarray):
    """Full GPU build: (sa, rounds); rounds = ceil(log2(max LCP + 1))."""
    from suffixgpu_b200 import ops
    t = _dev(tok.astype(np.int32))
    out = torch.empty(len(tok), dtype=torch.int32, device=DEV)
    r = ops.build_suffix_array_into(t, out) if len(tok) else 0
    return _host(out), r


def _append(tok, prev_sa, prev_n, evicted, kept, prev_rounds):
    from suffixgpu_b200 import ops
    out = torch.empty(len(tok), dtype=torch.int32, device=DEV)
    r = ops.append_suffix_array_into(_dev(tok.astype(np.int32)), out,
                                     _dev(prev_sa.astype(np.int32)), prev_n,
                                     evicted, kept, prev_rounds)
    return _host(out), r


def _doc_source(seed: int, vocab: int, n_templates: int, t_len: int,
                p_exact: float):
    """Documents cut from a few templates: exact repeats (long common
    prefixes across SEP boundaries) and substituted variants."""
    rng = np.random.default_rng(seed)
    temps = [rng.integers(0, vocab, size=int(rng.integers(t_len // 2,
                                                           t_len + 1)))
             for _ in range(n_templates)]

    def doc():
        t = temps[int(rng.integers(n_templates))].copy()
        if rng.random() > p_exact:
            sub = rng.random(t.shape) < 0.05
            t[sub] = rng.integers(0, vocab, size=int(sub.sum()))
        if rng.random() < 0.3:
            t = t[:int(rng.integers(1, len(t) + 1))]
        return np.concatenate([t, [SEP]]).astype(np.int32)
    return rng, doc


@pytest.mark.parametrize("cap,vocab,n_templates,t_len,p_exact,steps", [
    (3000, 4, 6, 120, 0.5, 40),          # tiny alphabet, many end ties
    (200_000, 50, 40, 1500, 0.6, 25),    # long exact repeats
    (1 << 20, 32000, 512, 1024, 0.3, 12),  # config-3-like documents
])
def test_append_chain_equals_full_build(cap, vocab, n_templates, t_len,
                                        p_exact, steps):
    """Chains of rebuilds with whole-document eviction: the merged array is
    the full build's and the rounds bound never undershoots."""
    rng, doc = _doc_source(cap + vocab, vocab, n_templates, t_len, p_exact)
    docs = []
    total = 0
    while total < cap // 2:
        docs.append(doc())
        total += len(docs[-1])
    corpus = np.concatenate(docs)
    lens = [len(d) for d in docs]
    snap = np.concatenate([corpus, [PAD]]).astype(np.int32)
    sa, rounds = _full(snap)
    used = 0
    for _ in range(steps):
        new = [doc()]
        for _ in range(int(rng.integers(0, 40))):
            d = doc()
            if sum(len(x) for x in new) + len(d) > cap // 3:
                break
            new.append(d)
        z = np.concatenate(new)
        keep_start, i = 0, 0
        while len(corpus) - keep_start + len(z) > cap - 1:
            keep_start += lens[i]
            i += 1
        lens = lens[i:] + [len(d) for d in new]
        kept = len(corpus) - keep_start
        corpus = np.concatenate([corpus[keep_start:], z])
        nxt = np.concatenate([corpus, [PAD]]).astype(np.int32)
        exp, exp_r = _full(nxt)
        got, got_r = _append(nxt, sa, len(snap), keep_start, kept, rounds)
        np.testing.assert_array_equal(got, exp)
        assert got_r >= exp_r
        used += (1 << rounds) < kept
        sa, rounds, snap = got, got_r, nxt
    assert used > 0  # the merge path ran, not only the full-build fallback


def test_append_small_vs_oracle():
    """Small snapshots checked directly against the oracle's build,
    including snapshots without a sentinel column (capacity reached)."""
    rng, doc = _doc_source(5, 3, 4, 30, 0.5)
    corpus = np.concatenate([doc() for _ in range(12)])
    snap = corpus.copy()  # no sentinel
    sa, rounds = _full(snap)
    for step in range(20):
        z = np.concatenate([doc() for _ in range(int(rng.integers(1, 4)))])
        ev = int(rng.integers(0, len(corpus) // 3))
        kept = len(corpus) - ev
        corpus = np.concatenate([corpus[ev:], z])
        nxt = corpus.copy() if step % 2 else np.concatenate(
            [corpus, [PAD]]).astype(np.int32)
        got, got_r = _append(nxt, sa, len(snap), ev, kept, rounds)
        np.testing.assert_array_equal(got, so.build_suffix_array(nxt))
        sa, rounds, snap = got, got_r, nxt


def test_append_edge_cases():
    """Everything evicted, a bound that covers the whole kept part (full
    build inside), a one-token tail, extreme token values."""
    rng = np.random.default_rng(9)
    base = rng.integers(-3, 4, size=500).astype(np.int32)
    base[::37] = PAD
    base[5::41] = -(2 ** 31)
    sa, r = _full(base)
    # nothing kept
    z = rng.integers(0, 3, size=50).astype(np.int32)
    got, _ = _append(z, sa, len(base), len(base), 0, r)
    np.testing.assert_array_equal(got, so.build_suffix_array(z))
    # bound larger than the kept part
    nxt = np.concatenate([base[100:], z]).astype(np.int32)
    got, _ = _append(nxt, sa, len(base), 100, 400, 20)
    np.testing.assert_array_equal(got, so.build_suffix_array(nxt))
    # nothing appended, bound 0 on a string whose first tokens are distinct
    uniq = np.arange(300, dtype=np.int32)[::-1].copy()
    usa, ur = _full(uniq)
    assert ur == 0
    got, gr = _append(uniq[10:].copy(), usa, 300, 10, 290, ur)
    np.testing.assert_array_equal(got, so.build_suffix_array(uniq[10:]))
    assert gr == 0
    # extreme tokens in the appended part
    nxt = np.concatenate([base, np.array([PAD, -(2 ** 31), PAD, 0],
                                         np.int32)]).astype(np.int32)
    got, _ = _append(nxt, sa, len(base), 0, len(base), r)
    np.testing.assert_array_equal(got, so.build_suffix_array(nxt))


def test_append_rejects_bad_arguments():
    from suffixgpu_b200 import ops
    t = _dev(np.arange(10, dtype=np.int32))
    out = torch.empty(10, dtype=torch.int32, device=DEV)
    prev = torch.arange(10, dtype=torch.int32, device=DEV)
    with pytest.raises(RuntimeError):
        ops.append_suffix_array_into(t, out, prev, 10, 5, 6, 0)  # past prev
    with pytest.raises(RuntimeError):
        ops.append_suffix_array_into(t, out, prev, 10, 0, 11, 0)  # kept > n


def test_global_index_incremental_matches_oracle():
    """Template documents harvested into an index that evicts: the
    incremental rebuilds (and the full ones they fall back to) keep
    corpus, SA and queries identical to the oracle's index."""
    from suffixgpu_b200 import workloads as wl
    from suffixgpu_b200.global_index import GlobalIndex
    rng = np.random.default_rng(31)
    z = wl.Zipf(1.1, 32000)
    templates = z.draw(rng, (32, 256))
    kw = dict(capacity=1 << 16, delta_capacity=1 << 13, k=8,
              max_occurrences=32, rebuild_threshold=4096)
    g = GlobalIndex(device=DEV, **kw)
    o = so.GlobalIndex(**kw)
    builds = set()
    for step in range(40):
        docs = list(wl.template_docs(rng, 4, int(rng.integers(200, 900)),
                                     templates, z, p_sub=0.02))
        g.append_documents([_dev(d) for d in docs])
        o.append_documents(docs)
        builds.add(g.last_build)
        assert (g.active_len, g.delta_len) == (o.active_len, o.delta_len)
    assert "append" in builds
    np.testing.assert_array_equal(_host(g.corpus), o.corpus)
    np.testing.assert_array_equal(_host(g.sa), o.sa)
    q = wl.template_docs(rng, 16, 40, templates, z)
    qlen = np.full(16, 40, dtype=np.int64)
    for a, b in zip(g.query(_dev(q), _dev(qlen), 32), o.query(q, qlen, 32)):
        np.testing.assert_array_equal(_host(a), b)
