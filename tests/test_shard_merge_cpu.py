"""The sharded suffix-array merge on CPU ranks (gloo, 127.0.0.1): the
protocol of distributed.ShardedSuffixDrafter restated in numpy and run by
spawned processes with real collectives, against the oracle's single
index (suffix_gpu/sa_search.py:110-163 and the strided sample of
suffix_gpu/global_index.py:339-352).

Each rank holds the suffixes that start in its share of the corpus positions
(suffix-array order) and their global ranks. It searches every row's tail
on that shard for every length; the bounds summed over the ranks (an
all-reduce) must equal search_interval on the whole suffix array. The
longest-match-first variant takes a MAX of each rank's longest local match
and must give the same per-cap lengths. Each rank then writes the sampled
positions it holds, zeros elsewhere; the sum over the ranks must be the
whole index's samples, every sample held by exactly one rank.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

R = 12
CAPS = np.array([8, 4, 2], dtype=np.int64)
M = 8


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _corpus_and_queries():
    from suffixgpu_b200 import workloads as wl
    rng = np.random.default_rng(123)
    z = wl.Zipf(1.1, 9)
    templates = z.draw(rng, (5, 20))
    docs = wl.template_docs(rng, 30, 40, templates, z, p_sub=0.1)
    corpus = np.concatenate([np.append(d, -2) for d in docs]).astype(np.int64)
    n = corpus.size + 40
    corpus = np.concatenate([corpus, np.full(40, np.iinfo(np.int32).max)])
    q = wl.template_docs(rng, 10, M, templates, z, p_sub=0.1).astype(np.int64)
    qlen = rng.integers(0, M + 1, size=10).astype(np.int64)
    return corpus, n, q, qlen


def _cmp(corpus, n, pos, pat, plen):
    """_cmp_pattern (sa_search.py:25-63) of the suffix at pos."""
    for j in range(plen):
        t = corpus[pos + j] if pos + j < n else -1
        if t != pat[j]:
            return -1 if t < pat[j] else 1
    return 0


def _bounds(sa_part, corpus, n, pat, plen):
    """Lower / upper bound of the pattern in a sorted list of suffixes."""
    lo, hi = 0, len(sa_part)
    while lo < hi:
        mid = (lo + hi) // 2
        if _cmp(corpus, n, sa_part[mid], pat, plen) < 0:
            lo = mid + 1
        else:
            hi = mid
    a = lo
    lo, hi = a, len(sa_part)
    while lo < hi:
        mid = (lo + hi) // 2
        if _cmp(corpus, n, sa_part[mid], pat, plen) <= 0:
            lo = mid + 1
        else:
            hi = mid
    return a, lo


def _per_cap(bounds_sum, qlen):
    best = np.zeros((len(qlen), len(CAPS)), dtype=np.int64)
    for b in range(len(qlen)):
        for c, cap in enumerate(CAPS):
            for ln in range(1, M + 1):
                s, e = bounds_sum[b, ln - 1]
                if ln <= cap and ln <= qlen[b] and e > s:
                    best[b, c] = ln
    return best


def _worker(rank: int, world: int, port: int, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import suffix_oracle as so
        corpus, n, q, qlen = _corpus_and_queries()
        sa = so.build_suffix_array(corpus[:n])
        lo, hi = rank * n // world, (rank + 1) * n // world
        keep = (sa >= lo) & (sa < hi)
        shard_pos, shard_rank = sa[keep], np.nonzero(keep)[0]
        b = q.shape[0]
        local = np.zeros((b, M, 2), dtype=np.int64)
        longest = np.zeros(b, dtype=np.int64)
        for r in range(b):
            for ln in range(1, int(qlen[r]) + 1):
                pat = q[r, qlen[r] - ln:qlen[r]]
                local[r, ln - 1] = _bounds(shard_pos, corpus, n, pat, ln)
                if local[r, ln - 1, 1] > local[r, ln - 1, 0]:
                    longest[r] = ln
        tot = torch.from_numpy(local.copy())
        dist.all_reduce(tot, op=dist.ReduceOp.SUM)
        lmax = torch.from_numpy(longest.copy())
        dist.all_reduce(lmax, op=dist.ReduceOp.MAX)
        bounds_sum = tot.numpy()
        best = _per_cap(bounds_sum, qlen)
        # this rank's samples: positions it holds, zeros elsewhere
        samples = np.zeros((b, len(CAPS), R), dtype=np.int64)
        owned = np.zeros((b, len(CAPS), R), dtype=np.int64)
        for r in range(b):
            for c in range(len(CAPS)):
                ln = best[r, c]
                if ln == 0:
                    continue
                start, end = bounds_sum[r, ln - 1]
                ilen = end - start
                l0, l1 = local[r, ln - 1]
                for j in range(min(ilen, R)):
                    g = start + (j * ilen // R if ilen > R else j)
                    k = np.searchsorted(shard_rank[l0:l1], g) + l0
                    if k < l1 and shard_rank[k] == g:
                        samples[r, c, j] = shard_pos[k]
                        owned[r, c, j] = 1
        st = torch.from_numpy(samples)
        ow = torch.from_numpy(owned)
        dist.all_reduce(st, op=dist.ReduceOp.SUM)
        dist.all_reduce(ow, op=dist.ReduceOp.SUM)
        out.put((rank, {"bounds": bounds_sum, "longest": lmax.numpy(),
                        "best": best, "samples": st.numpy(),
                        "owned": ow.numpy()}))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_shard_merge_equals_single_index(world):
    from oracle import suffix_oracle as so
    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q_out))
             for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        r, v = q_out.get(timeout=240)
        res[r] = v
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    corpus, n, q, qlen = _corpus_and_queries()
    sa = so.build_suffix_array(corpus[:n])
    b = q.shape[0]
    # summed bounds = search_interval on the whole suffix array
    lengths = np.arange(1, M + 1)
    offs = np.arange(M)
    idx = qlen[:, None, None] - lengths[None, :, None] + offs[None, None, :]
    pat = np.where((offs[None, None, :] < lengths[None, :, None]) & (idx >= 0),
                   q[np.arange(b)[:, None, None], np.clip(idx, 0, M - 1)], 0)
    s_all, e_all = so.search_interval(sa, corpus[:n], pat.reshape(b * M, M),
                                      np.broadcast_to(lengths,
                                                      (b, M)).reshape(-1))
    live = lengths[None, :] <= qlen[:, None]
    for r in range(world):
        got = res[r]["bounds"]
        np.testing.assert_array_equal(got[..., 0][live],
                                      s_all.reshape(b, M)[live])
        np.testing.assert_array_equal(got[..., 1][live],
                                      e_all.reshape(b, M)[live])
    # per-cap best lengths = the oracle's, and = min(cap, MAX of longest)
    exp_len, exp_s, exp_e = so.suffix_match_backoff(sa, corpus[:n], q, qlen,
                                                    M, CAPS)
    for r in range(world):
        np.testing.assert_array_equal(res[r]["best"], exp_len)
        np.testing.assert_array_equal(
            np.minimum(CAPS[None, :], res[r]["longest"][:, None]), exp_len)
    # samples: the whole index's strided sample, each held by one rank
    for r in range(world):
        for bi in range(b):
            for c in range(len(CAPS)):
                if exp_len[bi, c] == 0:
                    continue
                ilen = exp_e[bi, c] - exp_s[bi, c]
                cnt = min(ilen, R)
                js = np.arange(cnt)
                g = exp_s[bi, c] + (js * ilen // R if ilen > R else js)
                np.testing.assert_array_equal(res[r]["samples"][bi, c, :cnt],
                                              sa[g])
                assert (res[r]["owned"][bi, c, :cnt] == 1).all()
    assert (exp_e - exp_s).max() > R  # strided samples were exercised
