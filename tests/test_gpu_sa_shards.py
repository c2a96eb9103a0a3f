"""The sharded suffix-array drafter (distributed.ShardedSuffixDrafter) and
its kernels, bit-exact against the numpy oracle's single index.

* sg_shard_extract: each shard's (position, global rank) lists equal the
  whole suffix array restricted to the shard's positions;
* sg_shard_bounds summed over the shards equals search_interval over the
  whole suffix array for every (row, length) of suffix_match_backoff
  (suffix_gpu/sa_search.py:110-163), for 1, 2, 3 and 8 shards;
* the drafter's whole step (tails exchange, shard search, summed bounds,
  sample resolution, samples returned to their owner, fused global step)
  with G ranks emulated on one GPU by threads whose collectives are
  host-side barriers over one CUDA stream: every rank's drafts equal the
  oracle drafter's for the same rows (suffix_gpu/proposer.py:216-327,
  strided sample global_index.py:339-352), including config 5's drafter
  settings (k = 32, P = 64, R = 256);
* two real ranks over NCCL on two GPUs (skipped on one-GPU machines).
"""

from __future__ import annotations

import os
import socket
import threading

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


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.fixture(scope="module")
def world_one():
    """A one-rank NCCL group (the drafters need an initialised group)."""
    import torch.distributed as dist
    if dist.is_initialized():
        yield
        return
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(_free_port())
    torch.cuda.set_device(0)
    dist.init_process_group("nccl", rank=0, world_size=1)
    try:
        yield
    finally:
        dist.destroy_process_group()


def _loaded_index(seed, capacity, n_docs, doc_len, vocab=40):
    from suffixgpu_b200 import workloads as wl
    from suffixgpu_b200.global_index import GlobalIndex
    rng = np.random.default_rng(seed)
    z = wl.Zipf(1.1, vocab)
    templates = z.draw(rng, (8, 30))
    docs = wl.template_docs(rng, n_docs, doc_len, templates, z)
    g = GlobalIndex(capacity=capacity, delta_capacity=256, k=8,
                    max_occurrences=32, device=DEV)
    g.load_documents([_dev(d) for d in docs])
    return g, rng, templates, z


@pytest.mark.parametrize("parts", [1, 2, 3, 8])
def test_extract_and_summed_bounds_equal_whole_index(parts):
    from suffixgpu_b200 import workloads as wl
    from suffixgpu_b200.distributed import SuffixArrayShard
    g, rng, templates, z = _loaded_index(5 + parts, 4000, 60, 50)
    sa = _host(g.sa)
    corpus = _host(g.corpus)
    shards = [SuffixArrayShard(g, r, parts) for r in range(parts)]
    for sh in shards:
        keep = (sa >= sh.lo) & (sa < sh.hi)
        np.testing.assert_array_equal(_host(sh.pos)[:sh.size], sa[keep])
        np.testing.assert_array_equal(_host(sh.rank)[:sh.size],
                                      np.nonzero(keep)[0])
    # packed rows: template tails (most lengths match), a masked row, short
    b, m = 24, 16
    q = wl.template_docs(rng, b, m, templates, z)
    tlen = rng.integers(0, m + 1, size=b)
    tlen[:3] = [0, 1, m]
    mask = np.ones(b, dtype=np.int32)
    mask[3] = 0
    rows = np.concatenate([q, tlen[:, None], mask[:, None]], axis=1)
    total = None
    for sh in shards:
        bd = sh.bounds(_dev(rows.astype(np.int32)), m)
        total = bd.to(torch.int64) if total is None else total + bd
    total = _host(total)
    lengths = np.arange(1, m + 1)
    offs = np.arange(m)
    idx = tlen[:, None, None] - lengths[None, :, None] + offs[None, None, :]
    pat = np.where((offs[None, None, :] < lengths[None, :, None])
                   & (idx >= 0), q[np.arange(b)[:, None, None],
                                   np.clip(idx, 0, m - 1)], 0)
    st, en = so.search_interval(sa, corpus, pat.reshape(b * m, m),
                                np.broadcast_to(lengths, (b, m)).reshape(-1))
    live = (lengths[None, :] <= tlen[:, None]) & (mask[:, None] > 0)
    np.testing.assert_array_equal(total[..., 0][live], st.reshape(b, m)[live])
    np.testing.assert_array_equal(total[..., 1][live], en.reshape(b, m)[live])
    assert (total[~live] == 0).all()
    assert (en - st).max() > 32  # intervals wider than R exist
    # longest match: MAX over the shards = the longest found length (found
    # lengths are a prefix 1..L), or M + 1 for a tail holding -1
    found = live & (en > st).reshape(b, m)
    exp_long = np.where(found.any(axis=1),
                        m - np.argmax(found[:, ::-1], axis=1), 0)
    for L in range(b):
        assert found[L, :exp_long[L]].all(), L  # the prefix property
    rows_d = _dev(rows.astype(np.int32))
    longest = torch.stack([sh.longest(rows_d, m) for sh in shards]).amax(0)
    np.testing.assert_array_equal(_host(longest), exp_long)
    rows_neg = rows.copy()
    rows_neg[5, int(tlen[5]) - 1] = -1 if tlen[5] > 0 else 0
    if tlen[5] > 0:
        lneg = torch.stack([sh.longest(_dev(rows_neg.astype(np.int32)), m)
                            for sh in shards]).amax(0)
        assert int(lneg[5]) == m + 1
    # bounds of the cap-selected lengths only
    caps = np.array([16, 8, 4, 2], dtype=np.int64)
    sel = None
    for sh in shards:
        bd = sh.bounds(rows_d, m, longest=longest, caps=_dev(caps))
        sel = bd.to(torch.int64) if sel is None else sel + bd
    sel = _host(sel)
    for bi in range(b):
        need = {int(min(c, exp_long[bi])) for c in caps} - {0}
        for li in range(m):
            if li + 1 in need:
                np.testing.assert_array_equal(sel[bi, li], total[bi, li])
            else:
                assert (sel[bi, li] == 0).all()


class _ThreadComm:
    """Collectives among threads standing in for ranks. Each rank hands in
    its tensor with an event on its current stream; after a barrier every
    rank's current stream waits for all those events, combines, and records
    a second event; after a second barrier every stream waits for all of
    those, so that no rank overwrites an input another is still reading
    (the synchronisation a real collective gives its streams)."""

    def __init__(self, world: int):
        self.world = world
        self.barrier = threading.Barrier(world, timeout=120)
        self.slots = [None] * world
        self.ready = [None] * world
        self.done = [None] * world

    def _run(self, rank, t, combine):
        cur = torch.cuda.current_stream()
        ev = torch.cuda.Event()
        ev.record(cur)
        self.slots[rank], self.ready[rank] = t, ev
        self.barrier.wait()
        for e in self.ready:
            cur.wait_event(e)
        combine(self.slots)
        ev2 = torch.cuda.Event()
        ev2.record(cur)
        self.done[rank] = ev2
        self.barrier.wait()
        for e in self.done:
            cur.wait_event(e)
        self.barrier.wait()  # slots free for the next collective

    def view(self, rank: int):
        comm = self

        class _R:
            def all_gather(self, out, inp):
                comm._run(rank, inp,
                          lambda sl: torch.cat(sl, dim=0, out=out))

            def all_reduce_sum(self, t):
                src = t.clone()

                def comb(sl):
                    t.copy_(sum(x.to(torch.int64) for x in sl).to(t.dtype))
                comm._run(rank, src, comb)

            def all_reduce_max(self, t):
                src = t.clone()
                comm._run(rank, src,
                          lambda sl: t.copy_(torch.stack(sl).amax(dim=0)))

            def reduce_scatter_sum(self, out, inp):
                n = out.numel()

                def comb(sl):
                    tot = sum(x[rank * n:(rank + 1) * n].to(torch.int64)
                              for x in sl)
                    out.copy_(tot.to(out.dtype))
                comm._run(rank, inp, comb)
        return _R()


def _emulated_drafters(world: int, cfg: dict):
    from suffixgpu_b200.distributed import (ShardedSuffixDrafter,
                                            SuffixArrayShard)
    comm = _ThreadComm(world)
    ds = []
    for r in range(world):
        d = ShardedSuffixDrafter(device=DEV, **cfg)
        d.global_index.on_swap.remove(d.shard.refresh)
        d.rank, d.world_size = r, world
        d.shard = SuffixArrayShard(d.global_index, r, world)
        d._comm = comm.view(r)
        ds.append(d)
    return ds, comm


def _run_emulated(sc: dict, world: int, prefill=None, mode="auto"):
    """Each emulated rank drafts its share of the rows and ingests every
    document itself (the ingestion exchange is not emulated: replicas stay
    identical because they receive the same documents)."""
    data = sc["data"]
    b = data["token_ids"].shape[0]
    per = b // world
    ds, comm = _emulated_drafters(world, sc["drafter"])
    for d in ds:
        d.length_search = mode
    results = [None] * world
    errors = []

    def work(r):
        try:
            d = ds[r]
            if prefill is not None:
                d.global_index.load_documents([_dev(x) for x in prefill])
            rows = slice(r * per, (r + 1) * per)
            tok = _dev(data["token_ids"][rows])
            n = _dev(data["num_tokens"][rows])
            out = {"draft": [], "num_valid": [], "new_counts": []}
            for op, arg in sc["ops"]:
                if op == "pwu":
                    dr, nv, n = d.propose_with_update(
                        n, tok, _dev(data["sampled"][arg][rows]))
                    torch.cuda.synchronize()
                    out["draft"].append(_host(dr))
                    out["num_valid"].append(_host(nv))
                    out["new_counts"].append(_host(n))
                elif op == "harvest":
                    docs = data["docs"]
                    d.harvest_rows([_dev(docs[j]) for j in arg],
                                   [int(docs[j].shape[0]) for j in arg])
                elif op == "poll":
                    d.poll()
            results[r] = {k: np.stack(v) for k, v in out.items()}
            results[r]["sa"] = _host(d.global_index.sa)
        except BaseException as e:  # reported by the main thread
            errors.append(e)
            comm.barrier.abort()  # the other ranks stop at their next wait

    threads = [threading.Thread(target=work, args=(r,)) for r in range(world)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=600)
    if errors:
        raise errors[0]
    return results


@pytest.mark.parametrize("mode", ["all", "longest"])
@pytest.mark.parametrize("world", [2, 3])
@pytest.mark.parametrize("seed", [41, 45])
def test_emulated_ranks_match_oracle(world_one, world, seed, mode):
    sc = scenarios.global_scenario(seed, steps=10)
    exp = scenarios.run_scenario(sc, so.SuffixDrafter, lambda a: a.copy(),
                                 lambda a: np.asarray(a).copy())
    got = _run_emulated(sc, world, mode=mode)
    per = sc["data"]["token_ids"].shape[0] // world
    for r in range(world):
        rows = slice(r * per, (r + 1) * per)
        for key in ("draft", "num_valid", "new_counts"):
            np.testing.assert_array_equal(got[r][key], exp[key][:, rows],
                                          f"rank {r} {key}")
        np.testing.assert_array_equal(got[r]["sa"], exp["sa"])


@pytest.mark.parametrize("mode", ["all", "longest"])
def test_emulated_ranks_config5_settings_match_oracle(world_one, mode):
    """Config 5's drafter (k = 32, P = 64, R = 256, caps 64..2) on 4
    emulated ranks over a 2^18-token template corpus, 3 decode steps with
    harvests between them."""
    from suffixgpu_b200 import workloads as wl
    data = wl.config5(seed=57, rows=16, s=4096, n_docs=256, doc_len=1023,
                      steps=3)
    cfg = dict(wl.CONFIG5_DRAFTER)
    cfg["global_capacity"] = 1 << 19
    ops = []
    for j in range(3):
        ops += [("harvest", [2 * j, 2 * j + 1]), ("poll", None), ("pwu", j)]
    docs = list(data["corpus_docs"])
    data = dict(data)
    data["docs"] = [x[:1000] for x in data["token_ids"]]
    sc = {"drafter": cfg, "data": data, "ops": ops}
    ocfg = dict(cfg)
    o = so.SuffixDrafter(**ocfg)
    o.global_index.load_documents(docs)
    tok, n = data["token_ids"].copy(), data["num_tokens"].copy()
    exp = {"draft": [], "num_valid": []}
    for op, arg in ops:
        if op == "harvest":
            o.harvest_rows([data["docs"][j] for j in arg], [1000] * len(arg))
        elif op == "pwu":
            dr, nv, n = o.propose_with_update(n, tok, data["sampled"][arg])
            exp["draft"].append(dr)
            exp["num_valid"].append(nv)
    got = _run_emulated(sc, 4, prefill=docs, mode=mode)
    for r in range(4):
        rows = slice(4 * r, 4 * r + 4)
        np.testing.assert_array_equal(got[r]["draft"],
                                      np.stack(exp["draft"])[:, rows])
        np.testing.assert_array_equal(got[r]["num_valid"],
                                      np.stack(exp["num_valid"])[:, rows])
    assert (np.stack(exp["num_valid"]) > 0).mean() > 0.3


def _nccl_worker(rank, port, sc, q):
    import torch.distributed as dist
    from suffixgpu_b200.distributed import ShardedSuffixDrafter
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=2)
    try:
        dev = torch.device("cuda", rank)
        data = sc["data"]
        b = data["token_ids"].shape[0] // 2
        rows = slice(rank * b, (rank + 1) * b)
        d = ShardedSuffixDrafter(device=dev, **sc["drafter"])
        tok = torch.from_numpy(data["token_ids"][rows].copy()).to(dev)
        n = torch.from_numpy(data["num_tokens"][rows].copy()).to(dev)
        out = []
        for op, arg in sc["ops"]:
            if op == "pwu":
                s = torch.from_numpy(data["sampled"][arg][rows].copy()).to(dev)
                dr, nv, n = d.propose_with_update(n, tok, s)
                out.append((dr.cpu().numpy(), nv.cpu().numpy()))
            elif op == "harvest":
                # each rank contributes every other document; the exchange
                # gives both ranks all of them in rank order
                mine = [j for i, j in enumerate(arg) if i % 2 == rank]
                d.harvest_rows([torch.from_numpy(data["docs"][j].copy()).to(
                    dev) for j in mine],
                    [int(data["docs"][j].shape[0]) for j in mine])
            elif op == "poll":
                d.poll()
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpus_nccl_match_oracle():
    import torch.multiprocessing as mp
    sc = scenarios.global_scenario(46, steps=10)
    # the oracle receives each harvest in the exchange's order
    ops = []
    for op, arg in sc["ops"]:
        if op == "harvest":
            arg = [j for i, j in enumerate(arg) if i % 2 == 0] + \
                  [j for i, j in enumerate(arg) if i % 2 == 1]
        ops.append((op, arg))
    exp = scenarios.run_scenario(dict(sc, ops=ops), so.SuffixDrafter,
                                 lambda a: a.copy(),
                                 lambda a: np.asarray(a).copy())
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_worker, args=(r, port, sc, q))
             for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        r, out = q.get(timeout=300)
        res[r] = out
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    b = sc["data"]["token_ids"].shape[0] // 2
    for step in range(len(exp["draft"])):
        for r in range(2):
            rows = slice(r * b, (r + 1) * b)
            np.testing.assert_array_equal(res[r][step][0],
                                          exp["draft"][step][rows])
            np.testing.assert_array_equal(res[r][step][1],
                                          exp["num_valid"][step][rows])
