"""Multi-rank host logic of the multi-GPU drafter on CPU: two gloo ranks
(spawned processes, 127.0.0.1) exchange harvested documents and agree on
rebuild swaps. The per-rank index here is the oracle's, fed exactly as the
product's multi-GPU drafters feed their GlobalIndex, so the test shows the
replicas stay identical to one index that receives all ranks' documents in
rank order."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _docs_for(rank: int, step: int) -> list[np.ndarray]:
    rng = np.random.default_rng(1000 * step + rank)
    n = int(rng.integers(0, 4))  # some steps give a rank nothing
    return [rng.integers(0, 6, size=int(rng.integers(1, 40))).astype(np.int32)
            for _ in range(n)]


def _worker(rank: int, world: int, port: int, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from suffixgpu_b200.distributed import agree_all, exchange_documents
        from oracle import suffix_oracle as so
        res = {}
        # exchange: ragged, empty on some ranks, rank order kept
        got = exchange_documents(
            [torch.tensor([1, 2, 3], dtype=torch.int32)] if rank == 0 else
            [torch.tensor([7], dtype=torch.int32),
             torch.tensor([8, 9], dtype=torch.int32)])
        res["exchange"] = [g.tolist() for g in got]
        res["empty"] = [g.tolist() for g in exchange_documents([])]
        res["agree_mixed"] = agree_all(rank == 0)
        res["agree_all"] = agree_all(True)
        # replicas fed through the exchange
        idx = so.GlobalIndex(capacity=300, delta_capacity=90, k=4,
                             max_occurrences=8, rebuild_threshold=50)
        for step in range(12):
            mine = [torch.from_numpy(d) for d in _docs_for(rank, step)]
            all_docs = exchange_documents(mine)
            if all_docs:
                idx.append_documents([d.numpy() for d in all_docs])
        res["corpus"] = idx.corpus.copy()
        res["sa"] = idx.sa.copy()
        res["delta"] = idx.delta[:idx.delta_len].copy()
        res["doc_lens"] = list(idx.active_doc_lens)
        out.put((rank, res))
    finally:
        dist.destroy_process_group()


def test_two_rank_exchange_and_replicas():
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, out))
             for r in range(2)]
    for p in procs:
        p.start()
    results = dict(out.get(timeout=180) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    r0, r1 = results[0], results[1]
    assert r0["exchange"] == r1["exchange"] == [[1, 2, 3], [7], [8, 9]]
    assert r0["empty"] == r1["empty"] == []
    assert r0["agree_mixed"] is False and r1["agree_mixed"] is False
    assert r0["agree_all"] is True and r1["agree_all"] is True
    # the replicas are identical ...
    for key in ("corpus", "sa", "delta"):
        np.testing.assert_array_equal(r0[key], r1[key], key)
    assert r0["doc_lens"] == r1["doc_lens"]
    # ... and equal one index fed all documents in rank order
    from oracle import suffix_oracle as so
    ref = so.GlobalIndex(capacity=300, delta_capacity=90, k=4,
                         max_occurrences=8, rebuild_threshold=50)
    for step in range(12):
        docs = _docs_for(0, step) + _docs_for(1, step)
        if docs:
            ref.append_documents(docs)
    np.testing.assert_array_equal(r0["corpus"], ref.corpus)
    np.testing.assert_array_equal(r0["sa"], ref.sa)
    assert r0["doc_lens"] == list(ref.active_doc_lens)
