"""The multi-GPU drafters on GPUs. The replicated-index drafter: with one
rank it is the plain drafter; with two ranks (NCCL, one process per GPU;
skipped on one-GPU machines) each rank's drafts equal those of one drafter
that drafts all rows and receives every rank's harvested documents in rank
order, and replicas with background rebuilds stay identical. The sharded
suffix-array drafter: tested in test_gpu_sa_shards.py."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch

import scenarios

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _split(lst, world, rank):
    return [x for i, x in enumerate(lst) if i % world == rank]


def _run(sc, drafter, rows, world, rank, dev, async_rebuild=False):
    """Drive a global scenario; this rank drafts ``rows`` and harvests
    every world-th document of each harvest. Returns the drafts and an
    index checksum per step."""
    data = sc["data"]
    tok = torch.from_numpy(data["token_ids"][rows].copy()).to(dev)
    n = torch.from_numpy(data["num_tokens"][rows].copy()).to(dev)
    docs = data["docs"]
    out = []
    sums = []
    for op, arg in sc["ops"]:
        if op == "pwu":
            samp = torch.from_numpy(data["sampled"][arg][rows].copy()).to(dev)
            d, nv, n = drafter.propose_with_update(n, tok, samp)
            out.append((d.cpu().numpy(), nv.cpu().numpy(), n.cpu().numpy()))
        elif op == "harvest":
            mine = _split(arg, world, rank)
            drafter.harvest_rows(
                [torch.from_numpy(docs[j].copy()).to(dev) for j in mine],
                [int(docs[j].shape[0]) for j in mine])
        elif op == "poll":
            drafter.poll()
        gi = drafter.global_index
        sums.append((gi.active_len, gi.delta_len,
                     int(gi.corpus.to(torch.int64).sum().item()),
                     int((gi.sa.to(torch.int64) *
                          torch.arange(gi.sa.numel(), device=dev)).sum().item())))
    return out, sums


def _single_reference(sc):
    """One plain drafter: all rows; each harvest gets the documents in
    rank order (rank 0's share first)."""
    from suffixgpu_b200 import SuffixGPUDrafter
    sc2 = dict(sc)
    ops = []
    for op, arg in sc["ops"]:
        if op == "harvest":
            arg = _split(arg, 2, 0) + _split(arg, 2, 1)
        ops.append((op, arg))
    sc2["ops"] = ops
    b = sc["data"]["token_ids"].shape[0]
    d = SuffixGPUDrafter(device="cuda", **sc["drafter"])
    out, _ = _run(sc2, d, list(range(b)), 1, 0, torch.device("cuda"))
    return out


def test_replicated_world_one_matches_drafter():
    import torch.distributed as dist
    from suffixgpu_b200 import SuffixGPUDrafter
    from suffixgpu_b200.distributed import ReplicatedSuffixDrafter
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(_free_port())
    dist.init_process_group("nccl", rank=0, world_size=1)
    try:
        torch.cuda.set_device(0)
        sc = scenarios.global_scenario(43, steps=10)
        b = sc["data"]["token_ids"].shape[0]
        rows = list(range(b))
        dev = torch.device("cuda")
        got, _ = _run(sc, ReplicatedSuffixDrafter(device=dev, **sc["drafter"]),
                      rows, 1, 0, dev)
        exp, _ = _run(sc, SuffixGPUDrafter(device=dev, **sc["drafter"]),
                      rows, 1, 0, dev)
        for g, e in zip(got, exp):
            for a, x in zip(g, e):
                np.testing.assert_array_equal(a, x)
    finally:
        dist.destroy_process_group()


def _two_rank_worker(rank, port, sc, q):
    import torch.distributed as dist
    from suffixgpu_b200.distributed import ReplicatedSuffixDrafter
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=2)
    try:
        dev = torch.device("cuda", rank)
        b = sc["data"]["token_ids"].shape[0]
        rows = list(range(rank * b // 2, (rank + 1) * b // 2))
        d = ReplicatedSuffixDrafter(device=dev, **sc["drafter"])
        sync_out, _ = _run(sc, d, rows, 2, rank, dev)
        d2 = ReplicatedSuffixDrafter(device=dev,
                                  rebuild_stream=torch.cuda.Stream(dev),
                                  **sc["drafter"])
        _, sums = _run(sc, d2, rows, 2, rank, dev)
        q.put((rank, sync_out, sums))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_replicated_two_gpus_match_single_index():
    import torch.multiprocessing as mp
    sc = scenarios.global_scenario(44, steps=12)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_two_rank_worker, args=(r, port, sc, q))
             for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        r, out, sums = q.get(timeout=300)
        res[r] = (out, sums)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    exp = _single_reference(sc)
    b = sc["data"]["token_ids"].shape[0]
    for step, e in enumerate(exp):
        for r in range(2):
            sl = slice(r * b // 2, (r + 1) * b // 2)
            for a, x in zip(res[r][0][step], e):
                np.testing.assert_array_equal(a, x[sl], f"step {step}")
    # background rebuilds: the replicas agree after every operation
    assert res[0][1] == res[1][1]
