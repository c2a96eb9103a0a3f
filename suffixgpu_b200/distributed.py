"""Multi-GPU drafter for BASELINE config 5 (8-GPU sharded global drafter).

The reference has no multi-GPU code; this layer defines it on top of
SuffixGPUDrafter, one process per GPU under torch.distributed:

* request rows are data-parallel: every rank drafts its own rows with the
  local kernels, and the propose path has no collective;
* the global index is replicated: every rank holds the same corpus, suffix
  array and delta. Documents harvested on any rank are all-gathered (rank
  order, each rank's in its own order) and appended on every rank, and a
  background rebuild swaps in only when every rank's has finished (a MIN
  all-reduce at poll time), so the replicas stay identical.

The drafts of a rank's rows are therefore those of one SuffixGPUDrafter
whose harvest calls receive the concatenation of all ranks' documents in
rank order: the single-index semantics of the reference, bit for bit. The
collectives are on ingestion only: harvest_rows / harvest_finished /
ingest_active / load_documents / poll are collective calls (every rank
calls them, possibly with nothing to add).

Works with the NCCL backend (CUDA tensors) and with gloo (host tensors).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from suffixgpu_b200.proposer import SuffixGPUDrafter


def _comm_device(group) -> torch.device:
    backend = dist.get_backend(group)
    if backend == "nccl":
        return torch.device("cuda", torch.cuda.current_device())
    return torch.device("cpu")


def exchange_documents(docs: list[torch.Tensor], group=None
                       ) -> list[torch.Tensor]:
    """All ranks' documents in rank order (each rank's in its own order),
    as int32 tensors on the communication device: three all-gathers
    (counts, lengths, tokens padded to the largest rank's total)."""
    world = dist.get_world_size(group)
    dev = _comm_device(group)
    docs = [d.reshape(-1).to(device=dev, dtype=torch.int32) for d in docs]
    if world == 1:
        return docs
    n = torch.tensor([len(docs)], dtype=torch.int64, device=dev)
    counts = [torch.zeros_like(n) for _ in range(world)]
    dist.all_gather(counts, n, group=group)
    counts = [int(c.item()) for c in counts]
    max_n = max(counts)
    if max_n == 0:
        return []
    lens = torch.zeros(max_n, dtype=torch.int64, device=dev)
    if docs:
        lens[:len(docs)] = torch.tensor([d.numel() for d in docs],
                                        dtype=torch.int64)
    all_lens = [torch.zeros_like(lens) for _ in range(world)]
    dist.all_gather(all_lens, lens, group=group)
    all_lens = [ln.tolist() for ln in all_lens]
    totals = [sum(ln[:c]) for ln, c in zip(all_lens, counts)]
    max_total = max(max(totals), 1)
    flat = torch.zeros(max_total, dtype=torch.int32, device=dev)
    if docs and totals[dist.get_rank(group)] > 0:
        flat[:totals[dist.get_rank(group)]] = torch.cat(docs)
    all_flat = [torch.zeros_like(flat) for _ in range(world)]
    dist.all_gather(all_flat, flat, group=group)
    out = []
    for r in range(world):
        pos = 0
        for ln in all_lens[r][:counts[r]]:
            out.append(all_flat[r][pos:pos + ln])
            pos += ln
    return out


def agree_all(flag: bool, group=None) -> bool:
    """True on every rank iff it is true on every rank (MIN all-reduce)."""
    if dist.get_world_size(group) == 1:
        return flag
    t = torch.tensor([1 if flag else 0], dtype=torch.int32,
                     device=_comm_device(group))
    dist.all_reduce(t, op=dist.ReduceOp.MIN, group=group)
    return bool(t.item())


class ShardedSuffixDrafter(SuffixGPUDrafter):
    """SuffixGPUDrafter for one rank of a multi-GPU job: same constructor
    arguments plus ``group`` (default: the world). ``propose``,
    ``update_state`` and ``propose_with_update`` act on this rank's rows
    only and issue no collective; the ingestion calls are collective."""

    def __init__(self, *args, group=None, **kwargs):
        if not dist.is_initialized():
            raise RuntimeError("ShardedSuffixDrafter needs an initialised "
                               "torch.distributed process group")
        super().__init__(*args, **kwargs)
        self.group = group
        self.rank = dist.get_rank(group)
        self.world_size = dist.get_world_size(group)
        if self.global_index is not None and self.world_size > 1:
            self.global_index.rebuild_agree = (
                lambda done: agree_all(done, self.group))

    def _append_docs(self, docs: list[torch.Tensor]) -> None:
        all_docs = exchange_documents(docs, self.group)
        if all_docs:
            self.global_index.append_documents(all_docs)

    def _append_rows(self, token_ids: torch.Tensor, rows: list[int],
                     lengths: list[int]) -> None:
        self._append_docs([token_ids[r, :ln]
                           for r, ln in zip(rows, lengths) if ln > 0])

    def load_documents(self, docs: list[torch.Tensor]) -> None:
        """Bulk-load documents that every rank holds (the same list on
        every rank, e.g. generated from a shared seed): no exchange."""
        super().load_documents(docs)


__all__ = ["ShardedSuffixDrafter", "exchange_documents", "agree_all"]
