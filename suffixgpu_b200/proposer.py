"""SuffixGPUDrafter: the reference drafter API (suffix_gpu/proposer.py:26-393)
on the sm_100a kernels.

The local-only drafter is one fused kernel launch per propose /
propose_with_update call (``sg_local_draft``), with no host sync, so the
call can be captured into a CUDA graph. With ``enable_global=True`` the
global index (corpus suffix array + delta buffer) adds the SA search, the
delta scan and the global candidate expansion, combined with the local
winner by the reference's strict-greater rule.
"""

from __future__ import annotations

import torch

from suffixgpu_b200 import ops
from suffixgpu_b200.local_matcher import LocalMatchKernel


def global_caps(max_pattern_len: int, num_backoff: int) -> list[int]:
    """Descending global length caps (proposer.py:78-87)."""
    if num_backoff == 1:
        caps = [max_pattern_len]
    else:
        caps = [max(2, max_pattern_len >> i)
                for i in range(num_backoff - 1)] + [2]
    return sorted(set(caps), reverse=True)


class SuffixGPUDrafter:
    """Device-resident suffix-decoding drafter (device tensors in and out,
    no host synchronization on the propose path)."""

    def __init__(
        self,
        k: int,
        device: torch.device | str = "cuda",
        max_pattern_len: int = 32,
        min_match_len: int = 1,
        max_occurrences: int = 128,
        enable_global: bool = False,
        global_capacity: int = 1 << 22,
        delta_capacity: int = 1 << 16,
        rebuild_threshold: int | None = None,
        rebuild_stream: torch.cuda.Stream | None = None,
        max_spec_factor: float | None = None,
        max_spec_offset: float = 0.0,
        min_token_prob: float = 0.0,
        num_backoff: int = 8,
        vote_smoothing_alpha: float = 0.0,
        parallel_paths: bool = True,
    ):
        self.k = k
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("SuffixGPUDrafter (suffixgpu_b200) runs on CUDA "
                             f"devices only, got {self.device}")
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.max_pattern_len = max_pattern_len
        self.max_spec_factor = max_spec_factor
        self.max_spec_offset = max_spec_offset
        self.min_token_prob = min_token_prob
        self.num_backoff = max(1, int(num_backoff))
        self.vote_smoothing_alpha = float(vote_smoothing_alpha)
        self.parallel_paths = bool(parallel_paths)
        self._aux = None
        support_thresholds = tuple(2 ** i for i in range(self.num_backoff))
        caps = global_caps(max_pattern_len, self.num_backoff)
        self._global_caps = torch.tensor(caps, dtype=torch.int64,
                                         device=self.device)
        self.local_kernel = LocalMatchKernel(
            k=k, max_pattern_len=max_pattern_len,
            min_match_len=min_match_len, max_occurrences=max_occurrences,
            min_token_prob=min_token_prob, max_spec_factor=max_spec_factor,
            max_spec_offset=max_spec_offset,
            support_thresholds=support_thresholds,
            vote_smoothing_alpha=self.vote_smoothing_alpha)
        self.global_index = None
        self._ingested: dict = {}
        if enable_global:
            from suffixgpu_b200.global_index import GlobalIndex
            self.global_index = GlobalIndex(
                capacity=global_capacity, delta_capacity=delta_capacity,
                k=k, max_occurrences=max_occurrences,
                rebuild_threshold=rebuild_threshold, device=self.device,
                rebuild_stream=rebuild_stream)

    # ------------------------------------------------------------------
    def device_error(self, clear: bool = True,
                     raise_on_error: bool = False) -> int:
        """Bits of the device error word (SG_DEVERR_WAIT = 1: a row's load
        into the local kernel's shared memory did not land within the
        kernel's bounded wait, and that row drafted nothing); 0 when no
        kernel has failed. Clears the word by default. Synchronises the
        current stream, so call it off the decode loop's hot path (a
        periodic health check). No reference counterpart: the reference's
        kernels have no bounded waits."""
        from suffixgpu_b200._lib import check, lib, stream_of
        import ctypes
        bits = ctypes.c_uint32(0)
        check("sg_device_error", lib().sg_device_error(
            ctypes.byref(bits), int(clear), stream_of(self.device)))
        if bits.value and raise_on_error:
            raise RuntimeError(
                f"device error word {bits.value:#x}: a bounded wait of the "
                "local draft kernel ran out; the affected rows drafted "
                "nothing")
        return bits.value

    def poll(self) -> None:
        """Host-side: swap in a finished background rebuild, if any."""
        if self.global_index is not None:
            self.global_index.poll_rebuild()

    def update_state(self, num_tokens_no_spec: torch.Tensor,
                     token_ids_gpu: torch.Tensor,
                     sampled_token_ids: torch.Tensor,
                     valid_sampled_tokens_count: torch.Tensor | None = None
                     ) -> torch.Tensor:
        """Scatter the sampled ids into the resident buffer (in place) and
        return the updated counts [B] int32 (proposer.py:135-184)."""
        return ops.scatter_append(token_ids_gpu, num_tokens_no_spec,
                                  valid_sampled_tokens_count,
                                  sampled_token_ids)

    def propose_with_update(
        self,
        num_tokens_no_spec: torch.Tensor,
        token_ids_gpu: torch.Tensor,
        sampled_token_ids: torch.Tensor,
        valid_sampled_tokens_count: torch.Tensor | None = None,
        max_model_len: int | None = None,
        *,
        out: tuple[torch.Tensor, torch.Tensor] | None = None,
    ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """update_state + eligibility mask + propose, all on device
        (proposer.py:186-214). Returns (draft [B,k] int32, num_valid [B]
        int32, new_num_tokens [B] int32).

        Host buffers (no reference counterpart): ``sampled_token_ids`` and
        ``valid_sampled_tokens_count`` may be page-locked host tensors, and
        ``out=(draft, num_valid)`` names the tensors to fill, on the device
        or page-locked on the host. The local step reads and writes those
        host buffers from the kernel itself, so a host-driven loop makes
        one launch per step and no copies; read them only after the stream
        has passed the call (e.g. ``torch.cuda.current_stream()
        .synchronize()``). Host inputs must hold the CPU's writes: the
        kernel may read them before the previous kernel on the stream has
        finished, so they must not be the target of GPU work still in
        flight (a non-blocking device-to-host copy, say)."""
        s = token_ids_gpu.shape[1]
        limit = s if max_model_len is None else min(max_model_len, s)
        if self.global_index is None:
            o = self.local_kernel.run(
                num_tokens_no_spec, token_ids_gpu,
                sampled=sampled_token_ids,
                valid_count=valid_sampled_tokens_count, limit=limit,
                out=out)
            return o["draft"], o["num_valid"], o["new_counts"]
        # the global kernels read their inputs from device memory
        sampled_token_ids = self._on_device(sampled_token_ids)
        valid_sampled_tokens_count = self._on_device(
            valid_sampled_tokens_count)
        # the global searches fork off before the local step (they read the
        # rows' tails as the local step's scatter will leave them)
        streams = self._aux_streams()
        pend = self.global_index.start_global_step(
            self, num_tokens_no_spec, token_ids_gpu,
            sampled=sampled_token_ids,
            valid_count=valid_sampled_tokens_count, limit=limit,
            streams=streams)
        o = self.local_kernel.run(
            num_tokens_no_spec, token_ids_gpu, sampled=sampled_token_ids,
            valid_count=valid_sampled_tokens_count, limit=limit,
            extras=True)
        draft, nv = self.global_index.finish_global_step(pend, o, self,
                                                         streams)
        return (*self._into(out, draft, nv), o["new_counts"])

    def propose(self, num_tokens_no_spec: torch.Tensor,
                token_ids_gpu: torch.Tensor,
                combined_mask: torch.Tensor | None = None, *,
                out: tuple[torch.Tensor, torch.Tensor] | None = None
                ) -> tuple[torch.Tensor, torch.Tensor]:
        """Draft from local history (and the global index when enabled)
        (proposer.py:216-327). Returns (draft [B,k] int32, num_valid [B]
        int32); ``out`` as in propose_with_update."""
        if self.global_index is None:
            o = self.local_kernel.run(num_tokens_no_spec, token_ids_gpu,
                                      mask=combined_mask, out=out)
            return o["draft"], o["num_valid"]
        streams = self._aux_streams()
        pend = self.global_index.start_global_step(
            self, num_tokens_no_spec, token_ids_gpu, mask=combined_mask,
            streams=streams)
        o = self.local_kernel.run(num_tokens_no_spec, token_ids_gpu,
                                  mask=combined_mask, extras=True)
        return self._into(out, *self.global_index.finish_global_step(
            pend, o, self, streams))

    def _on_device(self, t: torch.Tensor | None) -> torch.Tensor | None:
        if t is None or t.is_cuda:
            return t
        return t.to(self.device, non_blocking=True)

    @staticmethod
    def _into(out, draft: torch.Tensor, nv: torch.Tensor):
        """Results into the caller's (draft, num_valid) tensors, if given
        (asynchronous copies on the current stream)."""
        if out is None:
            return draft, nv
        out[0].copy_(draft, non_blocking=True)
        out[1].copy_(nv, non_blocking=True)
        return out[0], out[1]

    def _aux_streams(self):
        """The two side streams of the global searches and the four events
        of their fork and join (the reference's parallel_paths, proposer.py:
        243-320), created on first use and reused; None runs everything on
        the current stream."""
        if not self.parallel_paths:
            return None
        if self._aux is None:
            s0 = torch.cuda.Stream(self.device)
            evs = tuple(torch.cuda.Event() for _ in range(4))
            if not torch.cuda.is_current_stream_capturing():
                # give the events their CUDA events now, so the global
                # step's operators can take their handles
                for e in evs:
                    e.record(s0)
            self._aux = (s0, torch.cuda.Stream(self.device), evs)
        return self._aux

    # ------------------------------------------------------------------
    # host-side ingestion (proposer.py:329-390)
    # ------------------------------------------------------------------
    def harvest_finished(self, row_indices: list[int], lengths: list[int],
                         token_ids_gpu: torch.Tensor) -> None:
        """Rows' first ``lengths`` tokens become documents of the global
        index (proposer.py:329-343)."""
        if self.global_index is None:
            return
        self._append_rows(token_ids_gpu, list(row_indices), list(lengths))

    def _append_rows(self, token_ids: torch.Tensor, rows: list[int],
                     lengths: list[int]) -> None:
        """harvest_finished's documents, written straight from the token
        buffer (one launch). The multi-GPU drafter exchanges them between
        ranks here."""
        self.global_index.append_rows(token_ids, rows, lengths)

    def harvest_rows(self, rows: list[torch.Tensor],
                     lengths: list[int]) -> None:
        if self.global_index is None:
            return
        docs = [row[:ln] for row, ln in zip(rows, lengths) if ln > 0]
        self._append_docs(docs)

    def _append_docs(self, docs: list[torch.Tensor]) -> None:
        """Documents into the global index; nothing happens for none
        (proposer.py:351-352, 384-385). The multi-GPU drafter exchanges
        them between ranks here."""
        if docs:
            self.global_index.append_documents(docs)

    def ingest_active(self, keys: list, rows: list[torch.Tensor],
                      lengths: list[int], final: bool = False,
                      chunk: int = 64) -> None:
        if self.global_index is None:
            return
        overlap = self.max_pattern_len + self.k
        docs = []
        for key, row, ln in zip(keys, rows, lengths):
            done = self._ingested.get(key, 0)
            if ln - done >= chunk or (final and ln > done):
                start = max(0, done - overlap)
                docs.append(row[start:ln])
                self._ingested[key] = ln
            if final:
                self._ingested.pop(key, None)
        self._append_docs(docs)

    def load_documents(self, docs: list[torch.Tensor]) -> None:
        """Bulk-load finished documents into the global index
        (GlobalIndex.load_documents; no reference counterpart)."""
        if self.global_index is None:
            raise ValueError("load_documents needs enable_global=True")
        self.global_index.load_documents(docs)

    def load_model(self, *args, **kwargs) -> None:
        pass
