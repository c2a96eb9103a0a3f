"""vLLM glue: SuffixGPUDrafter behind vLLM's GPU n-gram proposer contract.

The reference drafter "mirrors the vLLM ngram_gpu proposer contract —
device tensors in, device tensors out, no per-step host synchronization"
(README.md:5-10) but ships no adapter. This module is that adapter for the
vLLM V1 GPU model runner (vllm/v1/worker/gpu_model_runner.py), whose
``ngram_gpu`` branch calls, every decode step,

    next_ids, counts, sampled = drafter.update_token_ids_ngram(...)
    draft, num_valid = drafter.propose(num_tokens_no_spec[:B],
                                       token_ids_gpu[:B], sampled, counts)

and checks ``isinstance(drafter, NgramProposerGPU)``.

* ``SuffixGPUProposer`` subclasses vLLM's ``NgramProposerGPU``; its
  ``update_token_ids_ngram`` computes vLLM's result in one launch
  (``sg_vllm_prepare``; vLLM's own code for inputs that one does not
  cover), and its ``propose`` runs
  ``SuffixGPUDrafter.propose_with_update`` (proposer.py:186-214): scatter
  of the sampled ids, local and global matching, expansion and selection,
  all on the device, after a non-blocking ``poll`` for a finished
  background rebuild.
* ``drafter_kwargs`` maps vLLM's speculative config onto the drafter:
  ``num_speculative_tokens`` -> k, ``prompt_lookup_max`` /
  ``prompt_lookup_min`` -> max_pattern_len / min_match_len,
  ``suffix_decoding_max_spec_factor`` / ``suffix_decoding_min_token_prob``
  -> max_spec_factor / min_token_prob; the global index is on unless
  ``suffix_decoding_max_cached_requests`` is 0. Keyword overrides win.
* ``install(runner)`` puts the proposer on a model runner (configured with
  ``method="ngram_gpu"``) and wraps ``runner._update_states`` so that
  finished requests are harvested into the global index (prompt and
  output, the row's first ``num_tokens_no_spec`` tokens as the host sees
  them) before their rows are freed.
* ``SuffixGPUWorkerExtension`` is a ``worker_extension_cls`` mixin: with
  ``LLM(..., worker_extension_cls="suffixgpu_b200.vllm_adapter.SuffixGPUWorkerExtension")``
  every worker installs the proposer through
  ``llm.collective_rpc("install_suffixgpu_drafter")``.

Importing this module imports vLLM (needed for the base class).
"""

from __future__ import annotations

import torch

from vllm.v1.spec_decode.ngram_proposer_gpu import NgramProposerGPU

from suffixgpu_b200._lib import torch_ops
from suffixgpu_b200.proposer import SuffixGPUDrafter

_DEFAULTS = dict(max_pattern_len=32, min_match_len=1, max_occurrences=128,
                 global_capacity=1 << 22, delta_capacity=1 << 16,
                 num_backoff=8)


def drafter_kwargs(vllm_config, **overrides) -> dict:
    """SuffixGPUDrafter constructor arguments (without device) from a vLLM
    config (speculative_config / model_config attributes are read by name,
    so any object with those attributes works)."""
    spec = vllm_config.speculative_config
    kw = dict(_DEFAULTS)
    kw["k"] = int(spec.num_speculative_tokens)
    if getattr(spec, "prompt_lookup_max", None):
        kw["max_pattern_len"] = int(spec.prompt_lookup_max)
    if getattr(spec, "prompt_lookup_min", None):
        kw["min_match_len"] = int(spec.prompt_lookup_min)
    factor = getattr(spec, "suffix_decoding_max_spec_factor", None)
    kw["max_spec_factor"] = None if factor is None else float(factor)
    kw["min_token_prob"] = float(
        getattr(spec, "suffix_decoding_min_token_prob", 0.0) or 0.0)
    cached = getattr(spec, "suffix_decoding_max_cached_requests", 1)
    kw["enable_global"] = cached is None or int(cached) != 0
    kw.update(overrides)
    return kw


class SuffixGPUProposer(NgramProposerGPU):
    """vLLM ngram_gpu proposer backed by SuffixGPUDrafter (see module
    docstring). Constructor: (vllm_config, device, runner=None, **drafter
    overrides)."""

    def __init__(self, vllm_config, device: torch.device, runner=None,
                 **overrides):
        # NgramProposerGPU.__init__ compiles vLLM's own n-gram kernel; only
        # the attributes its update_token_ids_ngram reads are set here.
        self.vllm_config = vllm_config
        self.device = torch.device(device)
        self.runner = runner
        kw = drafter_kwargs(vllm_config, **overrides)
        self.k = kw["k"]
        self.max_model_len = int(vllm_config.model_config.max_model_len)
        if kw.get("enable_global") and "rebuild_stream" not in kw:
            kw["rebuild_stream"] = torch.cuda.Stream(self.device)
        self.drafter = SuffixGPUDrafter(device=self.device, **kw)

    def update_token_ids_ngram(self, sampled_token_ids, gpu_input_batch,
                               token_ids_gpu: torch.Tensor,
                               num_tokens_no_spec: torch.Tensor,
                               discard_request_mask: torch.Tensor):
        """NgramProposerGPU.update_token_ids_ngram's result (next token ids,
        valid sampled counts, sampled ids with discarded rows set to -1)
        from one launch (sg_vllm_prepare) instead of vLLM's chain of torch
        ops, for int32 sampled ids with one row per request; other inputs
        (the ragged list form, other dtypes) go to vLLM's own code."""
        b = gpu_input_batch.num_reqs
        if (isinstance(sampled_token_ids, torch.Tensor)
                and sampled_token_ids.is_cuda
                and sampled_token_ids.dtype == torch.int32
                and sampled_token_ids.dim() == 2
                and sampled_token_ids.shape[0] == b
                and token_ids_gpu.dtype == torch.int32):
            nxt, cnt, valid = torch_ops().vllm_prepare(
                sampled_token_ids, discard_request_mask[:b],
                token_ids_gpu[:b], num_tokens_no_spec[:b],
                int(gpu_input_batch.vocab_size))
            return nxt, cnt, valid
        return super().update_token_ids_ngram(
            sampled_token_ids, gpu_input_batch, token_ids_gpu,
            num_tokens_no_spec, discard_request_mask)

    def propose(self, num_tokens_no_spec: torch.Tensor,
                token_ids_gpu: torch.Tensor,
                valid_sampled_token_ids_gpu: torch.Tensor,
                valid_sampled_tokens_count: torch.Tensor
                ) -> tuple[torch.Tensor, torch.Tensor]:
        """NgramProposerGPU.propose's contract: scatters the sampled ids
        into token_ids_gpu (in place) and returns (draft [B, k] int32 with
        -1 past num_valid, num_valid [B] int32). No host sync."""
        self.drafter.poll()
        draft, num_valid, _ = self.drafter.propose_with_update(
            num_tokens_no_spec, token_ids_gpu, valid_sampled_token_ids_gpu,
            valid_sampled_tokens_count, max_model_len=self.max_model_len)
        return draft, num_valid

    def harvest_finished_requests(self, runner, req_ids) -> None:
        """Harvest the rows of finished requests still in the runner's
        persistent batch into the global index (host-side lengths, no
        sync)."""
        if self.drafter.global_index is None or not req_ids:
            return
        batch = runner.input_batch
        rows, lengths = [], []
        for rid in req_ids:
            idx = batch.req_id_to_index.get(rid)
            if idx is None:
                continue
            rows.append(int(idx))
            lengths.append(int(batch.num_tokens_no_spec[idx]))
        if rows:
            self.drafter.harvest_finished(rows, lengths,
                                          runner.token_ids_gpu_tensor)

    def load_model(self, *args, **kwargs) -> None:
        pass


def install(runner, **overrides) -> SuffixGPUProposer:
    """Replace ``runner.drafter`` (a model runner built with
    ``method="ngram_gpu"``) by a SuffixGPUProposer and harvest finished
    requests from ``runner._update_states``. Returns the proposer."""
    prop = SuffixGPUProposer(runner.vllm_config, runner.device, runner,
                             **overrides)
    runner.drafter = prop
    update = runner._update_states

    def _update_states(scheduler_output, *args, **kwargs):
        prop.harvest_finished_requests(
            runner, getattr(scheduler_output, "finished_req_ids", ()))
        return update(scheduler_output, *args, **kwargs)

    runner._update_states = _update_states
    return prop


class SuffixGPUWorkerExtension:
    """``worker_extension_cls`` mixin for vLLM workers."""

    def install_suffixgpu_drafter(self, **overrides) -> bool:
        install(self.model_runner, **overrides)
        return True


__all__ = ["SuffixGPUProposer", "SuffixGPUWorkerExtension", "drafter_kwargs",
           "install"]
