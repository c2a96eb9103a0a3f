"""Local (per-request) suffix matcher: the module-level API of the
reference's LocalMatchKernel (suffix_gpu/local_matcher.py:49-263), backed by
the fused sm_100a kernel ``sg_local_draft``."""

from __future__ import annotations

import ctypes
from collections.abc import Sequence

import torch

from suffixgpu_b200._lib import (DraftParams, LocalInputs, LocalOutputs,
                                 check, lib, stream_of)
from suffixgpu_b200.ops import as_i32, require_cuda


def _check_thresholds(support_thresholds: Sequence[int]) -> int:
    """The fused kernel derives thresholds as 2^0..2^(C-1), the set the
    drafter uses (proposer.py:75-78); return C."""
    th = tuple(int(t) for t in support_thresholds)
    if not th:
        raise ValueError("support_thresholds must be non-empty")
    if th != tuple(2 ** i for i in range(len(th))):
        raise ValueError("support_thresholds must be 1, 2, 4, ..., 2^(C-1)")
    return len(th)


class LocalMatchKernel:
    """Multi-length local suffix matcher with score-ranked expansion."""

    def __init__(self, k: int, max_pattern_len: int = 32,
                 min_match_len: int = 1, max_occurrences: int = 32,
                 min_token_prob: float = 0.0,
                 max_spec_factor: float | None = None,
                 max_spec_offset: float = 0.0,
                 support_thresholds: Sequence[int] = (1, 2, 4, 8),
                 vote_smoothing_alpha: float = 0.0):
        self.k = k
        self.max_pattern_len = max_pattern_len
        self.min_match_len = max(1, min_match_len)
        self.max_occurrences = max_occurrences
        self.min_token_prob = min_token_prob
        self.max_spec_factor = max_spec_factor
        self.max_spec_offset = max_spec_offset
        self.vote_smoothing_alpha = vote_smoothing_alpha
        self.support_thresholds = tuple(int(t) for t in support_thresholds)
        self.num_backoff = _check_thresholds(self.support_thresholds)
        self._pcache: dict = {}
        # per-call host work kept small: the argument structs are reused
        # (one host thread drives a drafter) and the entry point is bound
        # once
        self._ins = LocalInputs()
        self._outs = LocalOutputs()
        self._ins_ref = ctypes.byref(self._ins)
        self._outs_ref = ctypes.byref(self._outs)
        self._fn = None

    def to(self, device) -> "LocalMatchKernel":
        return self

    def params(self, b: int, s: int, stride: int) -> DraftParams:
        key = (b, s, stride)
        p = self._pcache.get(key)
        if p is None:
            p = DraftParams(
                batch=b, seq_len=s, row_stride=stride, k=self.k,
                max_pattern_len=self.max_pattern_len,
                max_occurrences=self.max_occurrences,
                num_backoff=self.num_backoff,
                min_match_len=self.min_match_len,
                has_spec_factor=int(self.max_spec_factor is not None),
                spec_factor=float(self.max_spec_factor or 0.0),
                spec_offset=float(self.max_spec_offset),
                min_token_prob=float(self.min_token_prob),
                vote_alpha=float(self.vote_smoothing_alpha))
            self._pcache[key] = p
        return p

    def run(self, num_tokens: torch.Tensor, token_ids: torch.Tensor,
            sampled: torch.Tensor | None = None,
            valid_count: torch.Tensor | None = None,
            mask: torch.Tensor | None = None, limit: int | None = None,
            extras: bool = False) -> dict:
        """One fused launch; returns a dict of newly allocated output
        tensors (the int32 ones are views of one allocation)."""
        if not (token_ids.is_cuda and num_tokens.is_cuda):
            require_cuda(num_tokens, token_ids)
        dev = token_ids.device
        if token_ids.dtype != torch.int32 or token_ids.dim() != 2 \
                or token_ids.stride(1) != 1:
            raise ValueError("token_ids must be an int32 [B, S] tensor with "
                             "unit column stride")
        b, s = token_ids.shape
        k = self.k
        n = num_tokens
        if n.dtype != torch.int32 or not n.is_contiguous():
            n = as_i32(n)
        ins, outs = self._ins, self._outs
        ins.num_tokens = n.data_ptr()
        ins.token_ids = token_ids.data_ptr()
        ins.limit = s if limit is None else int(limit)
        ins.sampled = None
        ins.sampled_cols = 0
        ins.valid_count = None
        ins.mask = None
        # one int32 allocation: draft [b, k], num_valid [b], new_counts [b]
        # (+ best_len, best_occ); their addresses follow from its base
        n_i32 = b * (k + 2 + (2 if extras else 0))
        buf = torch.empty(n_i32, dtype=torch.int32, device=dev)
        base = buf.data_ptr()
        out = {"draft": buf[:b * k].view(b, k),
               "num_valid": buf[b * k:b * (k + 1)]}
        outs.draft = base
        outs.num_valid = base + 4 * b * k
        outs.new_counts = None
        outs.best_score = None
        outs.best_len = None
        outs.best_occ = None
        outs.row_mask = None
        if sampled is not None:
            if sampled.dtype != torch.int32 or not sampled.is_contiguous():
                sampled = as_i32(sampled)
            ins.sampled = sampled.data_ptr()
            ins.sampled_cols = sampled.shape[1]
            if valid_count is not None:
                valid_count = as_i32(valid_count)
                ins.valid_count = valid_count.data_ptr()
            out["new_counts"] = buf[b * (k + 1):b * (k + 2)]
            outs.new_counts = base + 4 * b * (k + 1)
        elif mask is not None:
            mask = mask.to(torch.bool).contiguous()
            ins.mask = mask.data_ptr()
        if extras:
            out["best_len"] = buf[b * (k + 2):b * (k + 3)]
            out["best_occ"] = buf[b * (k + 3):b * (k + 4)]
            outs.best_len = base + 4 * b * (k + 2)
            outs.best_occ = base + 4 * b * (k + 3)
            out["best_score"] = torch.empty(b, dtype=torch.float32,
                                            device=dev)
            out["row_mask"] = torch.empty(b, dtype=torch.bool, device=dev)
            outs.best_score = out["best_score"].data_ptr()
            outs.row_mask = out["row_mask"].data_ptr()
        p = self.params(b, s, token_ids.stride(0))
        fn = self._fn
        if fn is None:
            fn = self._fn = lib().sg_local_draft
        st = fn(ctypes.byref(p), self._ins_ref, self._outs_ref,
                stream_of(dev))
        if st != 0:
            check("sg_local_draft", st)
        return out

    def forward(self, num_tokens_no_spec: torch.Tensor,
                token_ids: torch.Tensor, combined_mask: torch.Tensor):
        """local_matcher.py:198-242 -> (draft [B,K] int32, num_valid [B]
        int32, match_len [B] i64, occ_count [B] i64, score [B] f32)."""
        o = self.run(num_tokens_no_spec, token_ids, mask=combined_mask,
                     extras=True)
        return (o["draft"], o["num_valid"], o["best_len"].to(torch.int64),
                o["best_occ"].to(torch.int64), o["best_score"])

    __call__ = forward
