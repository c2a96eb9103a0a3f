"""Local (per-request) suffix matcher: the module-level API of the
reference's LocalMatchKernel (suffix_gpu/local_matcher.py:49-263), backed by
the fused sm_100a kernel ``sg_local_draft``."""

from __future__ import annotations

from collections.abc import Sequence

import torch

from suffixgpu_b200._lib import DraftParams, torch_ops
from suffixgpu_b200.ops import require_cuda


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
        self._op = None
        self._params_t: torch.Tensor | None = None

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
            extras: bool = False,
            out: tuple[torch.Tensor, torch.Tensor] | None = None) -> dict:
        """One fused launch (the torch operator over sg_local_draft);
        returns a dict of output tensors, newly allocated except the
        (draft, num_valid) pair given as ``out``. ``sampled`` /
        ``valid_count`` and ``out`` may be page-locked host tensors, which
        the kernel reads and writes in place (no separate copies)."""
        if not (token_ids.is_cuda and num_tokens.is_cuda):
            require_cuda(num_tokens, token_ids)
        op = self._op
        if op is None:
            op = self._op = torch_ops().local_draft
            # drafter settings as an sg_draft_params struct (the operator
            # fills in the batch shape)
            self._params_t = torch.frombuffer(
                bytearray(bytes(self.params(0, 1, 1))), dtype=torch.uint8)
        lim = token_ids.shape[1] if limit is None else int(limit)
        if out is None:
            res = op(num_tokens, token_ids, sampled, valid_count, mask,
                     self._params_t, lim, extras)
        else:
            res = op(num_tokens, token_ids, sampled, valid_count, mask,
                     self._params_t, lim, extras, out[0], out[1])
        out = {"draft": res[0], "num_valid": res[1]}
        if sampled is not None:
            out["new_counts"] = res[2]
        if extras:
            out["best_score"] = res[3]
            out["best_len"] = res[4]
            out["best_occ"] = res[5]
            out["row_mask"] = res[6]
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
