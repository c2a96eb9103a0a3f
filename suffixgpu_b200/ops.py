"""Tensor-level wrappers of the sm_100a kernels.

These mirror the reference's operator layer (suffix_gpu/triton_kernels.py
and the op functions in expand.py / sa_search.py / suffix_array.py) with the
same argument meaning, shapes and return dtypes. Every op runs on CUDA
tensors only and raises otherwise: there is no CPU path.
"""

from __future__ import annotations

import torch

from suffixgpu_b200 import _lib
from suffixgpu_b200._lib import call, ptr, stream_of


def require_cuda(*tensors: torch.Tensor) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("suffixgpu_b200 ops need CUDA tensors "
                             f"(got a tensor on {t.device})")
        dev = t.device if dev is None else dev
    if dev is None:
        raise ValueError("no tensor given")
    return dev


def as_i32(t: torch.Tensor) -> torch.Tensor:
    t = t if t.dtype == torch.int32 else t.to(torch.int32)
    return t.contiguous()


def as_i64(t: torch.Tensor) -> torch.Tensor:
    t = t if t.dtype == torch.int64 else t.to(torch.int64)
    return t.contiguous()


def scatter_append(token_ids: torch.Tensor, base: torch.Tensor,
                   cnt: torch.Tensor | None,
                   sampled: torch.Tensor) -> torch.Tensor:
    """Append each row's valid sampled ids at its base offset, in place
    (triton_kernels.py:392-402). Returns the new counts [B] int32."""
    dev = require_cuda(token_ids, base, sampled)
    if token_ids.dtype != torch.int32 or token_ids.dim() != 2 \
            or token_ids.stride(1) != 1:
        raise ValueError("token_ids must be an int32 [B, S] tensor with "
                         "unit column stride")
    b, s = token_ids.shape
    base = as_i32(base)
    sampled = as_i32(sampled)
    cnt32 = None if cnt is None else as_i32(cnt)
    new = torch.empty(b, dtype=torch.int32, device=dev)
    call("sg_scatter_append", ptr(token_ids), token_ids.stride(0), b, s,
         ptr(base), ptr(cnt32), ptr(sampled), sampled.shape[1], ptr(new),
         stream_of(dev))
    return new


def match_back(src: torch.Tensor, pat: torch.Tensor,
               n_out: int) -> torch.Tensor:
    """match_back[b, i] = longest L with src[.., i-L:i] == tail_L
    (triton_kernels.py:259-281). src is [B, S] or a shared [N] buffer."""
    dev = require_cuda(src, pat)
    src = as_i32(src)
    pat = as_i32(pat)
    b, p = pat.shape
    out = torch.empty(b, n_out, dtype=torch.int32, device=dev)
    stride = src.stride(0) if src.dim() == 2 else 0
    n_src = src.shape[-1]
    call("sg_match_back", ptr(src), stride, n_src, ptr(pat), b, p, n_out,
         ptr(out), stream_of(dev))
    return out


def first_occurrences(mb: torch.Tensor, thr: torch.Tensor, c: int,
                      r: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Earliest r positions with mb >= per-candidate threshold
    (triton_kernels.py:362-389). Returns (pos [B*C, r] i64, count i64)."""
    dev = require_cuda(mb, thr)
    mb = as_i32(mb)
    thr = as_i64(thr)
    bc = thr.shape[0]
    pos = torch.empty(bc, r, dtype=torch.int64, device=dev)
    cnt = torch.empty(bc, dtype=torch.int64, device=dev)
    call("sg_first_occurrences", ptr(mb), mb.shape[1], ptr(thr), bc, c, r,
         ptr(pos), ptr(cnt), stream_of(dev))
    return pos, cnt


def expand_chain(cont: torch.Tensor, num_occ: torch.Tensor, k: int,
                 sentinel: int = -1, min_token_prob: float = 0.0,
                 cap: torch.Tensor | None = None,
                 weights: torch.Tensor | None = None,
                 alpha: float = 0.0):
    """Majority-vote chain expansion with fused scoring
    (suffix_gpu/expand.py:59-147). Returns (chain [B, k] int32, num_valid
    [B] i64, num_emit [B] i64, score [B] f32)."""
    if sentinel != -1:
        raise ValueError("only sentinel=-1 is supported")
    if weights is not None:
        raise NotImplementedError("weighted votes are not supported")
    dev = require_cuda(cont, num_occ)
    b, r, kk = cont.shape
    if kk < k:
        raise ValueError("cont has fewer than k columns")
    cont = as_i32(cont)
    if kk != k:
        cont = cont[:, :, :k].contiguous()
    num_occ = as_i64(num_occ)
    capc = None if cap is None else as_i64(cap)
    chain = torch.empty(b, k, dtype=torch.int32, device=dev)
    nv = torch.empty(b, dtype=torch.int64, device=dev)
    emit = torch.empty(b, dtype=torch.int64, device=dev)
    score = torch.empty(b, dtype=torch.float32, device=dev)
    call("sg_expand_chain", ptr(cont), b, r, k, ptr(num_occ), ptr(capc),
         float(min_token_prob), float(alpha), ptr(chain), ptr(nv),
         ptr(emit), ptr(score), stream_of(dev))
    return chain, nv, emit, score
