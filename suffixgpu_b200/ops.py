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


# ---------------------------------------------------------------------------
# suffix array (suffix_gpu/suffix_array.py, sa_search.py)
# ---------------------------------------------------------------------------
_ws_cache: dict = {}


def _workspace(device: torch.device, nbytes: int, tag: str) -> torch.Tensor:
    """Cached per-device scratch buffer of at least nbytes."""
    key = (device.index, tag)
    buf = _ws_cache.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=device)
        _ws_cache[key] = buf
    return buf


def build_suffix_array_into(tokens: torch.Tensor, out: torch.Tensor,
                            workspace: torch.Tensor | None = None,
                            stream: int | None = None) -> int:
    """Suffix array of the 1-D int32 tokens into the int32 `out` (same
    length). Returns the number of doubling rounds. Synchronises the
    stream it runs on (once per round)."""
    dev = require_cuda(tokens, out)
    tokens = as_i32(tokens.reshape(-1))
    n = tokens.numel()
    if out.dtype != torch.int32 or out.numel() < n or not out.is_contiguous():
        raise ValueError("out must be a contiguous int32 tensor of length n")
    L = _lib.lib()
    need = int(L.sg_suffix_array_workspace_size(n))
    if workspace is None or workspace.numel() < need:
        workspace = _workspace(dev, need, "sa")
    rounds = _lib.c_int32(0)
    call("sg_build_suffix_array", ptr(tokens), n, ptr(out), ptr(workspace),
         workspace.numel(), _lib.ctypes.byref(rounds),
         stream if stream is not None else stream_of(dev))
    return int(rounds.value)


def append_suffix_array_into(tokens: torch.Tensor, out: torch.Tensor,
                             prev_sa: torch.Tensor, prev_n: int,
                             evicted: int, kept: int, prev_rounds: int,
                             workspace: torch.Tensor | None = None,
                             stream: int | None = None) -> int:
    """Suffix array of the 1-D int32 tokens into `out` from the suffix
    array of the previous snapshot (sg_suffix_array_append): tokens[:kept]
    must equal the previous snapshot's tokens[evicted:evicted + kept],
    prev_sa[:prev_n] be its suffix array and prev_rounds the rounds its
    build reported. Returns the new snapshot's rounds bound. Synchronises
    the stream it runs on."""
    dev = require_cuda(tokens, out, prev_sa)
    tokens = as_i32(tokens.reshape(-1))
    n = tokens.numel()
    if out.dtype != torch.int32 or out.numel() < n or not out.is_contiguous():
        raise ValueError("out must be a contiguous int32 tensor of length n")
    if (prev_sa.dtype != torch.int32 or not prev_sa.is_contiguous()
            or prev_sa.numel() < prev_n):
        raise ValueError("prev_sa must be a contiguous int32 tensor holding "
                         "prev_n entries")
    L = _lib.lib()
    need = int(L.sg_suffix_array_append_workspace_size(n))
    if workspace is None or workspace.numel() < need:
        workspace = _workspace(dev, need, "sa_append")
    rounds = _lib.c_int32(0)
    call("sg_suffix_array_append", ptr(tokens), n, ptr(prev_sa), prev_n,
         evicted, kept, prev_rounds, ptr(out), ptr(workspace),
         workspace.numel(), _lib.ctypes.byref(rounds),
         stream if stream is not None else stream_of(dev))
    return int(rounds.value)


def build_suffix_array(tokens: torch.Tensor) -> torch.Tensor:
    """build_suffix_array (suffix_array.py:15-63): int64 start positions of
    the suffixes in lexicographic order."""
    dev = require_cuda(tokens)
    n = tokens.numel()
    out = torch.empty(n, dtype=torch.int32, device=dev)
    if n:
        build_suffix_array_into(tokens, out)
    return out.to(torch.int64)


def search_interval(sa: torch.Tensor, corpus: torch.Tensor,
                    pattern: torch.Tensor, pattern_len: torch.Tensor):
    """search_interval (sa_search.py:66-107): SA interval [start, end) of
    the suffixes starting with each pattern. Returns (start, end) int64."""
    dev = require_cuda(sa, corpus, pattern, pattern_len)
    sa = as_i32(sa)
    corpus = as_i32(corpus)
    pattern = as_i32(pattern)
    plen = as_i64(pattern_len)
    b, m = pattern.shape
    start = torch.empty(b, dtype=torch.int64, device=dev)
    end = torch.empty(b, dtype=torch.int64, device=dev)
    call("sg_sa_search", ptr(sa), ptr(corpus), sa.numel(), ptr(pattern), b,
         m, ptr(plen), ptr(start), ptr(end), stream_of(dev))
    return start, end


def suffix_match_backoff(sa, corpus, query, query_len, max_len: int, caps,
                         row_mask=None):
    """suffix_match_backoff (sa_search.py:110-163). Returns (match_len,
    start, end), each [B, C] int64."""
    dev = require_cuda(sa, corpus, query, query_len, caps)
    sa = as_i32(sa)
    corpus = as_i32(corpus)
    query = as_i32(query)
    qlen = as_i64(query_len)
    caps = as_i64(caps)
    b, q = query.shape
    c = caps.numel()
    out = [torch.empty(b, c, dtype=torch.int64, device=dev) for _ in range(3)]
    rm = None if row_mask is None else row_mask.to(torch.bool).contiguous()
    call("sg_suffix_match_backoff", ptr(sa), ptr(corpus), sa.numel(),
         ptr(query), b, q, ptr(qlen), max_len, ptr(caps), c, ptr(rm),
         ptr(out[0]), ptr(out[1]), ptr(out[2]), stream_of(dev))
    return out[0], out[1], out[2]


def longest_suffix_match(sa, corpus, query, query_len, max_len: int):
    """longest_suffix_match (sa_search.py:166-185)."""
    caps = torch.full((1,), max_len, dtype=torch.int64, device=sa.device)
    best, s, e = suffix_match_backoff(sa, corpus, query, query_len, max_len,
                                      caps)
    return best[:, 0], s[:, 0], e[:, 0]
