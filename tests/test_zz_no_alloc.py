"""The allocation-free suffix-array entry point.

Callers such as a serving engine that has reserved all GPU memory for its
KV cache, or a plugin host that only hands a plugin its input and output
buffers, cannot call cudaMalloc. sg_build_suffix_array_noalloc serves them
from a scratch array compiled into the library. These tests call it through
the C ABI, twice in a row with different inputs (the second call reuses the
scratch the first one left behind), and require the same suffix arrays and
round counts as sg_build_suffix_array with a caller-allocated workspace.
Inputs and outputs are allocated by the test, as the caller would. The
largest accepted input is checked against the numpy oracle's suffix array
(suffix_gpu/suffix_array.py:15-63 restated), and the size limit is checked
at its exact boundary.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from suffixgpu_b200 import _lib as L
    return L.lib()


def _build_with_workspace(lib, tok: torch.Tensor) -> tuple[np.ndarray, int]:
    n = tok.numel()
    out = torch.empty(n, dtype=torch.int32, device=tok.device)
    ws = torch.empty(int(lib.sg_suffix_array_workspace_size(n)),
                     dtype=torch.uint8, device=tok.device)
    rounds = ctypes.c_int32(0)
    st = lib.sg_build_suffix_array(
        tok.data_ptr(), n, out.data_ptr(), ws.data_ptr(), ws.numel(),
        ctypes.byref(rounds), torch.cuda.current_stream().cuda_stream)
    assert st == 0, lib.sg_status_string(st)
    return out.cpu().numpy(), rounds.value


def _build_noalloc(lib, tok: torch.Tensor, out: torch.Tensor) -> int:
    rounds = ctypes.c_int32(0)
    st = lib.sg_build_suffix_array_noalloc(
        tok.data_ptr(), tok.numel(), out.data_ptr(), ctypes.byref(rounds),
        torch.cuda.current_stream().cuda_stream)
    assert st == 0, lib.sg_status_string(st)
    return rounds.value


def _tokens(seed: int, n: int, vocab: int) -> torch.Tensor:
    from suffixgpu_b200 import workloads as wl
    rng = np.random.default_rng(seed)
    z = wl.Zipf(1.1, vocab)
    t = wl.copy_stream(rng, n, z, 0.5, 8, 400, fresh_len=(8, 400))
    return torch.from_numpy(t).cuda()


def test_noalloc_matches_workspace_build_twice_in_a_row():
    lib = _lib()
    first = _tokens(1, 150_000, 5000)   # near the scratch limit
    second = _tokens(2, 3_001, 7)       # small, many deep repeats
    outs = []
    for tok in (first, second):
        out = torch.full((tok.numel(),), -7, dtype=torch.int32,
                         device=tok.device)
        rounds = _build_noalloc(lib, tok, out)
        torch.cuda.synchronize()
        outs.append((out.cpu().numpy(), rounds))
    for tok, (got, rounds) in zip((first, second), outs):
        exp, exp_rounds = _build_with_workspace(lib, tok)
        np.testing.assert_array_equal(got, exp)
        assert rounds == exp_rounds


def _max_tokens(lib) -> int:
    """Largest n whose build workspace fits the 8 MiB scratch array."""
    lo, hi = 0, 1 << 23
    while lo < hi:
        mid = (lo + hi + 1) // 2
        if lib.sg_suffix_array_workspace_size(mid) <= 8 << 20:
            lo = mid
        else:
            hi = mid - 1
    return lo


def test_noalloc_at_its_limit_matches_the_oracle():
    """The largest accepted n builds the oracle's suffix array; n + 1 is
    refused before any launch."""
    from oracle import suffix_oracle as so
    lib = _lib()
    n = _max_tokens(lib)
    assert 150_000 < n < 160_000
    tok = _tokens(3, n + 1, 3000)
    out = torch.full((n + 1,), -7, dtype=torch.int32, device=tok.device)
    rounds = ctypes.c_int32(0)
    st = lib.sg_build_suffix_array_noalloc(
        tok.data_ptr(), n + 1, out.data_ptr(), ctypes.byref(rounds),
        torch.cuda.current_stream().cuda_stream)
    assert st == 4  # SG_ERR_UNSUPPORTED
    torch.cuda.synchronize()
    assert (out == -7).all()  # nothing was launched
    _build_noalloc(lib, tok[:n], out[:n])
    torch.cuda.synchronize()
    exp = so.build_suffix_array(tok[:n].cpu().numpy())
    np.testing.assert_array_equal(out[:n].cpu().numpy(), exp)


def test_noalloc_rejects_inputs_beyond_its_scratch():
    lib = _lib()
    n = 1_000_000
    tok = torch.zeros(n, dtype=torch.int32, device="cuda")
    out = torch.empty(n, dtype=torch.int32, device="cuda")
    rounds = ctypes.c_int32(0)
    st = lib.sg_build_suffix_array_noalloc(
        tok.data_ptr(), n, out.data_ptr(), ctypes.byref(rounds),
        torch.cuda.current_stream().cuda_stream)
    assert st == 4  # SG_ERR_UNSUPPORTED: larger than the static scratch
    assert "limits" in lib.sg_status_string(st).decode()
