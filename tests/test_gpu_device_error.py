"""Device-side failure reporting of the local draft kernel, without a GPU
fault: the test shortens the kernel's bounded wait for a row's bulk load
to zero polls (sg_set_wait_polls), so the wait runs out on purpose while
the copy itself still lands. Every row must then draft nothing (num_valid
0, drafts -1) while its update still happens, and the device error word
(sg_device_error) must report the timeout until it is cleared. With the
default bound restored, the next calls draft exactly like the oracle and
set no error."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import suffix_oracle as so

pytestmark = pytest.mark.gpu

DEV = "cuda"
SG_DEVERR_WAIT = 1


def _error_word(lib, clear: bool) -> int:
    bits = ctypes.c_uint32(0xFFFFFFFF)
    st = lib.sg_device_error(ctypes.byref(bits), int(clear),
                             torch.cuda.current_stream().cuda_stream)
    assert st == 0
    return bits.value


def test_wait_timeout_reports_error_and_drafts_nothing():
    from suffixgpu_b200 import SuffixGPUDrafter, _lib
    from suffixgpu_b200 import workloads as wl
    lib = _lib.lib()
    data = wl.config2(seed=61, steps=2, b=16, s=8192)
    cfg = dict(wl.CONFIG2_DRAFTER)
    g = SuffixGPUDrafter(device=DEV, **cfg)
    o = so.SuffixDrafter(**cfg)
    tok = torch.from_numpy(data["token_ids"]).to(DEV)
    n = torch.from_numpy(data["num_tokens"]).to(DEV)
    tok_o, n_o = data["token_ids"].copy(), data["num_tokens"].copy()
    torch.cuda.synchronize()
    _error_word(lib, clear=True)
    assert _error_word(lib, clear=False) == 0
    prev = lib.sg_set_wait_polls(0)
    try:
        s0 = torch.from_numpy(data["sampled"][0]).to(DEV)
        draft, nv, n = g.propose_with_update(n, tok, s0)
        torch.cuda.synchronize()
    finally:
        lib.sg_set_wait_polls(-1)
    assert prev == 1 << 22
    assert _error_word(lib, clear=False) & SG_DEVERR_WAIT
    assert (nv.cpu().numpy() == 0).all()
    assert (draft.cpu().numpy() == -1).all()
    # the update happened regardless
    _, _, n_o = o.propose_with_update(n_o, tok_o, data["sampled"][0])
    np.testing.assert_array_equal(n.cpu().numpy(), n_o)
    np.testing.assert_array_equal(tok.cpu().numpy(), tok_o)
    # the word stays set until cleared; clearing returns the bits once
    assert _error_word(lib, clear=True) & SG_DEVERR_WAIT
    assert _error_word(lib, clear=False) == 0
    # default bound: exact drafts again, no error
    s1 = torch.from_numpy(data["sampled"][1]).to(DEV)
    draft, nv, n = g.propose_with_update(n, tok, s1)
    do, nvo, n_o = o.propose_with_update(n_o, tok_o, data["sampled"][1])
    np.testing.assert_array_equal(draft.cpu().numpy(), do)
    np.testing.assert_array_equal(nv.cpu().numpy(), nvo)
    assert (nvo > 0).any()
    assert _error_word(lib, clear=False) == 0
    assert g.device_error() == 0


def test_drafter_device_error_raises_on_request():
    """SuffixGPUDrafter.device_error(raise_on_error=True) turns a set word
    into an exception (and clears it)."""
    from suffixgpu_b200 import SuffixGPUDrafter, _lib
    from suffixgpu_b200 import workloads as wl
    lib = _lib.lib()
    data = wl.config1(seed=62)
    g = SuffixGPUDrafter(device=DEV, k=16, max_pattern_len=32,
                         max_occurrences=128, num_backoff=8)
    tok = torch.from_numpy(data["token_ids"]).to(DEV)
    n = torch.from_numpy(data["num_tokens"]).to(DEV)
    lib.sg_set_wait_polls(0)
    try:
        g.propose(n, tok)
    finally:
        lib.sg_set_wait_polls(-1)
    with pytest.raises(RuntimeError, match="bounded wait"):
        g.device_error(raise_on_error=True)
    assert g.device_error() == 0
