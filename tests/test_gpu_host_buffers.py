"""Host-buffer calls of the drafter on the GPU: sampled ids (and valid
counts) in page-locked host memory, draft / num_valid written into
caller-provided tensors on the host or the device. The results must equal
the device-tensor call bit for bit, and the oracle's, over a decode loop."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import suffix_oracle as so
from suffixgpu_b200 import SuffixGPUDrafter
from suffixgpu_b200 import workloads as wl

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
CFG = dict(k=16, max_pattern_len=32, max_occurrences=128, num_backoff=8,
           max_spec_factor=2.0, min_token_prob=0.1)


def _data(seed=11, b=64, s=2048, steps=6):
    return wl.local_config(seed, b=b, s=s, vocab=400, p_copy=0.7,
                           span=(16, 200), q_range=(0, s), steps=steps)


@pytest.mark.parametrize("with_count", [False, True])
def test_host_buffers_equal_device_call_and_oracle(with_count):
    data = _data()
    steps = data["sampled"].shape[0]
    b = data["token_ids"].shape[0]
    d_host = SuffixGPUDrafter(device=DEV, **CFG)
    d_dev = SuffixGPUDrafter(device=DEV, **CFG)
    ora = so.SuffixDrafter(**CFG)
    tok_h = torch.from_numpy(data["token_ids"]).to(DEV)
    tok_d = tok_h.clone()
    n_h = torch.from_numpy(data["num_tokens"]).to(DEV)
    n_d = n_h.clone()
    tok_o = data["token_ids"].copy()
    n_o = data["num_tokens"].copy()
    out_draft = torch.full((b, CFG["k"]), 7, dtype=torch.int32).pin_memory()
    out_nv = torch.full((b,), 7, dtype=torch.int32).pin_memory()
    for i in range(steps):
        s = data["sampled"][i]
        cnt = (s != -1).sum(1).astype(np.int32)
        samp_pin = torch.from_numpy(s).pin_memory()
        cnt_pin = torch.from_numpy(cnt).pin_memory() if with_count else None
        dh, nvh, n_h = d_host.propose_with_update(
            n_h, tok_h, samp_pin, cnt_pin, out=(out_draft, out_nv))
        assert dh.data_ptr() == out_draft.data_ptr()
        assert nvh.data_ptr() == out_nv.data_ptr()
        dd, nvd, n_d = d_dev.propose_with_update(
            n_d, tok_d, torch.from_numpy(s).to(DEV),
            torch.from_numpy(cnt).to(DEV) if with_count else None)
        do, nvo, n_o = ora.propose_with_update(n_o, tok_o, s,
                                               cnt if with_count else None)
        torch.cuda.synchronize(DEV)
        np.testing.assert_array_equal(out_draft.numpy(), dd.cpu().numpy())
        np.testing.assert_array_equal(out_nv.numpy(), nvd.cpu().numpy())
        np.testing.assert_array_equal(out_draft.numpy(), do)
        np.testing.assert_array_equal(out_nv.numpy(), nvo)
        np.testing.assert_array_equal(n_h.cpu().numpy(), n_o)
    np.testing.assert_array_equal(tok_h.cpu().numpy(), tok_o)
    np.testing.assert_array_equal(tok_h.cpu().numpy(), tok_d.cpu().numpy())


def test_device_out_tensors_and_propose():
    data = _data(seed=5, b=16, s=1024, steps=2)
    d = SuffixGPUDrafter(device=DEV, **CFG)
    tok = torch.from_numpy(data["token_ids"]).to(DEV)
    n = torch.from_numpy(data["num_tokens"]).to(DEV)
    ref_d, ref_nv = d.propose(n, tok)
    od = torch.empty_like(ref_d)
    onv = torch.empty_like(ref_nv)
    got_d, got_nv = d.propose(n, tok, out=(od, onv))
    assert got_d.data_ptr() == od.data_ptr()
    hd = torch.empty(ref_d.shape, dtype=torch.int32).pin_memory()
    hnv = torch.empty(ref_nv.shape, dtype=torch.int32).pin_memory()
    d.propose(n, tok, out=(hd, hnv))
    torch.cuda.synchronize(DEV)
    assert torch.equal(od, ref_d) and torch.equal(onv, ref_nv)
    assert torch.equal(hd, ref_d.cpu()) and torch.equal(hnv, ref_nv.cpu())


def test_pageable_or_misshaped_host_buffers_are_refused():
    data = _data(seed=3, b=8, s=512, steps=1)
    d = SuffixGPUDrafter(device=DEV, **CFG)
    tok = torch.from_numpy(data["token_ids"]).to(DEV)
    n = torch.from_numpy(data["num_tokens"]).to(DEV)
    before = tok.clone()
    pageable = torch.from_numpy(data["sampled"][0].copy())
    assert not pageable.is_pinned()
    with pytest.raises(RuntimeError, match="page-locked"):
        d.propose_with_update(n, tok, pageable)
    pinned = pageable.pin_memory()
    bad_out = (torch.empty(8, CFG["k"], dtype=torch.int32),  # pageable
               torch.empty(8, dtype=torch.int32).pin_memory())
    with pytest.raises(RuntimeError, match="page-locked"):
        d.propose_with_update(n, tok, pinned, out=bad_out)
    wrong_shape = (torch.empty(8, CFG["k"] + 1, dtype=torch.int32,
                               device=DEV),
                   torch.empty(8, dtype=torch.int32, device=DEV))
    with pytest.raises(RuntimeError, match=r"\[B, k\]"):
        d.propose_with_update(n, tok, pinned, out=wrong_shape)
    torch.cuda.synchronize(DEV)
    # refused calls launch nothing: the buffer is untouched
    assert torch.equal(tok, before)


def test_global_drafter_host_buffers_equal_device_call():
    """The global path copies host inputs to the device and its results
    into the caller's tensors; same drafts as device tensors."""
    rng = np.random.default_rng(2)
    cfg = dict(k=8, max_pattern_len=16, max_occurrences=32, num_backoff=5,
               enable_global=True, global_capacity=1 << 14,
               delta_capacity=1 << 10, max_spec_factor=2.0,
               min_token_prob=0.05)
    data = wl.local_config(9, b=8, s=512, vocab=60, p_copy=0.6,
                           span=(4, 32), q_range=(64, 480), steps=3)
    docs = [torch.from_numpy(rng.integers(0, 60, size=300).astype(np.int32))
            .to(DEV) for _ in range(6)]
    ds = []
    for _ in range(2):
        d = SuffixGPUDrafter(device=DEV, **cfg)
        d.harvest_rows(docs, [300] * 6)
        ds.append(d)
    tok = [torch.from_numpy(data["token_ids"]).to(DEV) for _ in range(2)]
    n = [torch.from_numpy(data["num_tokens"]).to(DEV) for _ in range(2)]
    hd = torch.empty(8, cfg["k"], dtype=torch.int32).pin_memory()
    hnv = torch.empty(8, dtype=torch.int32).pin_memory()
    for i in range(3):
        s = data["sampled"][i]
        _, _, n[0] = ds[0].propose_with_update(
            n[0], tok[0], torch.from_numpy(s).pin_memory(), out=(hd, hnv))
        dd, nvd, n[1] = ds[1].propose_with_update(
            n[1], tok[1], torch.from_numpy(s).to(DEV))
        torch.cuda.synchronize(DEV)
        assert torch.equal(hd, dd.cpu()) and torch.equal(hnv, nvd.cpu())
        assert torch.equal(n[0], n[1])


def test_rejected_settings_raise_instead_of_crashing():
    """Settings the kernel cannot run (draft length above 64; a row layout
    beyond shared memory) raise RuntimeError with the library's status."""
    tok = torch.zeros(4, 97, dtype=torch.int32, device=DEV)
    n = torch.full((4,), 50, dtype=torch.int32, device=DEV)
    samp = torch.ones(4, 3, dtype=torch.int32, device=DEV)
    with pytest.raises(RuntimeError, match="invalid argument"):
        SuffixGPUDrafter(device=DEV, k=65).propose_with_update(n, tok, samp)
    big = torch.zeros(4, 30000, dtype=torch.int32, device=DEV)
    d = SuffixGPUDrafter(device=DEV, k=12, max_pattern_len=20,
                         max_occurrences=1024, num_backoff=10)
    with pytest.raises(RuntimeError, match="beyond supported limits"):
        d.propose_with_update(n, big, samp)
    torch.cuda.synchronize(DEV)
