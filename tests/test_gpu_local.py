"""GPU parity of the fused local draft kernel and the operator kernels
against the reference goldens and the numpy oracle. Bit-exact: drafts,
counts and token buffers are integers; scores are compared as fp32 bit
patterns."""

from __future__ import annotations

import os

import numpy as np
import pytest
import torch

import scenarios
from oracle import suffix_oracle as so

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def _host(t):
    return t.detach().cpu().numpy().copy()


def _gpu_drafter(**cfg):
    from suffixgpu_b200 import SuffixGPUDrafter
    return SuffixGPUDrafter(device=DEV, **cfg)


def _run_both(sc):
    got = scenarios.run_scenario(sc, _gpu_drafter, _dev, _host)
    exp = scenarios.run_scenario(sc, so.SuffixDrafter, lambda a: a.copy(),
                                 lambda a: np.asarray(a).copy())
    return got, exp


def _assert_same(got, exp, keys=("draft", "num_valid", "new_counts",
                                 "final_tokens")):
    for key in keys:
        np.testing.assert_array_equal(got[key], exp[key], err_msg=key)


@pytest.mark.parametrize("name", ["cfg1", "cfg2s", "tiny", "overflow"])
def test_local_scenarios_match_goldens(golden_dir, name):
    z = np.load(os.path.join(golden_dir, f"local_{name}.npz"))
    sc = scenarios.local_scenarios()[name]
    got = scenarios.run_scenario(sc, _gpu_drafter, _dev, _host)
    for key in ("draft", "num_valid", "new_counts", "final_tokens"):
        np.testing.assert_array_equal(got[key], z["out_" + key], key)


RANDOM_CFGS = [
    dict(k=4, max_pattern_len=6, max_occurrences=8, num_backoff=4),
    dict(k=8, max_pattern_len=16, max_occurrences=32, num_backoff=6,
         max_spec_factor=1.0, max_spec_offset=0.5, min_token_prob=0.15),
    dict(k=16, max_pattern_len=32, max_occurrences=128, num_backoff=8,
         max_spec_factor=2.0, min_token_prob=0.1),
    dict(k=5, max_pattern_len=9, max_occurrences=200, num_backoff=8,
         min_match_len=2, vote_smoothing_alpha=0.5),
    dict(k=12, max_pattern_len=20, max_occurrences=600, num_backoff=10,
         max_spec_factor=0.7, max_spec_offset=-0.25, min_token_prob=0.02),
    dict(k=64, max_pattern_len=255, max_occurrences=64, num_backoff=3),
]


@pytest.mark.parametrize("ci", range(len(RANDOM_CFGS)))
@pytest.mark.parametrize("shape", [(16, 97, 4), (8, 512, 6), (5, 2051, 3)])
def test_local_random_vs_oracle(ci, shape):
    b, s, vocab = shape
    sc = scenarios.local_scenario(
        100 + ci * 7 + s, b=b, s=s, steps=3, vocab=vocab, p_copy=0.6,
        span=(4, 40), q_range=(0, s), drafter=RANDOM_CFGS[ci])
    got, exp = _run_both(sc)
    _assert_same(got, exp)


def test_config2_full_size_vs_oracle():
    """B=256, S=8192 (benchmark config 2): two decode steps bit-exact."""
    from suffixgpu_b200 import workloads as wl
    data = wl.config2(seed=5, steps=2)
    sc = {"drafter": dict(wl.CONFIG2_DRAFTER), "data": data,
          "ops": [("pwu", 0), ("pwu", 1)]}
    got, exp = _run_both(sc)
    _assert_same(got, exp)
    assert (exp["num_valid"] > 0).mean() > 0.3


def test_config1_full_size_vs_oracle():
    from suffixgpu_b200 import workloads as wl
    data = wl.config1(seed=6)
    sc = {"drafter": dict(k=16, max_pattern_len=32, max_occurrences=128,
                          num_backoff=8),
          "data": data, "ops": [("pwu", 0)]}
    got, exp = _run_both(sc)
    _assert_same(got, exp)


def test_propose_mask_and_forward_outputs():
    """LocalMatchKernel.forward returns (draft, nv, match_len, occ, score)
    like local_matcher.py:198-242; masked rows draft nothing."""
    from suffixgpu_b200.local_matcher import LocalMatchKernel
    rng = np.random.default_rng(3)
    b, s = 24, 300
    tok = rng.integers(0, 5, size=(b, s)).astype(np.int32)
    q = rng.integers(0, s + 1, size=b).astype(np.int32)
    mask = rng.random(b) < 0.7
    kw = dict(k=6, max_pattern_len=10, max_occurrences=20, min_token_prob=0.1,
              max_spec_factor=1.5, support_thresholds=(1, 2, 4, 8, 16))
    exp = so.LocalMatcher(**kw).forward(q, tok, mask)
    got = LocalMatchKernel(**kw).forward(_dev(q), _dev(tok), _dev(mask))
    for g, e, name in zip(got, exp, ("draft", "nv", "len", "occ", "score")):
        g = _host(g)
        if name == "score":
            np.testing.assert_array_equal(g.view(np.int32),
                                          np.asarray(e, np.float32).view(
                                              np.int32))
        else:
            np.testing.assert_array_equal(g, np.asarray(e).astype(g.dtype),
                                          err_msg=name)
    assert (_host(got[1])[~mask] == 0).all()


def test_edge_rows():
    """q = 0, q = 1, q = S, q > S (propose mode clamps reads), buffers of
    -1 and negative ids, rows that are all one token."""
    from suffixgpu_b200 import SuffixGPUDrafter
    s = 37
    rows = [np.full(s, 7), np.full(s, -1), np.arange(s) % 3 - 2,
            np.arange(s) % 5, np.full(s, 2 ** 31 - 1), np.arange(s)]
    tok = np.stack(rows).astype(np.int32)
    b = tok.shape[0]
    for q in ([0] * b, [1] * b, [s] * b, [s + 5] * b, [3, 36, 37, 38, 2, 20]):
        q = np.array(q, dtype=np.int32)
        cfg = dict(k=6, max_pattern_len=8, max_occurrences=16, num_backoff=6)
        exp = so.SuffixDrafter(**cfg).propose(q, tok.copy())
        got = SuffixGPUDrafter(device=DEV, **cfg).propose(_dev(q), _dev(tok))
        np.testing.assert_array_equal(_host(got[0]), exp[0])
        np.testing.assert_array_equal(_host(got[1]), exp[1])


def test_update_semantics():
    """valid_count with -1 inside the counted range, counts past T, writes
    clipped at the buffer end, max_model_len."""
    from suffixgpu_b200 import SuffixGPUDrafter
    rng = np.random.default_rng(9)
    b, s, t = 10, 40, 4
    tok = rng.integers(0, 4, size=(b, s)).astype(np.int32)
    n = np.array([0, 5, 36, 38, 39, 40, 12, 20, 30, 1], dtype=np.int32)
    sampled = rng.integers(0, 4, size=(b, t)).astype(np.int32)
    sampled[1, 1] = -1
    sampled[6, :] = -1
    vc = np.array([1, 3, 4, 2, 1, 3, 0, 6, 2, 4], dtype=np.int32)
    cfg = dict(k=4, max_pattern_len=6, max_occurrences=8, num_backoff=4)
    for valid, mml in ((None, None), (vc, None), (vc, 33)):
        o = so.SuffixDrafter(**cfg)
        tok_o = tok.copy()
        exp = o.propose_with_update(n, tok_o, sampled, valid, mml)
        g = SuffixGPUDrafter(device=DEV, **cfg)
        tok_g = _dev(tok)
        got = g.propose_with_update(_dev(n), tok_g, _dev(sampled),
                                    None if valid is None else _dev(valid),
                                    mml)
        for x, y in zip(got, exp):
            np.testing.assert_array_equal(_host(x), y)
        np.testing.assert_array_equal(_host(tok_g), tok_o)
        # update_state alone
        tok_g2 = _dev(tok)
        tok_o2 = tok.copy()
        nc = g.update_state(_dev(n), tok_g2, _dev(sampled),
                            None if valid is None else _dev(valid))
        nce = o.update_state(n, tok_o2, sampled, valid)
        np.testing.assert_array_equal(_host(nc), nce)
        np.testing.assert_array_equal(_host(tok_g2), tok_o2)


def test_unaligned_row_stride():
    """Rows that are not 16-byte aligned take the plain-load path."""
    from suffixgpu_b200 import SuffixGPUDrafter
    rng = np.random.default_rng(4)
    b, s = 9, 203
    big = rng.integers(0, 4, size=(b, s + 3)).astype(np.int32)
    q = rng.integers(1, s, size=b).astype(np.int32)
    cfg = dict(k=5, max_pattern_len=7, max_occurrences=12, num_backoff=5)
    exp = so.SuffixDrafter(**cfg).propose(q, big[:, 1:s + 1].copy())
    gbig = _dev(big)
    view = gbig[:, 1:s + 1]
    assert view.stride(0) == s + 3
    got = SuffixGPUDrafter(device=DEV, **cfg).propose(_dev(q), view)
    np.testing.assert_array_equal(_host(got[0]), exp[0])
    np.testing.assert_array_equal(_host(got[1]), exp[1])


def test_expand_op_matches_goldens(golden_dir):
    from suffixgpu_b200 import ops
    z = np.load(os.path.join(golden_dir, "expand_cases.npz"))
    for i in range(int(z["n"])):
        p = f"c{i}_"
        r, k = z[p + "meta"].tolist()
        chain, nv, ne, sc = ops.expand_chain(
            _dev(z[p + "cont"]), _dev(z[p + "occ"]), int(k),
            min_token_prob=float(z[p + "minp"]), cap=_dev(z[p + "cap"]),
            alpha=float(z[p + "alpha"]))
        np.testing.assert_array_equal(_host(chain), z[p + "chain"])
        np.testing.assert_array_equal(_host(nv), z[p + "nv"])
        np.testing.assert_array_equal(_host(ne), z[p + "emit"])
        np.testing.assert_array_equal(_host(sc).view(np.int32),
                                      z[p + "score"].view(np.int32))


def test_match_back_and_first_occurrences_ops():
    from suffixgpu_b200 import ops
    rng = np.random.default_rng(12)
    b, s, p = 6, 2500, 9
    src = rng.integers(0, 3, size=(b, s)).astype(np.int32)
    pat = rng.integers(0, 3, size=(b, p)).astype(np.int32)
    exp = so.match_back(src, pat, s)
    got = ops.match_back(_dev(src), _dev(pat), s)
    np.testing.assert_array_equal(_host(got), exp)
    # shared buffer (the delta layout): n_out = N + 1
    shared = rng.integers(0, 3, size=3000).astype(np.int32)
    exp = so.match_back(shared, pat, 3001)
    got = ops.match_back(_dev(shared), _dev(pat), 3001)
    np.testing.assert_array_equal(_host(got), exp)
    # first occurrences with per-candidate thresholds
    c, r = 4, 50
    thr = rng.integers(-1, 5, size=b * c).astype(np.int64)
    pos, cnt = ops.first_occurrences(got, _dev(thr), c, r)
    mbv = exp[np.arange(b * c) // c]
    mask = (mbv >= thr[:, None]) & (thr[:, None] > 0)
    epos, ecnt = so.first_occurrences_masked(mask, r)
    np.testing.assert_array_equal(_host(pos), epos)
    np.testing.assert_array_equal(_host(cnt), ecnt)


def test_graph_capture_matches_eager():
    """propose_with_update captured in a CUDA graph replays the same
    results as eager calls (the serving loop's usage)."""
    from suffixgpu_b200 import SuffixGPUDrafter
    from suffixgpu_b200 import workloads as wl
    data = wl.config2(seed=8, steps=4, b=32, s=2048)
    d = SuffixGPUDrafter(device=DEV, **wl.CONFIG2_DRAFTER)
    # eager reference run
    tok_e = _dev(data["token_ids"])
    n_e = _dev(data["num_tokens"])
    eager = []
    for i in range(4):
        dr, nv, n_e = d.propose_with_update(n_e, tok_e,
                                            _dev(data["sampled"][i]))
        eager.append((_host(dr), _host(nv)))
    # graph run: static input buffers, counts fed back in place
    tok_g = _dev(data["token_ids"])
    n_g = _dev(data["num_tokens"])
    samp = _dev(data["sampled"][0])
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):  # warm-up on scratch copies
        d.propose_with_update(n_g.clone(), tok_g.clone(), samp)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        dr_g, nv_g, nc_g = d.propose_with_update(n_g, tok_g, samp)
        n_g.copy_(nc_g)
    for i in range(4):
        samp.copy_(_dev(data["sampled"][i]))
        g.replay()
        torch.cuda.synchronize()
        np.testing.assert_array_equal(_host(dr_g), eager[i][0])
        np.testing.assert_array_equal(_host(nv_g), eager[i][1])
    np.testing.assert_array_equal(_host(tok_g), _host(tok_e))
