"""GPU parity at the settings of the benchmark configurations, bit-exact
against the numpy oracle:

* config 5's drafter (k = 32, P = 64, R = 256, six global caps 64..2), with
  its 2^20-token template corpus and harvests between decode steps, which
  runs the fused global step's 256-occurrence variant; and a drafter with
  more than 256 occurrences (the widest variant);
* config 3 at full size: capacity 2^22, delta 2^16, threshold 32768,
  B = 64, S = 4096, four harvests and a poll per step, synchronous
  rebuilds with eviction (drafts, corpus and suffix array compared);
* all 100 decode steps of config 2 on a 32-row slice (rows that run past
  the buffer end included).

The reference behaviour followed by the oracle: suffix_gpu/proposer.py:
186-327 (propose, selection), global_index.py:86-253 (harvest, rebuild,
eviction) and :286-370 (strided suffix-array sample), expand.py:59-147.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import suffix_oracle as so
from suffixgpu_b200 import workloads as wl

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def _host(t):
    return t.detach().cpu().numpy().copy()


class _Side:
    """Drives the GPU drafter or the oracle drafter through one script."""

    def __init__(self, drafter, gpu: bool):
        self.d = drafter
        self.gpu = gpu

    def arr(self, a):
        return _dev(a) if self.gpu else np.array(a, copy=True)

    def host(self, x):
        return _host(x) if self.gpu else np.asarray(x).copy()


def _run_loop(side: _Side, data: dict, steps: int, harvest_per_step: int,
              prefill=None, check_every=None, graph: bool = False):
    """Optional bulk prefill of the global index, then per step: harvest
    ``harvest_per_step`` rows of the batch at their current counts, poll,
    propose_with_update. Returns the per-step outputs and the final state.

    ``graph`` (GPU side): step 0 runs eagerly on a capture stream (it
    creates the side streams and buffers), then propose_with_update is
    captured once into a CUDA graph over static count and sampled-id
    buffers (the graph writes the new counts back into its count buffer)
    and every later step replays it."""
    d = side.d
    if prefill is not None:
        d.global_index.load_documents([side.arr(x) for x in prefill])
    tok = side.arr(data["token_ids"])
    n = side.arr(data["num_tokens"])
    b = data["token_ids"].shape[0]
    out = {"draft": [], "num_valid": [], "new_counts": [], "active_len": [],
           "delta_len": []}
    cap = cg = None
    for j in range(steps):
        if harvest_per_step:
            rows = [(harvest_per_step * j + i) % b
                    for i in range(harvest_per_step)]
            cnt = side.host(n)
            d.harvest_finished(rows, [int(cnt[r]) for r in rows], tok)
            d.poll()
        if graph and j == 0:
            cap = torch.cuda.Stream()
            cap.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(cap):
                draft, nv, n = d.propose_with_update(
                    n, tok, side.arr(data["sampled"][j]))
            torch.cuda.synchronize()
            n = n.clone()  # the static count buffer
            samp_s = side.arr(data["sampled"][min(1, steps - 1)])
            cg = torch.cuda.CUDAGraph()
            with torch.cuda.graph(cg, stream=cap):
                g_draft, g_nv, g_n = d.propose_with_update(n, tok, samp_s)
                n.copy_(g_n)
        elif graph:
            samp_s.copy_(side.arr(data["sampled"][j]))
            cg.replay()
            draft, nv = g_draft, g_nv
        else:
            draft, nv, n = d.propose_with_update(n, tok,
                                                 side.arr(data["sampled"][j]))
        out["draft"].append(side.host(draft))
        out["num_valid"].append(side.host(nv))
        out["new_counts"].append(side.host(n))
        gi = d.global_index
        if gi is not None:
            out["active_len"].append(gi.active_len)
            out["delta_len"].append(gi.delta_len)
    res = {k: np.stack(v) if v and isinstance(v[0], np.ndarray)
           else np.array(v) for k, v in out.items()}
    res["final_tokens"] = side.host(tok)
    del cg
    gi = d.global_index
    if gi is not None:
        res["corpus"] = side.host(gi.corpus)
        res["sa"] = side.host(gi.sa)
        res["delta"] = side.host(gi.delta)[:gi.delta_len]
        res["rebuilds"] = gi.rebuilds
    return res


def _both(cfg: dict, data: dict, steps: int, harvest_per_step: int,
          prefill=None):
    from suffixgpu_b200 import SuffixGPUDrafter
    g = _run_loop(_Side(SuffixGPUDrafter(device=DEV, **cfg), True), data,
                  steps, harvest_per_step, prefill)
    ocfg = {k: v for k, v in cfg.items() if k != "rebuild_stream"}
    o = _run_loop(_Side(so.SuffixDrafter(**ocfg), False), data, steps,
                  harvest_per_step, prefill)
    return g, o


def _assert_same(g, o, keys):
    for key in keys:
        np.testing.assert_array_equal(g[key], o[key], err_msg=key)


_LOOP_KEYS = ("draft", "num_valid", "new_counts", "final_tokens")
_INDEX_KEYS = ("active_len", "delta_len", "corpus", "sa", "delta")


def test_config5_settings_vs_oracle():
    """Config 5's drafter on 16 rows of S = 16384 over a 2^20-token corpus
    of 512 x 512 templates (workloads.config5's generator), 5 decode steps
    with 2 harvested rows each (delta matches and one rebuild)."""
    data = wl.config5(seed=55, rows=16, s=16384, n_docs=1024, doc_len=1023,
                      steps=5)
    cfg = dict(wl.CONFIG5_DRAFTER)
    cfg["global_capacity"] = 1 << 21
    assert (cfg["k"], cfg["max_pattern_len"], cfg["max_occurrences"]) \
        == (32, 64, 256)
    assert so.global_caps(64, 8) == [64, 32, 16, 8, 4, 2]
    g, o = _both(cfg, data, steps=5, harvest_per_step=2,
                 prefill=list(data["corpus_docs"]))
    _assert_same(g, o, _LOOP_KEYS + _INDEX_KEYS)
    assert g["rebuilds"] >= 2
    # the global candidates decided some drafts: at least one row drafts
    # more tokens than its local history alone gives
    loc = _run_loop(_Side(so.SuffixDrafter(**{
        **{k: v for k, v in cfg.items()}, "enable_global": False}), False),
        data, 5, 0)
    assert (o["num_valid"] != loc["num_valid"]).any()
    assert (o["num_valid"] > 0).mean() > 0.3


def test_more_than_256_occurrences_vs_oracle():
    """max_occurrences = 300: the fused global step's widest variant
    (32 occurrence slots per lane) and the local kernel at R > 256, on a
    corpus so repetitive that intervals exceed R (strided samples)."""
    rng = np.random.default_rng(56)
    z = wl.Zipf(1.1, 40)
    templates = z.draw(rng, (6, 24))
    docs = wl.template_docs(rng, 160, 200, templates, z, p_sub=0.02)
    b, s, steps = 12, 2048, 4
    rows = wl.template_docs(rng, b, s, templates, z, p_sub=0.02)
    data = {"token_ids": rows,
            "num_tokens": rng.integers(800, 2000, size=b).astype(np.int32),
            "sampled": np.stack([wl.sampled_tokens(rng, b, 5, z)
                                 for _ in range(steps)])}
    cfg = dict(k=8, max_pattern_len=16, max_occurrences=300, num_backoff=8,
               enable_global=True, global_capacity=1 << 16,
               delta_capacity=1 << 13, max_spec_factor=2.0,
               min_token_prob=0.05)
    g, o = _both(cfg, data, steps=steps, harvest_per_step=1,
                 prefill=list(docs))
    _assert_same(g, o, _LOOP_KEYS + _INDEX_KEYS)
    assert (o["num_valid"] > 0).mean() > 0.5


def test_config3_full_size_loop_vs_oracle():
    """Config 3 at full size: 4096 x 1024 template documents bulk-loaded
    into a 2^22 capacity (which evicts the oldest), then 6 decode steps of
    B = 64 x S = 4096 with 4 harvested rows and a poll each; the delta
    passes the 32768-token threshold every few steps, and each rebuild
    evicts whole documents. Rebuilds are synchronous (no rebuild stream) so
    the swap lands on the same step in both."""
    data = wl.config3(seed=33, steps=6)
    cfg = dict(k=16, max_pattern_len=32, max_occurrences=128, num_backoff=8,
               enable_global=True, global_capacity=1 << 22,
               delta_capacity=1 << 16, rebuild_threshold=32768)
    g, o = _both(cfg, data, steps=6, harvest_per_step=4,
                 prefill=list(data["corpus_docs"]))
    _assert_same(g, o, _LOOP_KEYS + _INDEX_KEYS)
    assert g["rebuilds"] >= 3          # the prefill's two, then the loop's
    assert (o["active_len"] > (1 << 22) - 4096).all()
    assert (o["num_valid"] > 0).mean() > 0.5


def test_config3_loop_with_captured_propose_vs_oracle():
    """The config-3 loop (template corpus, harvested rows, a poll every
    step, synchronous rebuilds that evict and swap in place) with
    propose_with_update captured once into a CUDA graph and replayed on
    every step after the first: drafts, counts, rows and the index equal
    the oracle's eager loop, across every rebuild."""
    from suffixgpu_b200 import SuffixGPUDrafter
    data = wl.config3(seed=34, n_docs=512, doc_len=256, b=16, s=1024,
                      steps=8)
    cfg = dict(k=16, max_pattern_len=32, max_occurrences=128, num_backoff=8,
               enable_global=True, global_capacity=1 << 17,
               delta_capacity=1 << 13, rebuild_threshold=2048)
    prefill = list(data["corpus_docs"])
    g = _run_loop(_Side(SuffixGPUDrafter(device=DEV, **cfg), True), data,
                  8, 4, prefill, graph=True)
    o = _run_loop(_Side(so.SuffixDrafter(**cfg), False), data, 8, 4,
                  prefill)
    _assert_same(g, o, _LOOP_KEYS + _INDEX_KEYS)
    assert g["rebuilds"] >= 4
    assert (o["num_valid"] > 0).mean() > 0.3


def test_config2_all_decode_steps_vs_oracle():
    """All 100 decode steps of config 2 (32 of its 256 rows, S = 8192):
    drafts, counts and buffers bit-exact, including rows whose count runs
    past the buffer end and stop drafting."""
    data = wl.config2(seed=22, steps=100, b=32)
    # four rows start near the buffer end, as config 2's U[2048, 8192]
    # counts do for some of its 256 rows, and overflow within 100 steps
    data["num_tokens"][:4] = [8191, 8100, 8000, 7950]
    cfg = dict(wl.CONFIG2_DRAFTER)
    g, o = _both(cfg, data, steps=100, harvest_per_step=0)
    _assert_same(g, o, _LOOP_KEYS)
    assert (o["new_counts"][-1] > 8192).any()
    assert (o["num_valid"] > 0).mean() > 0.3
