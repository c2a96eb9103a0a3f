"""Deterministic drafter scenarios shared by the golden-vector generator
(which runs them on the reference) and the parity tests (which run them on
the oracle and on the CUDA path).

A scenario is a drafter configuration plus a list of operations over host
numpy arrays. ``run_scenario`` drives any object exposing the reference
drafter API through a small adapter, so the same script produces the
reference's goldens, the oracle's outputs and the GPU outputs.
"""

from __future__ import annotations

import numpy as np

from suffixgpu_b200 import workloads as wl


def local_scenario(seed: int, b: int, s: int, steps: int, vocab: int,
                   p_copy: float, span, q_range, drafter: dict) -> dict:
    data = wl.local_config(seed, b=b, s=s, vocab=vocab, p_copy=p_copy,
                           span=span, q_range=q_range, steps=steps)
    ops = [("pwu", i) for i in range(steps)]
    return {"drafter": drafter, "data": data, "ops": ops}


def global_scenario(seed: int, steps: int = 10) -> dict:
    """Small config-3-like run: template corpus harvested step by step with
    frequent synchronous rebuilds, delta overflow and eviction."""
    rng = np.random.default_rng(seed)
    z = wl.Zipf(1.1, 500)
    templates = z.draw(rng, (12, 40))
    docs = wl.template_docs(rng, 48, 120, templates, z)
    b, s = 6, 512
    rows = wl.template_docs(rng, b, s, templates, z)
    q = rng.integers(200, 400, size=b).astype(np.int32)
    sampled = np.stack([wl.sampled_tokens(rng, b, 5, z)
                        for _ in range(steps)])
    drafter = dict(k=8, max_pattern_len=16, max_occurrences=32,
                   enable_global=True, global_capacity=2048,
                   delta_capacity=512, rebuild_threshold=300,
                   max_spec_factor=2.0, max_spec_offset=0.5,
                   min_token_prob=0.05, num_backoff=8)
    ops = []
    d = 0
    for i in range(steps):
        n_h = 2 + (i % 3)
        ops.append(("harvest", list(range(d, d + n_h))))
        d += n_h
        ops.append(("poll", None))
        ops.append(("pwu", i))
    data = {"token_ids": rows, "num_tokens": q, "sampled": sampled,
            "docs": docs}
    return {"drafter": drafter, "data": data, "ops": ops}


def run_scenario(sc: dict, make_drafter, to_dev, to_host) -> dict:
    """Run ``sc`` on a drafter built by ``make_drafter(**cfg)``.

    ``to_dev`` turns a numpy array into the drafter's tensor type,
    ``to_host`` back. Returns per-step draft/num_valid/new_counts plus the
    final token buffer (and global-index state when enabled).
    """
    data = sc["data"]
    d = make_drafter(**sc["drafter"])
    tok = to_dev(data["token_ids"].copy())
    n = to_dev(data["num_tokens"].copy())
    out = {"draft": [], "num_valid": [], "new_counts": []}
    docs = data.get("docs")
    for op, arg in sc["ops"]:
        if op == "pwu":
            sampled = to_dev(data["sampled"][arg].copy())
            draft, nv, n = d.propose_with_update(n, tok, sampled)
            out["draft"].append(to_host(draft))
            out["num_valid"].append(to_host(nv))
            out["new_counts"].append(to_host(n))
        elif op == "harvest":
            rows = [to_dev(docs[j].copy()) for j in arg]
            lens = [int(docs[j].shape[0]) for j in arg]
            d.harvest_rows(rows, lens)
        elif op == "poll":
            d.poll()
    res = {k: np.stack(v) for k, v in out.items() if v}
    res["final_tokens"] = to_host(tok)
    gi = getattr(d, "global_index", None)
    if gi is not None:
        res["active_len"] = np.array(gi.active_len)
        res["delta_len"] = np.array(gi.delta_len)
        res["corpus"] = to_host(gi.corpus)
        res["sa"] = to_host(gi.sa)
    return res


def local_scenarios() -> dict:
    """Named local-only scenarios used for goldens and parity tests."""
    return {
        "cfg1": local_scenario(
            11, b=8, s=2048, steps=3, vocab=32000, p_copy=0.5, span=(8, 64),
            q_range=(512, 2040),
            drafter=dict(k=16, max_pattern_len=32, max_occurrences=128,
                         num_backoff=8)),
        "cfg2s": local_scenario(
            12, b=8, s=8192, steps=3, vocab=128256, p_copy=0.7,
            span=(16, 256), q_range=(2048, 8192),
            drafter=dict(wl.CONFIG2_DRAFTER)),
        "tiny": local_scenario(
            13, b=16, s=96, steps=4, vocab=5, p_copy=0.4, span=(3, 12),
            q_range=(1, 92),
            drafter=dict(k=6, max_pattern_len=8, max_occurrences=8,
                         num_backoff=5, max_spec_factor=1.5,
                         max_spec_offset=1.0, min_token_prob=0.2,
                         vote_smoothing_alpha=0.5)),
        "overflow": local_scenario(
            14, b=12, s=64, steps=6, vocab=6, p_copy=0.5, span=(4, 16),
            q_range=(50, 64),
            drafter=dict(k=4, max_pattern_len=6, max_occurrences=16,
                         num_backoff=3)),
    }
