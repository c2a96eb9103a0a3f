"""Pin the numpy oracle against golden vectors produced by the reference's
own torch CPU path (tests/golden/make_golden.py). CPU only."""

from __future__ import annotations

import os

import numpy as np
import pytest

import scenarios
from oracle import suffix_oracle as so


def _load(golden_dir, name):
    return np.load(os.path.join(golden_dir, name))


def test_expand_matches_reference(golden_dir):
    z = _load(golden_dir, "expand_cases.npz")
    for i in range(int(z["n"])):
        p = f"c{i}_"
        r, k = z[p + "meta"].tolist()
        chain, nv, ne, sc = so.expand_chain(
            z[p + "cont"], z[p + "occ"], int(k),
            min_token_prob=float(z[p + "minp"]), cap=z[p + "cap"],
            alpha=float(z[p + "alpha"]))
        np.testing.assert_array_equal(chain, z[p + "chain"], f"case {i}")
        np.testing.assert_array_equal(nv, z[p + "nv"])
        np.testing.assert_array_equal(ne, z[p + "emit"])
        # bit-exact fp32 scores
        np.testing.assert_array_equal(sc.view(np.int32),
                                      z[p + "score"].view(np.int32))


def _oracle_drafter(**cfg):
    return so.SuffixDrafter(**cfg)


def _ident(a):
    return np.asarray(a).copy()


@pytest.mark.parametrize("name", ["cfg1", "cfg2s", "tiny", "overflow"])
def test_local_scenarios_match_reference(golden_dir, name):
    z = _load(golden_dir, f"local_{name}.npz")
    sc = scenarios.local_scenarios()[name]
    for k in sc["data"]:
        np.testing.assert_array_equal(sc["data"][k], z["in_" + k])
    res = scenarios.run_scenario(sc, _oracle_drafter, _ident, _ident)
    for key in ("draft", "num_valid", "new_counts", "final_tokens"):
        np.testing.assert_array_equal(res[key], z["out_" + key], key)


def test_suffix_array_matches_reference(golden_dir):
    z = _load(golden_dir, "sa_cases.npz")
    for i in range(int(z["n"])):
        sa = so.build_suffix_array(z[f"t{i}"])
        np.testing.assert_array_equal(sa, z[f"sa{i}"], f"case {i}")
        # the early exit is a fixpoint of the reference's full rounds
        if z[f"t{i}"].shape[0] <= 4096:
            sa_full = so.build_suffix_array(z[f"t{i}"], early_exit=False)
            np.testing.assert_array_equal(sa_full, z[f"sa{i}"])


def test_sa_search_matches_reference(golden_dir):
    z = _load(golden_dir, "sa_search_cases.npz")
    s, e = so.search_interval(z["sa"], z["corpus"], z["pat"], z["plen"])
    np.testing.assert_array_equal(s, z["start"])
    np.testing.assert_array_equal(e, z["end"])
    ml, bs, be = so.suffix_match_backoff(z["sa"], z["corpus"], z["q"],
                                         z["qlen"], 12, z["caps"])
    np.testing.assert_array_equal(ml, z["b_len"])
    np.testing.assert_array_equal(bs, z["b_start"])
    np.testing.assert_array_equal(be, z["b_end"])


@pytest.mark.parametrize("seed", [41, 42])
def test_global_scenarios_match_reference(golden_dir, seed):
    z = _load(golden_dir, f"global_{seed}.npz")
    sc = scenarios.global_scenario(seed)
    for k in sc["data"]:
        np.testing.assert_array_equal(sc["data"][k], z["in_" + k])
    res = scenarios.run_scenario(sc, _oracle_drafter, _ident, _ident)
    for key in ("draft", "num_valid", "new_counts", "final_tokens",
                "active_len", "delta_len", "corpus", "sa"):
        np.testing.assert_array_equal(res[key], z["out_" + key], key)
