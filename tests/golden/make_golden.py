"""Generate the golden vectors that pin the oracle (and the CUDA path).

Runs the reference project's own pure-PyTorch CPU path (zip95297/SuffixGPU,
imported from the local checkout given by --ref) on seeded inputs and
writes compressed ``.npz`` fixtures next to this file. The reference is
never needed at test time: the fixtures are committed.

Usage: python tests/golden/make_golden.py --ref PATH_TO_REFERENCE_CHECKOUT
"""

from __future__ import annotations

import argparse
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, HERE)

import scenarios  # noqa: E402
from suffixgpu_b200 import workloads as wl  # noqa: E402


def _save(name: str, **arrays) -> None:
    path = os.path.join(HERE, name)
    np.savez_compressed(path, **arrays)
    print(f"wrote {path} ({os.path.getsize(path)} bytes)")


def expand_cases(torch, ref_expand) -> None:
    """Random continuation blocks with monotone -1 tails, fully padded
    rows, caps, cutoffs and smoothing."""
    out = {}
    i = 0
    for r in (4, 32, 128, 256):
        for minp in (0.0, 0.1):
            for alpha in (0.0, 0.5):
                g = torch.Generator().manual_seed(1000 + r + i)
                b, k = 33, 16
                cont = torch.randint(0, 9, (b, r, k), dtype=torch.int32,
                                     generator=g)
                tail = torch.randint(0, k + 1, (b, r), generator=g)
                idx = torch.arange(k).view(1, 1, k)
                cont = torch.where(idx < tail.unsqueeze(2), cont, -1)
                occ = torch.randint(0, r + 1, (b,), dtype=torch.int64,
                                    generator=g)
                cap = torch.randint(0, k + 1, (b,), dtype=torch.int64,
                                    generator=g)
                chain, nv, ne, sc = ref_expand(cont, occ, k,
                                               min_token_prob=minp,
                                               cap=cap, alpha=alpha)
                p = f"c{i}_"
                out[p + "cont"] = cont.numpy()
                out[p + "occ"] = occ.numpy()
                out[p + "cap"] = cap.numpy()
                out[p + "meta"] = np.array([r, k], dtype=np.int64)
                out[p + "minp"] = np.array(minp, dtype=np.float64)
                out[p + "alpha"] = np.array(alpha, dtype=np.float64)
                out[p + "chain"] = chain.numpy()
                out[p + "nv"] = nv.numpy()
                out[p + "emit"] = ne.numpy()
                out[p + "score"] = sc.numpy()
                i += 1
    out["n"] = np.array(i)
    _save("expand_cases.npz", **out)


def local_cases(torch, Drafter) -> None:
    def mk(**cfg):
        return Drafter(device="cpu", **cfg)

    def to_dev(a):
        return torch.from_numpy(a)

    def to_host(t):
        return t.numpy().copy()

    scs = scenarios.local_scenarios()
    for name, sc in scs.items():
        res = scenarios.run_scenario(sc, mk, to_dev, to_host)
        arrays = {f"in_{k}": v for k, v in sc["data"].items()}
        arrays.update({f"out_{k}": v for k, v in res.items()})
        _save(f"local_{name}.npz", **arrays)


def sa_cases(torch, build) -> None:
    out = {}
    i = 0
    rng = np.random.default_rng(21)
    seqs = [[0], [2, 1], [5, 5, 5, 5, 5], [1, 2, 1, 2, 1, 2, 1],
            [-2, 3, -2, 3, 2147483647, 2147483647, 0, -1]]
    for n, v in ((31, 3), (64, 8), (200, 16), (7, 2), (1000, 2),
                 (4096, 50)):
        seqs.append(rng.integers(0, v, size=n).tolist())
    z = wl.Zipf(1.1, 128256)
    seqs.append(wl.copy_stream(rng, 1 << 15, z, 0.5, 32, 1024,
                               fresh_len=(32, 1024)).tolist())
    for s in seqs:
        t = torch.tensor(s, dtype=torch.int32)
        sa = build(t)
        out[f"t{i}"] = np.array(s, dtype=np.int32)
        out[f"sa{i}"] = sa.numpy()
        i += 1
    out["n"] = np.array(i)
    _save("sa_cases.npz", **out)


def sa_search_cases(torch, build, search_interval, backoff) -> None:
    rng = np.random.default_rng(31)
    out = {}
    corpus = rng.integers(0, 4, size=300).astype(np.int32)
    sa = build(torch.from_numpy(corpus)).to(torch.int32)
    pats, plens = [], []
    for _ in range(64):
        m = int(rng.integers(1, 9))
        if rng.random() < 0.7:
            st = int(rng.integers(0, 300 - m))
            p = corpus[st:st + m].tolist()
        else:
            p = rng.integers(0, 5, size=m).tolist()
        pats.append(p + [0] * (8 - m))
        plens.append(m)
    pat = torch.tensor(pats, dtype=torch.int32)
    plen = torch.tensor(plens, dtype=torch.int64)
    s, e = search_interval(sa, torch.from_numpy(corpus), pat, plen)
    out.update(corpus=corpus, sa=sa.numpy(), pat=pat.numpy(),
               plen=plen.numpy(), start=s.numpy(), end=e.numpy())
    # backoff over lengths 1..M with caps
    q = rng.integers(0, 4, size=(16, 12)).astype(np.int32)
    for i in range(0, 16, 2):
        st = int(rng.integers(0, 280))
        q[i] = corpus[st:st + 12]
    qlen = rng.integers(0, 13, size=16).astype(np.int64)
    caps = torch.tensor([12, 6, 3, 2], dtype=torch.int64)
    ml, bs, be = backoff(sa, torch.from_numpy(corpus), torch.from_numpy(q),
                         torch.from_numpy(qlen), 12, caps)
    out.update(q=q, qlen=qlen, caps=caps.numpy(), b_len=ml.numpy(),
               b_start=bs.numpy(), b_end=be.numpy())
    _save("sa_search_cases.npz", **out)


def global_cases(torch, Drafter) -> None:
    def mk(**cfg):
        return Drafter(device="cpu", **cfg)

    def to_dev(a):
        return torch.from_numpy(a)

    def to_host(t):
        return t.numpy().copy()

    for seed in (41, 42):
        sc = scenarios.global_scenario(seed)
        res = scenarios.run_scenario(sc, mk, to_dev, to_host)
        arrays = {f"in_{k}": v for k, v in sc["data"].items()}
        arrays.update({f"out_{k}": v for k, v in res.items()})
        _save(f"global_{seed}.npz", **arrays)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True,
                    help="checkout of the reference project")
    args = ap.parse_args()
    sys.path.insert(0, args.ref)
    import torch
    torch.manual_seed(0)
    from suffix_gpu.expand import expand_chain
    from suffix_gpu.proposer import SuffixGPUDrafter
    from suffix_gpu.sa_search import search_interval, suffix_match_backoff
    from suffix_gpu.suffix_array import build_suffix_array
    expand_cases(torch, expand_chain)
    local_cases(torch, SuffixGPUDrafter)
    sa_cases(torch, build_suffix_array)
    sa_search_cases(torch, build_suffix_array, search_interval,
                    suffix_match_backoff)
    global_cases(torch, SuffixGPUDrafter)


if __name__ == "__main__":
    main()
