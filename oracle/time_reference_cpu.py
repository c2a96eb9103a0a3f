"""One-time cross-check of the CPU baseline's speed -- TEST INFRASTRUCTURE.

bench.py's CPU baseline and its ``--impl reference`` arm time the numpy
port (oracle/suffix_oracle.py) because the reference (Python) cannot be
shipped to the GPU box. This script ties that number to the reference's
own CPU path: it imports the reference from a local checkout (its
pure-PyTorch fallback, device='cpu'), runs it and the port on the same
config-2 rows and decode steps, checks that both produce the same drafts,
and prints each one's rows/s.

    python oracle/time_reference_cpu.py --reference /path/to/SuffixGPU \
        [--rows 16] [--steps 3] [--threads N]

It needs the reference checkout, so it runs only where one exists (the
build container), never on the GPU box.
"""

from __future__ import annotations

import argparse
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True,
                    help="checkout of the reference project")
    ap.add_argument("--rows", type=int, default=16)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=1)
    ap.add_argument("--threads", type=int, default=os.cpu_count())
    args = ap.parse_args()
    sys.path.insert(0, ROOT)
    sys.path.insert(0, args.reference)
    import torch
    from suffix_gpu.proposer import SuffixGPUDrafter

    from oracle import suffix_oracle as so
    from suffixgpu_b200 import workloads as wl

    torch.set_num_threads(args.threads)
    steps = args.warmup + args.steps
    data = wl.config2(seed=2, steps=steps, b=args.rows)
    cfg = dict(wl.CONFIG2_DRAFTER)

    def run_reference():
        d = SuffixGPUDrafter(device="cpu", **cfg)
        tok = torch.from_numpy(data["token_ids"].copy())
        n = torch.from_numpy(data["num_tokens"].copy())
        outs, t0 = [], None
        for j in range(steps):
            if j == args.warmup:
                t0 = time.perf_counter()
            s = torch.from_numpy(data["sampled"][j].copy())
            dr, nv, n = d.propose_with_update(n, tok, s)
            outs.append((dr.numpy().copy(), nv.numpy().copy()))
        return time.perf_counter() - t0, outs

    def run_port():
        d = so.SuffixDrafter(**cfg)
        tok, n = data["token_ids"].copy(), data["num_tokens"].copy()
        outs, t0 = [], None
        for j in range(steps):
            if j == args.warmup:
                t0 = time.perf_counter()
            dr, nv, n = d.propose_with_update(n, tok, data["sampled"][j])
            outs.append((dr.copy(), nv.copy()))
        return time.perf_counter() - t0, outs

    t_ref, o_ref = run_reference()
    t_port, o_port = run_port()
    for (a, b), (c, e) in zip(o_ref, o_port):
        np.testing.assert_array_equal(a, c)
        np.testing.assert_array_equal(b, e)
    rows = args.rows * args.steps
    print(f"config 2, {args.rows} rows x {args.steps} timed steps "
          f"({args.warmup} warm-up), identical drafts")
    print(f"reference torch CPU path ({args.threads} threads): "
          f"{t_ref / args.steps * 1e3:.1f} ms/step, {rows / t_ref:.1f} rows/s")
    print(f"numpy port (1 process): {t_port / args.steps * 1e3:.1f} ms/step, "
          f"{rows / t_port:.1f} rows/s")
    print(f"port / reference speed: {t_ref / t_port:.2f}")


if __name__ == "__main__":
    main()
