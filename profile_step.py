"""Runs a few scoring calls of a synthetic workload, for profilers (ncu) to capture:

  python profile_step.py [--model gemma3-270m] [--tokens 512]
      [--calls 2] [--head two-level|full] [--schedule auto|sequential|pipelined|parallel] [--seqs 1]
      [--head-batch N]

Prints the mean log-prob and the kernels launched per call, so a plain run (without the profiler)
also checks that the workload ran. --head-batch N runs only the head: N hidden states drawn from
N(0, 1) through gem_head_full_dev or gem_head_twolevel_dev, `calls` times."""
from __future__ import annotations

import argparse
import sys
from pathlib import Path

import numpy as np

sys.path.insert(0, str(Path(__file__).resolve().parent / "prefix-head_b200"))
from gem_b200 import AUTO, FULL, PARALLEL, PIPELINED, SEQUENTIAL, TWO_LEVEL, Gemma, synth  # noqa: E402


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--model", default="gemma3-270m", choices=sorted(synth.CONFIGS))
    p.add_argument("--tokens", type=int, default=512)
    p.add_argument("--calls", type=int, default=2)
    p.add_argument("--head", default="two-level", choices=["two-level", "full"])
    p.add_argument("--schedule", default="auto", choices=["auto", "sequential", "pipelined", "parallel"])
    p.add_argument("--seqs", type=int, default=1, help="> 1: batched scoring of this many sequences")
    p.add_argument("--head-batch", type=int, default=0, help="> 0: only the head, for this many hidden states")
    a = p.parse_args(argv)
    mf = synth.ensure(a.model, classes=2048 if a.model.startswith("gemma3") else 64)
    g = Gemma(mf.gguf, ctx=max(2048, a.tokens + 1), max_seqs=min(a.seqs, 8))
    g.load_twolevel(mf.twolevel)
    g.set_schedule({"auto": AUTO, "sequential": SEQUENTIAL, "pipelined": PIPELINED, "parallel": PARALLEL}[a.schedule])
    head = TWO_LEVEL if a.head == "two-level" else FULL
    if a.head_batch > 0:
        import torch
        rng = np.random.default_rng(9)
        n = a.head_batch
        hs = torch.tensor(rng.standard_normal((n, g.d)).astype(np.float32), device="cuda")
        ts = torch.tensor(rng.integers(0, g.vocab, n).astype(np.int32), device="cuda")
        lp_d = torch.empty(n, device="cuda")
        am_d = torch.empty(n, dtype=torch.int32, device="cuda")
        fn = g.head_full_dev if head == FULL else g.head_twolevel_dev
        for _ in range(a.calls):
            fn(hs.data_ptr(), ts.data_ptr(), n, lp_d.data_ptr(), am_d.data_ptr())
        print(f"ok head {a.head} batch {n} mean_logprob {float(lp_d.mean()):.6f}")
        return
    if a.seqs > 1:
        toks = np.stack([synth.tokens(a.tokens + 1, g.vocab, seed=1000 + s) for s in range(a.seqs)])
        for _ in range(a.calls):
            lp, _ = g.score_batch(toks, head)
    else:
        toks = synth.tokens(a.tokens + 1, g.vocab, seed=1000)
        for _ in range(a.calls):
            lp, _ = g.score(toks, head)
    print(f"ok mean_logprob {float(np.mean(lp)):.6f} launches_per_call {g.last_launches()}")


if __name__ == "__main__":
    main()
