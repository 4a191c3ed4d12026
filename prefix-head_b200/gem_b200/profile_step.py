"""Runs a few scoring calls of a synthetic workload, for profilers (ncu) to capture:

  PYTHONPATH=prefix-head_b200 python -m gem_b200.profile_step [--model gemma3-270m] [--tokens 512]
      [--calls 2] [--head two-level|full] [--schedule auto|sequential|pipelined|parallel] [--seqs 1]

Prints the mean log-prob and the kernels launched per call, so a plain run (without the profiler)
also checks that the workload ran."""
from __future__ import annotations

import argparse

import numpy as np

from . import AUTO, FULL, PARALLEL, PIPELINED, SEQUENTIAL, TWO_LEVEL, Gemma, synth


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--model", default="gemma3-270m", choices=sorted(synth.CONFIGS))
    p.add_argument("--tokens", type=int, default=512)
    p.add_argument("--calls", type=int, default=2)
    p.add_argument("--head", default="two-level", choices=["two-level", "full"])
    p.add_argument("--schedule", default="auto", choices=["auto", "sequential", "pipelined", "parallel"])
    p.add_argument("--seqs", type=int, default=1, help="> 1: batched scoring of this many sequences")
    a = p.parse_args(argv)
    mf = synth.ensure(a.model, classes=2048 if a.model.startswith("gemma3") else 64)
    g = Gemma(mf.gguf, ctx=max(2048, a.tokens + 1), max_seqs=min(a.seqs, 8))
    g.load_twolevel(mf.twolevel)
    g.set_schedule({"auto": AUTO, "sequential": SEQUENTIAL, "pipelined": PIPELINED, "parallel": PARALLEL}[a.schedule])
    head = TWO_LEVEL if a.head == "two-level" else FULL
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
