"""Writes the golden fixtures in this folder (run from anywhere: `python tests/golden/make_golden.py`).

gem ships no test vectors of its own, so the fixtures come from two independent implementations run
here on the seeded synthetic models the tests use, plus the oracle's own outputs frozen as a
regression pin:

  gguf_blocks.npz   llama.cpp's Q8_0 / Q4_0 block bytes (gguf-py's quantizer) with gguf-py's
                    dequantization of them: the block formats q8.rs:29-52 reads.
  small_gemma3.npz  the "small" Gemma 3 geometry: sha256 of its GGUF and class files; transformers'
                    Gemma3ForCausalLM log-probs on the same dequantized weights; the oracle's (AVX-512
                    path, 8-thread pool) log-probs and argmax ids for the full and two-level heads,
                    and its final-norm hidden states at a few positions.
  small_qwen2.npz   the same for the qwen2 branch (transformers' Qwen2ForCausalLM).

The oracle part is only written from a host whose CPU has AVX-512 (the path the exact numerics
follow); transformers is used fp32 in eager mode.
"""
from __future__ import annotations

import hashlib
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT / "prefix-head_b200"))
sys.path.insert(0, str(ROOT))

SCORE_TOKENS = (49, 5)     # (count, seed) of the scored sequence
HF_TOKENS = {"small": (41, 11), "small-qwen2": (41, 9)}
HIDDEN_POS = (0, 15, 16, 17, 39, 47)  # first, around the 16-position window, last
REF_THREADS = 8


def sha256(*paths) -> str:
    h = hashlib.sha256()
    for p in paths:
        h.update(Path(p).read_bytes())
    return h.hexdigest()


def blocks():
    import gguf
    from gguf import quants
    rng = np.random.default_rng(3)
    w = (rng.standard_normal((8, 256)) * 0.02).astype(np.float32)
    w[5, :32] = 0.0              # an all-zero block: scale 0
    w[6, 32:64] *= 40.0          # a block whose scale is far from the rest
    out = {"w": w}
    for name in ("Q8_0", "Q4_0"):
        t = getattr(gguf.GGMLQuantizationType, name)
        raw = np.ascontiguousarray(quants.quantize(w, t)).view(np.uint8).reshape(-1)
        out[f"{name}_raw"] = raw
        out[f"{name}_dequant"] = quants.dequantize(raw, t).reshape(w.shape).astype(np.float32)
    np.savez_compressed(HERE / "gguf_blocks.npz", **out)


def hf_logprobs(name, files, toks):
    sys.path.insert(0, str(ROOT / "tests"))
    import test_oracle_vs_transformers as tv
    n = len(toks) - 1
    if name == "small":
        c, build = tv._hf_model(files.cfg, files.gguf)
        return tv._hf_logprobs(build(c), toks, n)
    return tv.qwen2_logprobs(files, toks)


def model(name: str, out: str, classes: int | None, directory: Path):
    from gem_b200 import synth
    from oracle import oracle as orc
    files = synth.ensure(name, classes=classes, directory=directory)
    fx = {"gguf_sha256": sha256(files.gguf)}
    if files.twolevel is not None:
        p = str(files.twolevel)
        fx["twolevel_sha256"] = sha256(p + ".order", p + ".A", p + ".b")
    n, seed = HF_TOKENS[name]
    fx["hf_tokens"] = synth.tokens(n, files.cfg["vocab"], seed=seed)
    fx["hf_lp"] = np.asarray(hf_logprobs(name, files, fx["hf_tokens"]), np.float64)
    if orc.detect_isa() != "avx512":
        raise SystemExit("the oracle's pinned outputs come from its AVX-512 path; this host has none")
    n, seed = SCORE_TOKENS
    toks = synth.tokens(n, files.cfg["vocab"], seed=seed)
    fx["tokens"] = toks
    o = orc.Model(files.gguf, ctx=128, threads=REF_THREADS, isa="avx512")
    heads = [("full", 0)]
    if files.twolevel is not None:
        o.load_twolevel(files.twolevel)
        heads.append(("twolevel", 1))
    for tag, head in heads:
        lp, am, _, _ = o.score(toks, head)
        fx[f"lp_{tag}"], fx[f"am_{tag}"] = lp, am
    o = orc.Model(files.gguf, ctx=128, threads=REF_THREADS, isa="avx512")
    hs = {}
    for i, t in enumerate(toks[:max(HIDDEN_POS) + 1]):
        h = o.forward(int(t), i)
        if i in HIDDEN_POS:
            hs[i] = h
    fx["hidden_pos"] = np.array(HIDDEN_POS, np.int64)
    fx["hidden"] = np.stack([hs[i] for i in HIDDEN_POS])
    np.savez_compressed(HERE / out, **fx)


def main():
    blocks()
    with tempfile.TemporaryDirectory() as d:
        model("small", "small_gemma3.npz", 64, Path(d))
        model("small-qwen2", "small_qwen2.npz", 64, Path(d))
    for p in sorted(HERE.glob("*.npz")):
        print(p.name, p.stat().st_size, "bytes")


if __name__ == "__main__":
    main()
