"""Seeded synthetic models in the formats gem reads.

The reference's GGUF checkpoints, hidden-state dumps and class files are not part of its repository,
so every workload here is generated: random-init Gemma 3 geometries written as real GGUF files
(llama.cpp's own gguf-py writer and quantizers), plus the two-level head's class files in the byte
layout `TwoLevel::load` reads (crates/gem/src/main.rs:57-61: `.order` u32 LE token ids, `.A` f32 LE
k x d row-major, `.b` f32 LE k).

Weights: projections and the embedding are N(0, 0.02), quantized per 32 values (Q8_0: f16 scale
amax/127 and round-half-away int8, as ggml's quantize_row_q8_0; Q4_0: ggml's nibble convention).
Norm weights are 1 + N(0, 0.02): Gemma folds the +1 into its GGUF norm weights, and all-ones weights
would leave the per-element scaling untested. Tokens are uniform ids. Every tensor is drawn from its
own PCG64 stream keyed by (seed, tensor index), so files are identical across machines.
"""
from __future__ import annotations

import dataclasses
import os
from pathlib import Path

import numpy as np

GEMMA3_270M = dict(arch="gemma3", d=640, layers=18, nh=4, nkv=1, hd=256, ff=2048, vocab=262144,
                   window=512, rope_base=1e6, eps=1e-6)
GEMMA3_1B = dict(arch="gemma3", d=1152, layers=26, nh=4, nkv=1, hd=256, ff=6912, vocab=262144,
                 window=512, rope_base=1e6, eps=1e-6)
# Small geometries for tests: same head_dim as the real models, short window so sliding layers slide.
SMALL = dict(arch="gemma3", d=256, layers=6, nh=4, nkv=1, hd=256, ff=512, vocab=8192,
             window=16, rope_base=1e6, eps=1e-6)
SMALL_GQA2 = dict(arch="gemma3", d=512, layers=6, nh=4, nkv=2, hd=128, ff=1024, vocab=4096,
                  window=12, rope_base=1e6, eps=1e-6)
# qwen2 branch (model.rs:160-161, 188-190, 311-315, 400-407): biases on q/k/v, SiLU gate, no norm
# folding or post-norms, untied output matrix; 7 query heads per kv head as Qwen2.5-0.5B (14 / 2).
SMALL_QWEN2 = dict(arch="qwen2", d=256, layers=4, nh=7, nkv=1, hd=32, ff=512, vocab=4096,
                   rope_base=1e6, eps=1e-6, untied=True)
CONFIGS = {"gemma3-270m": GEMMA3_270M, "gemma3-1b": GEMMA3_1B, "small": SMALL, "small-gqa2": SMALL_GQA2,
           "small-qwen2": SMALL_QWEN2}


@dataclasses.dataclass
class ModelFiles:
    gguf: Path
    twolevel: Path | None  # prefix of .order/.A/.b
    cfg: dict


def _rng(seed: int, idx: int) -> np.random.Generator:
    return np.random.default_rng([seed, idx])


def _normal(seed: int, idx: int, shape, std: float) -> np.ndarray:
    return (_rng(seed, idx).standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(np.float32)


def _quant(w: np.ndarray, kind: str):
    import gguf
    from gguf import quants
    if kind == "q8_0":
        return quants.quantize(w, gguf.GGMLQuantizationType.Q8_0), gguf.GGMLQuantizationType.Q8_0
    if kind == "q4_0":
        return quants.quantize(w, gguf.GGMLQuantizationType.Q4_0), gguf.GGMLQuantizationType.Q4_0
    if kind == "f16":
        return w.astype(np.float16), None
    raise ValueError(kind)


def write_model(path: str | os.PathLike, cfg: dict, seed: int = 1, body: str = "q8_0",
                head: str = "q8_0", bos: bool = False, alignment: int | None = None, vocab_strings: bool = False) -> Path:
    """Writes a random-init decoder as GGUF. `head` is the (tied) token_embd.weight type. `alignment`
    sets general.alignment (tensor data offsets padded to it); `vocab_strings` adds a
    tokenizer.ggml.tokens array of `vocab` strings (a header of several MiB for large vocabularies)."""
    import gguf
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    a = cfg["arch"]
    d, nl, nh, nkv, hd, ff, V = (cfg[k] for k in ("d", "layers", "nh", "nkv", "hd", "ff", "vocab"))
    w = gguf.GGUFWriter(str(path), arch=a)
    if alignment:
        w.add_custom_alignment(alignment)
    if vocab_strings:
        w.add_token_list([f"<tok-{i:06d}-{'x' * 24}>" for i in range(V)])
    w.add_uint32(f"{a}.context_length", 32768)
    w.add_uint32(f"{a}.embedding_length", d)
    w.add_uint32(f"{a}.block_count", nl)
    w.add_uint32(f"{a}.feed_forward_length", ff)
    w.add_uint32(f"{a}.attention.head_count", nh)
    w.add_uint32(f"{a}.attention.head_count_kv", nkv)
    w.add_uint32(f"{a}.attention.key_length", hd)
    w.add_uint32(f"{a}.attention.value_length", hd)
    w.add_float32(f"{a}.attention.layer_norm_rms_epsilon", float(cfg["eps"]))
    if cfg.get("window"):
        w.add_uint32(f"{a}.attention.sliding_window", cfg["window"])
    w.add_float32(f"{a}.rope.freq_base", float(cfg["rope_base"]))
    w.add_bool("tokenizer.ggml.add_bos_token", bool(bos))
    w.add_uint32("tokenizer.ggml.bos_token_id", 2)
    w.add_uint32("tokenizer.ggml.eos_token_id", 1)

    idx = 0

    def mat(name, rows, cols, kind):
        nonlocal idx
        idx += 1
        q, dt = _quant(_normal(seed, idx, (rows, cols), 0.02), kind)
        if dt is None:
            w.add_tensor(name, q)
        else:
            w.add_tensor(name, q, raw_dtype=dt)

    def norm(name, n):
        nonlocal idx
        idx += 1
        w.add_tensor(name, (np.float32(1.0) + _normal(seed, idx, (n,), 0.02)).astype(np.float32))

    def bias(name, n):
        nonlocal idx
        idx += 1
        w.add_tensor(name, _normal(seed, idx, (n,), 0.02).astype(np.float32))

    gemma = a == "gemma3"
    mat("token_embd.weight", V, d, head)
    if cfg.get("untied"):
        mat("output.weight", V, d, head)
    norm("output_norm.weight", d)
    for l in range(nl):
        p = f"blk.{l}."
        mat(p + "attn_q.weight", nh * hd, d, body)
        mat(p + "attn_k.weight", nkv * hd, d, body)
        mat(p + "attn_v.weight", nkv * hd, d, body)
        if not gemma:
            bias(p + "attn_q.bias", nh * hd)
            bias(p + "attn_k.bias", nkv * hd)
            bias(p + "attn_v.bias", nkv * hd)
        mat(p + "attn_output.weight", d, nh * hd, body)
        mat(p + "ffn_gate.weight", ff, d, body)
        mat(p + "ffn_up.weight", ff, d, body)
        mat(p + "ffn_down.weight", d, ff, body)
        norm(p + "attn_norm.weight", d)
        norm(p + "ffn_norm.weight", d)
        if gemma:
            norm(p + "attn_q_norm.weight", hd)
            norm(p + "attn_k_norm.weight", hd)
            norm(p + "post_attention_norm.weight", d)
            norm(p + "post_ffw_norm.weight", d)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return path


def write_twolevel(prefix: str | os.PathLike, vocab: int, k: int, d: int, seed: int = 7) -> Path:
    """Class files: a seeded vocab permutation cut into k equal contiguous blocks; A ~ N(0, 0.02); b = 0."""
    prefix = Path(prefix)
    prefix.parent.mkdir(parents=True, exist_ok=True)
    order = _rng(seed, 0).permutation(vocab).astype("<u4")
    A = _normal(seed, 1, (k, d), 0.02).astype("<f4")
    b = np.zeros(k, dtype="<f4")
    order.tofile(str(prefix) + ".order")
    A.tofile(str(prefix) + ".A")
    b.tofile(str(prefix) + ".b")
    return prefix


def tokens(n: int, vocab: int, seed: int = 11) -> np.ndarray:
    """n uniform token ids in [0, vocab)."""
    return _rng(seed, 0).integers(0, vocab, size=n, dtype=np.int64).astype(np.uint32)


def cache_dir() -> Path:
    """Where generated models live: $GEM_CACHE, else ~/.cache/gem-b200 (outside the repository)."""
    d = Path(os.environ.get("GEM_CACHE", Path.home() / ".cache" / "gem-b200"))
    d.mkdir(parents=True, exist_ok=True)
    return d


def ensure(name: str, body: str = "q8_0", head: str = "q8_0", classes: int | None = None, seed: int = 1,
           directory: str | os.PathLike | None = None) -> ModelFiles:
    """Generates (once) the named config and, if `classes` is set, its two-level class files."""
    cfg = CONFIGS[name]
    root = Path(directory) if directory else cache_dir()
    tag = f"{name}-{body}-{head}-s{seed}"
    g = root / f"{tag}.gguf"
    if not g.exists():
        tmp = g.with_suffix(".tmp")
        write_model(tmp, cfg, seed=seed, body=body, head=head)
        tmp.rename(g)
    tl = None
    if classes:
        tl = root / f"{name}-k{classes}-s{seed}"
        if not Path(str(tl) + ".b").exists():
            write_twolevel(tl, cfg["vocab"], classes, cfg["d"], seed=seed + 100)
    return ModelFiles(g, tl, cfg)
